// On-device sampling head: suppress / repetition penalty / top-k / temperature /
// Gumbel-max / counts update, one CTA per row.
//
// Talker (talker_unified_modules.py:373-388): ids [V-1024, V) except EOS are
// set to -1e9; where token_counts > 0 a logit g becomes g/penalty if g > 0
// else g*penalty; the top-k values (descending) are divided by the
// temperature, the j-th gets gumbel[j] added, the argmax picks the token and
// token_counts[token] += 1.  Code predictor (utils.py:986-1001): the same
// without suppress, penalty and counts.
//
// Top-k: a 4-pass 8-bit radix select on order-preserving integer keys finds
// the k-th largest key; the candidates (>= that key) are sorted by
// (value desc, index asc) in one warp, which fixes the rank each Gumbel
// sample is added to.  Noise, when not supplied, is Philox4x32-10
// (Salmon et al., SC'11) keyed by (seed, per-stream key, step, rank) and
// mapped to -log(-log(u)) with u clamped to [1e-8, 1] as
// engine/backend/executor.py:1238-1251 does.
#pragma once

#include "common.cuh"
#include "small_ops.cuh"

namespace qtts {

struct SampleParams {
    const float* logits;
    int R, V, ld, topk;
    const float* gumbel;
    int gumbel_ld;
    uint64_t seed;
    const int64_t* noise_key;   // per counts-row key (NULL: row index)
    const int32_t* noise_step;  // per counts-row frame counter (NULL: 0); counter = 16*frame + step
    int step;
    const float* temperature;
    const float* penalty;
    int64_t* counts;
    const int32_t* counts_row;  // counts row of batch row r (NULL: r)
    int eos_id;
    int64_t* tok_out;
    int tok_ld;
    // code predictor: after sampling, the CTA of row r also writes the next stage's input,
    // embed_projected_row(table, next_ids[r * next_ld]) (table null: off)
    const float* next_table;
    int next_V, next_H;
    const int64_t* next_ids;  // the sampled token's slot, or a forced code
    int next_ld;
    const __nv_bfloat16* next_gamma;
    float* next_x;
    __nv_bfloat16* next_xn;
    __nv_bfloat16* next_xn_lo;
    float* next_ss;
};

__device__ __forceinline__ uint32_t float_key(float f) {
    const uint32_t b = __float_as_uint(f);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

// Philox4x32 with 10 rounds; constants from the published algorithm.
__device__ __forceinline__ uint4 philox4x32_10(uint4 c, uint2 k) {
    const uint32_t M0 = 0xD2511F53u, M1 = 0xCD9E8D57u, W0 = 0x9E3779B9u, W1 = 0xBB67AE85u;
#pragma unroll
    for (int i = 0; i < 10; ++i) {
        const uint32_t hi0 = __umulhi(M0, c.x), lo0 = M0 * c.x;
        const uint32_t hi1 = __umulhi(M1, c.z), lo1 = M1 * c.z;
        c = make_uint4(hi1 ^ c.y ^ k.x, lo1, hi0 ^ c.w ^ k.y, lo0);
        k.x += W0;
        k.y += W1;
    }
    return c;
}

__device__ __forceinline__ float gumbel_noise(uint64_t seed, uint64_t key, int step, int j) {
    const uint4 ctr = make_uint4((uint32_t)j, (uint32_t)step, (uint32_t)key, (uint32_t)(key >> 32));
    const uint4 r = philox4x32_10(ctr, make_uint2((uint32_t)seed, (uint32_t)(seed >> 32)));
    float u = ((float)r.x + 0.5f) * 2.3283064365386963e-10f;  // (0, 1)
    u = fminf(fmaxf(u, 1e-8f), 1.0f);
    return -logf(-logf(u));
}

constexpr int kSampleThreads = 256;
constexpr int kSampleMaxPer = 16;   // V <= 4096
constexpr int kSampleCand = 128;    // candidate buffer (>= topk, room for ties)

__global__ void __launch_bounds__(kSampleThreads) sample_kernel(const SampleParams p) {
    __shared__ uint32_t hist[256];
    __shared__ uint32_t s_prefix, s_need;
    __shared__ int s_stop;
    __shared__ int s_ncand;
    __shared__ float c_val[kSampleCand];
    __shared__ float s_noise[64];  // Gumbel noise of ranks 0..topk-1
    __shared__ int c_idx[kSampleCand];

    const int r = blockIdx.x, tid = threadIdx.x;
    griddep_wait();
    griddep_launch();
    const float* lg = p.logits + (size_t)r * p.ld;
    const int crow = p.counts_row ? p.counts_row[r] : r;  // per-stream state row (slot)
    const float pen = p.penalty ? p.penalty[crow] : 1.0f;
    const float temp = p.temperature ? p.temperature[crow] : 1.0f;
    int64_t* cnt_rw = p.counts ? p.counts + (size_t)crow * p.V : nullptr;
    const int64_t* cnt = cnt_rw;

    float val[kSampleMaxPer];
    uint32_t key[kSampleMaxPer];
#pragma unroll
    for (int i = 0; i < kSampleMaxPer; ++i) {
        const int idx = tid + i * kSampleThreads;
        float g = -INFINITY;
        if (idx < p.V) {
            g = lg[idx];
            if (cnt) {
                if (idx >= p.V - 1024 && idx != p.eos_id) g = -1e9f;
                if (cnt[idx] > 0) g = g > 0.f ? g / pen : g * pen;
            }
        }
        val[i] = g;
        key[i] = idx < p.V ? float_key(g) : 0u;  // padding sorts below every real value
    }

    // radix select of the topk-th largest key; stops early once every key at or above the
    // bucket holding it fits the candidate buffer (the sort below then orders them all)
    uint32_t prefix = 0, mask = 0;
    uint32_t need = (uint32_t)p.topk;
    bool early = false;
    for (int shift = 24; shift >= 0; shift -= 8) {
        for (int i = tid; i < 256; i += kSampleThreads) hist[i] = 0;
        __syncthreads();
#pragma unroll
        for (int i = 0; i < kSampleMaxPer; ++i) {
            // plain shared atomics: measured faster than aggregating equal bins with
            // __match_any_sync (9.3 vs 11.3 us per 64-row launch)
            const int idx = tid + i * kSampleThreads;
            if (idx < p.V && (key[i] & mask) == prefix) atomicAdd(&hist[(key[i] >> shift) & 255u], 1u);
        }
        __syncthreads();
        if (tid < 32) {
            // warp scan from the top bin down: lane l owns bins 255-8l .. 248-8l
            const int lane = tid;
            uint32_t c[8], tot = 0;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                c[j] = hist[255 - 8 * lane - j];
                tot += c[j];
            }
            uint32_t incl = tot;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const uint32_t nb = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o) incl += nb;
            }
            const uint32_t excl = incl - tot;
            const unsigned hit = __ballot_sync(0xffffffffu, excl < need && need <= incl);
            const int src = hit ? __ffs(hit) - 1 : 31;
            if (lane == src) {
                uint32_t above = excl;
                int b = 255 - 8 * lane;
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    b = 255 - 8 * lane - j;
                    if (above + c[j] >= need || b == 0) break;
                    above += c[j];
                }
                s_prefix = prefix | ((uint32_t)b << shift);
                s_need = need - above;
                // keys above the bucket + the bucket itself
                const uint32_t bucket = hist[b];
                s_stop = shift > 0 && (uint32_t)p.topk - (need - above) + bucket <= (uint32_t)kSampleCand;
            }
        }
        __syncthreads();
        prefix = s_prefix;
        need = s_need;
        mask |= 255u << shift;
        early = s_stop != 0;
        __syncthreads();
        if (early) break;
    }
    // gather candidates.  Early stop: every key whose high bits reach the bucket (at most
    // kSampleCand; the sort orders them and the first topk are exactly the top-k with ties
    // broken by index).  Otherwise every key > the k-th key (fewer than topk), then the
    // lowest-index keys equal to it until topk are taken, in index order, so the selection is
    // deterministic when values tie.
    if (tid == 0) s_ncand = 0;
    __syncthreads();
    {
        // one shared atomic per warp and round: the lanes' slots follow from the ballot
        const int lane = tid & 31;
#pragma unroll
        for (int i = 0; i < kSampleMaxPer; ++i) {
            const int idx = tid + i * kSampleThreads;
            const bool c = idx < p.V && (early ? key[i] >= prefix : key[i] > prefix);
            const unsigned b = __ballot_sync(0xffffffffu, c);
            int base = 0;
            if (lane == 0 && b) base = atomicAdd(&s_ncand, __popc(b));
            base = __shfl_sync(0xffffffffu, base, 0);
            if (c) {
                const int slot = base + __popc(b & ((1u << lane) - 1u));
                c_val[slot] = val[i];
                c_idx[slot] = idx;
            }
        }
    }
    __syncthreads();
    if (!early) {
        __shared__ int s_wcnt[kSampleThreads / 32];
        const int lane = tid & 31, wid = tid >> 5;
        int base = s_ncand;
#pragma unroll 1
        for (int i = 0; i < kSampleMaxPer && base < p.topk; ++i) {
            const int idx = tid + i * kSampleThreads;  // indices of round i are consecutive across threads
            const bool tie = idx < p.V && key[i] == prefix;
            const unsigned b = __ballot_sync(0xffffffffu, tie);
            if (lane == 0) s_wcnt[wid] = __popc(b);
            __syncthreads();
            int off = 0, total = 0;
            for (int w = 0; w < kSampleThreads / 32; ++w) {
                off += w < wid ? s_wcnt[w] : 0;
                total += s_wcnt[w];
            }
            const int pos = base + off + __popc(b & ((1u << lane) - 1u));
            if (tie && pos < p.topk) {
                c_val[pos] = val[i];
                c_idx[pos] = idx;
            }
            base += total;
            __syncthreads();
        }
        if (tid == 0) s_ncand = min(base, p.topk);
    }
    __syncthreads();
    if (tid >= 32 && tid < 64) {
        // the noise of rank j does not depend on the sort: warp 1 makes it while warp 0 sorts
        const int lane = tid - 32;
        const uint64_t nkey = p.noise_key ? (uint64_t)p.noise_key[crow] : (uint64_t)crow;
        const int nstep = (p.noise_step ? p.noise_step[crow] * 16 : 0) + p.step;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int j = lane + 32 * h;
            if (j < p.topk)
                s_noise[j] = p.gumbel ? p.gumbel[(size_t)r * p.gumbel_ld + j] : gumbel_noise(p.seed, nkey, nstep, j);
        }
    }
    if (tid < 32) {
        const int n = min(s_ncand, kSampleCand);
        // bitonic sort of 128 entries by (value desc, index asc) in registers: lane l holds
        // positions 4l..4l+3; partners 4 or more positions apart are exchanged by shuffles
        float v[4];
        int ix[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const int e = tid * 4 + k;
            v[k] = e < n ? c_val[e] : -INFINITY;
            ix[k] = e < n ? c_idx[e] : 0x7fffffff;
        }
#pragma unroll
        for (int size = 2; size <= kSampleCand; size <<= 1) {
#pragma unroll
            for (int j = size >> 1; j > 0; j >>= 1) {
                if (j >= 4) {
                    const int lm = j >> 2;  // partner lane = tid ^ lm, same register
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        const float pv = __shfl_xor_sync(0xffffffffu, v[k], lm);
                        const int pi = __shfl_xor_sync(0xffffffffu, ix[k], lm);
                        const int pos = tid * 4 + k;
                        const bool up = (pos & size) == 0;
                        const bool lower = (pos & j) == 0;
                        const bool me_first = (v[k] > pv) || (v[k] == pv && ix[k] < pi);
                        const bool keep = (lower == up) ? me_first : !me_first;
                        if (!keep) {
                            v[k] = pv;
                            ix[k] = pi;
                        }
                    }
                } else {
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        const int k2 = k ^ j;
                        if (k2 > k) {
                            const bool up = ((tid * 4 + k) & size) == 0;
                            const bool a_first = (v[k] > v[k2]) || (v[k] == v[k2] && ix[k] < ix[k2]);
                            if (up != a_first) {
                                const float tv = v[k];
                                v[k] = v[k2];
                                v[k2] = tv;
                                const int ti = ix[k];
                                ix[k] = ix[k2];
                                ix[k2] = ti;
                            }
                        }
                    }
                }
            }
        }
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            c_val[tid * 4 + k] = v[k];
            c_idx[tid * 4 + k] = ix[k];
        }
    }
    __syncthreads();  // sorted candidates (warp 0) and noise (warp 1)
    if (tid < 32) {
        // Gumbel-max over the first topk ranks
        float best = -INFINITY;
        int best_j = 0x7fffffff;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int j = tid + 32 * h;
            if (j >= p.topk) break;
            const float sc = c_val[j] / temp + s_noise[j];
            if (sc > best || (sc == best && j < best_j)) {
                best = sc;
                best_j = j;
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ob = __shfl_xor_sync(0xffffffffu, best, o);
            const int oj = __shfl_xor_sync(0xffffffffu, best_j, o);
            if (ob > best || (ob == best && oj < best_j)) {
                best = ob;
                best_j = oj;
            }
        }
        if (tid == 0) {
            const int tok = c_idx[best_j];
            p.tok_out[(size_t)r * p.tok_ld] = tok;
            if (cnt_rw) cnt_rw[tok] += 1;
        }
    }
    if (p.next_table) {
        __syncthreads();  // thread 0's token store is visible to the block
        embed_projected_row(p.next_table, p.next_V, p.next_H, p.next_ids[(size_t)r * p.next_ld], p.next_gamma,
                            p.next_x, p.next_xn, p.next_xn_lo, p.next_ss, r);
    }
}

// The Gumbel noise the samplers draw when it is not supplied: out[r][j] =
// gumbel_noise(seed, keys[r], 16 * frames[r] + stage, j), stage 0 = the talker
// head, 1 + s = code-predictor stage s (the counter layout of sample_kernel).
__global__ void philox_gumbel_kernel(uint64_t seed, const int64_t* keys, const int32_t* frames, int stage, int cols,
                                     float* out) {
    const int r = blockIdx.x;
    const uint64_t key = (uint64_t)keys[r];
    const int step = frames[r] * 16 + stage;
    for (int j = threadIdx.x; j < cols; j += blockDim.x) out[(size_t)r * cols + j] = gumbel_noise(seed, key, step, j);
}

inline int launch_sample(const SampleParams& p, cudaStream_t st) {
    if (p.R <= 0) return QTTS_OK;
    if (p.V > kSampleThreads * kSampleMaxPer || p.topk < 1 || p.topk > 64 || p.topk > p.V) {
        set_error("sample: need V <= %d and 1 <= topk <= min(64, V)", kSampleThreads * kSampleMaxPer);
        return QTTS_ERR_UNSUPPORTED;
    }
    QTTS_LAUNCH(sample_kernel, dim3(p.R), dim3(kSampleThreads), 0, st, p);
    return QTTS_OK;
}

}  // namespace qtts
