// tcgen05 bf16 GEMM for weight-streaming projections: Y[M,N] = X[M,K] · W[N,K]^T.
//
// Decode runs the projections at M = 64 tokens, where the work is reading the
// weights once from HBM.  The kernel therefore puts the WEIGHT rows on the
// UMMA M side (128 rows per tile, TMEM lanes) and the tokens on the N side
// (BN columns of the TMEM accumulator), so one 128 x BN x 16 UMMA consumes a
// 4 KB slice of weights.  Split-K spreads the K range of one 128-row weight
// tile over the CTAs of a thread-block cluster (1 x splits x 1); the fp32
// partial tiles are reduced through distributed shared memory — each CTA
// reduces a slice of about BN/splits tokens across the cluster — so there is no
// global workspace and no atomics, and the result is deterministic.
//
// Activation precision: at decode the MMA pipe is idle (the kernel waits on
// weight bytes), so an activation operand can be carried as a bf16 pair
// hi + lo (hi = bf16(x), lo = bf16(x - hi)); the lo tile follows the hi tile in
// shared memory, so one UMMA of N = 2·BN per k-slice puts W·hi and W·lo in
// adjacent TMEM columns, which the staging adds: ~16 mantissa bits of the fp32
// activation for no extra HBM bytes.
//
// Roles in a 128- (or 256-) thread CTA: warp 0 lane 0 issues TMA loads into a
// STAGES-deep ring (full/empty mbarriers), warp 1 lane 0 issues UMMAs and
// commits, warp 2 owns the TMEM allocation; all warps run the epilogue (warp w
// reads TMEM lanes 32(w%4)..32(w%4)+31; with 256 threads warps w and w+4 split
// the token columns).  The 256-thread form serves the wide-row convolution
// GEMMs of the code2wav decoder, whose epilogues carry most of the work.
//
// Epilogues (fused, applied by the reducing CTA to its token slice):
//   BF16 / F32 store (+bias), RESIDUAL (fp32 residual += Y, the "residual +"
//   of talker_unified_modules.py:222, 227), SWIGLU (silu(gate)*up of
//   Qwen3MLP; weight rows interleaved 64 gate / 64 up per tile), QKV_ROPE
//   (per-head q_norm/k_norm RMSNorm, RoPE, q to a buffer, k/v stored into the
//   paged KV pool through the slot mapping — talker_unified_modules.py:173-190),
//   CONV (code2wav: bias, layer scale, residual, SnakeBeta/GELU, strided and
//   slot-indexed stores; see ConvEpi).
#pragma once

#include "common.cuh"

namespace qtts {

// Element (stream, time, channel) of an activation buffer.  Streams are
// indexed by their slot (per-stream state that persists across steps) or by
// the row of this call; time t sits at row ctx + t of the stream's
// seq_rows-row segment, so the ctx rows before it hold the left context of a
// causal convolution.
struct ActView {
    void* ptr;  // null: not used
    int by_slot, seq_rows, ctx, ld;
    unsigned long long limit_bytes;  // bytes of the allocation behind ptr (0: not checked)
};

// Self-check of an epilogue access of `bytes` at element `idx` of a view of `esize`-byte elements:
// false (and the device error recorded) when it would leave the view's allocation.
__device__ __forceinline__ bool view_ok(const ActView& v, size_t idx, int esize, int bytes) {
    if (v.limit_bytes == 0 || idx * (size_t)esize + (size_t)bytes <= v.limit_bytes) return true;
    record_error(DEV_ERR_GEMM_BOUNDS);
    return false;
}

__host__ __device__ __forceinline__ size_t view_index(const ActView& v, int r, int slot, int t, int c) {
    return ((size_t)(v.by_slot ? slot : r) * v.seq_rows + v.ctx + t) * v.ld + c;
}

enum ConvAct : int { ACT_NONE = 0, ACT_SNAKE = 1, ACT_GELU = 2 };

// Epilogue of the code2wav GEMMs.  GEMM row m is (stream r = m / T_rows,
// step i = m % T_rows); column n is (phase n / C_o, channel n % C_o), so a
// transposed convolution written as a GEMM (phases = stride) lands at time
// t = i * phases + phase.  With y = acc + bias[n]:
//   v = (res ? res[r,t,c] : 0) + (scale ? scale[c] : 1) * y
//   out32[r,t,c] = v ;  out16[r,t,c] = bf16(act(v))
// Columns n >= n_valid are tile padding and are not stored.
struct ConvEpi {
    int T_rows, phases, C_o, n_valid, act;
    int T_valid;  // rows per stream that exist (0: all T_rows); the rest pad a stream to whole row tiles
    const int32_t* row_slot;
    const __nv_bfloat16* scale;  // per channel, or null
    const float* act_p;          // SnakeBeta: [2][C_o] = exp(alpha), exp(-beta)
    ActView res, out32, out16;
};

constexpr int kEpiConv = 16;  // internal epilogue id (not part of the C ABI)

// Implicit convolution operand: instead of a dense [M][K] X, row tile (stream r,
// steps t0..t0+BN) at k-block kb = (tap, channel block cb) is the box
// H[slot(r)][t0 + tap*dil ..][cb*64 ..] of a slot-indexed history buffer whose
// segments hold ctx = (taps-1)*dil context rows before the T current rows.
// Needs T % BN == 0 (a row tile never spans two streams).
struct ImplicitX {
    int on;
    int T;         // rows per stream
    int seq_rows;  // rows per slot segment of the history buffer
    int dil;       // tap stride in rows
    int cblocks;   // 64-channel blocks per tap (channels padded to a multiple of 64)
    const int32_t* row_slot;
};

// RMSNorm folded into the GEMMs around it.  RMSNorm(x)·W^T = inv_rms(x) · ((x∘γ)·W^T)
// with inv_rms(x) = 1/sqrt(mean(x²) + eps) a per-token scalar, so
//  - the PRODUCER of x (an F32 or RESIDUAL epilogue) also writes the bf16 hi/lo
//    pair of x∘γ (the next GEMM's operand) and, per token, the sum of x² over its
//    128 columns into ss[token][tile_n];
//  - the CONSUMER (QKV or SwiGLU epilogue) sums the partials of each token in a
//    fixed order and scales its accumulators by inv_rms before anything else.
struct NormOut {
    const __nv_bfloat16* gamma;  // null: off
    __nv_bfloat16* hi;
    __nv_bfloat16* lo;
    float* ss;  // [M][N / 128]
};
struct NormIn {
    const float* ss;  // null: off; [M][parts]
    int parts;
    int K;
    float eps;
};

// Paired QKV tiles (head_dim 64, two query heads per KV head): the weight rows are ordered
// per KV head g as tile 2g = [q_{2g}; q_{2g+1}] and tile 2g+1 = [k_g; v_g], and the two tiles of
// a pair share a cluster (2 x splits).  After the epilogue has stored q and the pool K/V, the
// q tile's CTAs run the decode attention of their tokens for both heads (keys 0..position of
// the token's block) and write its output as the o-projection's hi/lo operand.
struct PairAttn {
    int on;
    __nv_bfloat16* out;     // [M][num_heads * 64]
    __nv_bfloat16* out_lo;
    float scale_log2;       // log2(e) / sqrt(64)
};

struct GemmParams {
    int M, N, K;
    int kblocks;   // K / 64
    int splits;    // cluster size along grid.y
    int epilogue;
    void* out;
    void* out_lo;  // SwiGLU: bf16 residual part of the output (hi/lo pair), or NULL
    const __nv_bfloat16* bias;
    qtts_qkv_epilogue qkv;
    ConvEpi conv;
    ImplicitX ix;
    NormOut nout;
    NormIn nin;
    PairAttn pair;
    // L2 prefetch hint: the weights of the GEMM that runs after this one (prefetched in
    // slices by the launch's CTAs while their own chain of latencies runs), or NULL
    const uint8_t* l2_next;
    unsigned long long l2_next_bytes;
};

template <int BN, int STAGES, bool SPLIT, bool PUSH = false>
struct GemmLayout {
    static constexpr int A_BYTES = 128 * 64 * 2;  // weight tile 128 rows x 64 k
    static constexpr int B_BYTES = BN * 64 * 2;   // token tile BN rows x 64 k (hi, then lo when SPLIT)
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES * (SPLIT ? 2 : 1);
    static constexpr int PIPE_BYTES = STAGES * STAGE_BYTES;
    static constexpr int PART_BYTES = BN * 128 * 4;  // fp32 partial, [BN tokens][128 rows]
    static constexpr int RING = PIPE_BYTES > PART_BYTES ? PIPE_BYTES : PART_BYTES;
    // push reduction: the partials the cluster's CTAs send this one, [split][128 rows][BN/splits tokens];
    // not aliased with the ring, which peers may still be reading from TMA when they push
    static constexpr int RECV_BYTES = PUSH ? BN * 128 * 4 : 0;
    static constexpr int BODY = RING + RECV_BYTES;
    static constexpr int SCRATCH_BYTES = 7 * 128 * 4;  // epilogue scratch: [0,136) norm sums / RoPE exchange,
                                                        // [256,512) token metadata, [0,512) norm-out sums,
                                                        // [512,640) per-token inv_rms of the norm-in,
                                                        // [640,896) paired-QKV attention metadata
    static constexpr int BAR_BYTES = 256;
    static constexpr int SMEM = 1024 + BODY + SCRATCH_BYTES + BAR_BYTES;
    static_assert(A_BYTES % 1024 == 0 && B_BYTES % 1024 == 0, "stage buffers must keep 1024-B alignment");
};

// ---------------------------------------------------------------------------
// epilogue helpers: operate on the reduced slice R[m][128] (fp32, shared)
// ---------------------------------------------------------------------------
__device__ __forceinline__ float silu(float x) { return x / (1.0f + __expf(-x)); }

// NT threads: thread (row = tid % 128, group = tid / 128) handles weight row
// `row` of the tile for tokens group, group + NT/128, ...
template <int BN, int NT>
__device__ void gemm_epilogue(const GemmParams& p, float* R, int m0, int per, int tile_n, int tile_m,
                              float* scratch, const float* pre_old = nullptr) {
    constexpr int NG = NT / 128;
    const int t = threadIdx.x & 127;  // row within the 128-row weight tile
    const int grp = threadIdx.x >> 7;
    const int n_g = tile_n * 128 + t;
    // folded RMSNorm of the operand: each token's row is scaled by its inv_rms
    // (scratch[512 + i]); the QKV and SwiGLU epilogues apply it as they read R
    const bool nin_inline = p.epilogue == QTTS_EPI_SWIGLU || p.epilogue == QTTS_EPI_QKV_ROPE;
    if (p.nin.ss && !nin_inline) {
        const float* inv = scratch + 512;
        for (int e = threadIdx.x; e < per * 128; e += NT) R[(m0 + (e >> 7)) * 128 + (e & 127)] *= inv[e >> 7];
        __syncthreads();
    }
    switch (p.epilogue) {
        case QTTS_EPI_BF16:
        case QTTS_EPI_F32:
        case QTTS_EPI_RESIDUAL: {
            // tokens in batches of 8 so the residual loads of a batch are in flight together
            const float b = p.bias ? __bfloat162float(p.bias[n_g]) : 0.0f;
            const float gam = p.nout.gamma ? __bfloat162float(p.nout.gamma[n_g]) : 0.0f;
            constexpr int B = 8;
            for (int i0 = grp; i0 < per; i0 += NG * B) {
                float v[B];
                size_t o[B];
                bool ok[B];
#pragma unroll
                for (int u = 0; u < B; ++u) {
                    const int i = i0 + NG * u;
                    const int m_g = tile_m * BN + m0 + i;
                    ok[u] = i < per && m_g < p.M;
                    v[u] = ok[u] ? R[(m0 + i) * 128 + t] + b : 0.f;
                    o[u] = ok[u] ? (size_t)m_g * p.N + n_g : 0;
                }
                if (p.epilogue == QTTS_EPI_RESIDUAL) {
                    float old[B];
#pragma unroll
                    for (int u = 0; u < B; ++u)
                        old[u] = pre_old ? pre_old[u] : (ok[u] ? __ldcg(reinterpret_cast<const float*>(p.out) + o[u]) : 0.f);
#pragma unroll
                    for (int u = 0; u < B; ++u) {
                        v[u] += old[u];
                        if (ok[u]) reinterpret_cast<float*>(p.out)[o[u]] = v[u];
                    }
                } else if (p.epilogue == QTTS_EPI_F32) {
#pragma unroll
                    for (int u = 0; u < B; ++u)
                        if (ok[u]) reinterpret_cast<float*>(p.out)[o[u]] = v[u];
                } else {
#pragma unroll
                    for (int u = 0; u < B; ++u)
                        if (ok[u]) reinterpret_cast<__nv_bfloat16*>(p.out)[o[u]] = __float2bfloat16(v[u]);
                }
                if (p.nout.gamma) {
                    // the next GEMM's operand x∘γ as a bf16 pair, and each token's sum of
                    // squares over this tile's 128 columns (warp sums, combined below)
                    float sq[B];
#pragma unroll
                    for (int u = 0; u < B; ++u) {
                        const float xg = v[u] * gam;
                        const __nv_bfloat16 hi = __float2bfloat16(xg);
                        if (ok[u]) {
                            p.nout.hi[o[u]] = hi;
                            p.nout.lo[o[u]] = __float2bfloat16(xg - __bfloat162float(hi));
                        }
                        sq[u] = ok[u] ? v[u] * v[u] : 0.f;
                    }
#pragma unroll
                    for (int off = 16; off > 0; off >>= 1)  // the B reductions interleaved
#pragma unroll
                        for (int u = 0; u < B; ++u) sq[u] += __shfl_xor_sync(0xffffffffu, sq[u], off);
                    if ((t & 31) == 0) {
#pragma unroll
                        for (int u = 0; u < B; ++u) {
                            const int i = i0 + NG * u;
                            if (i < per) scratch[(t >> 5) * 128 + i] = sq[u];
                        }
                    }
                }
            }
            if (p.nout.gamma) {
                __syncthreads();
                for (int i = threadIdx.x; i < per; i += NT) {
                    const int m_g = tile_m * BN + m0 + i;
                    if (m_g < p.M)  // fixed order over the four warps of the 128 columns
                        p.nout.ss[(size_t)m_g * (p.N >> 7) + tile_n] =
                            ((scratch[i] + scratch[128 + i]) + scratch[256 + i]) + scratch[384 + i];
                }
            }
            break;
        }
        case QTTS_EPI_SWIGLU: {
            // thread = (pair column c of the tile's 64 gate/up pairs, token lane); batches of
            // 8 tokens with every load of a batch issued before the math
            constexpr int TL = NT / 64, B = 8;
            const int c = threadIdx.x & 63, tl = threadIdx.x >> 6;
            const int half_n = p.N >> 1;
            const float* inv = scratch + 512;
            for (int i0 = tl; i0 < per; i0 += TL * B) {
                float g[B], u[B];
#pragma unroll
                for (int k = 0; k < B; ++k) {
                    const int i = i0 + TL * k;
                    const bool ok = i < per;
                    const float sc = (ok && p.nin.ss) ? inv[i] : 1.f;
                    g[k] = ok ? R[(m0 + i) * 128 + c] * sc : 0.f;
                    u[k] = ok ? R[(m0 + i) * 128 + 64 + c] * sc : 0.f;
                }
#pragma unroll
                for (int k = 0; k < B; ++k) {
                    const int i = i0 + TL * k;
                    const int m_g = tile_m * BN + m0 + i;
                    if (i >= per || m_g >= p.M) continue;
                    const float a = __fdividef(g[k], 1.0f + __expf(-g[k])) * u[k];
                    const size_t o = (size_t)m_g * half_n + tile_n * 64 + c;
                    const __nv_bfloat16 hi = __float2bfloat16(a);
                    reinterpret_cast<__nv_bfloat16*>(p.out)[o] = hi;
                    if (p.out_lo)
                        reinterpret_cast<__nv_bfloat16*>(p.out_lo)[o] = __float2bfloat16(a - __bfloat162float(hi));
                }
            }
            break;
        }
        case QTTS_EPI_QKV_ROPE: {
            if constexpr (NT == 128) {  // the plans never pair this epilogue with wider CTAs
                const qtts_qkv_epilogue& e = p.qkv;
                const int D = e.head_dim;
                const int q_rows = e.num_heads * D;
                const int k_rows = e.kv_heads * D;
                const int d = n_g % D;
                const int warp = t >> 5, lane = t & 31;
                // region (q / k / v) and the column within it; paired tiles: tile 2g = q heads 2g, 2g+1,
                // tile 2g+1 = k_g then v_g
                int region, col;
                if (p.pair.on) {
                    region = (tile_n & 1) ? (t < 64 ? 1 : 2) : 0;
                    col = (tile_n & 1) ? (tile_n >> 1) * 64 + (t & 63) : (tile_n >> 1) * 128 + t;
                } else {
                    region = n_g < q_rows ? 0 : (n_g < q_rows + k_rows ? 1 : 2);
                    col = region == 0 ? n_g : (region == 1 ? n_g - q_rows : n_g - q_rows - k_rows);
                }
                const __nv_bfloat16* nw = region == 0 ? (const __nv_bfloat16*)e.q_norm_w
                                                      : (const __nv_bfloat16*)e.k_norm_w;
                const float wn = region < 2 ? __bfloat162float(nw[d]) : 0.f;
                const int half = D >> 1;
                const int dd = d < half ? d : d - half;
                const int partner_t = d < half ? t + half : t - half;
                const int wpd = D >> 5, w0 = (warp / wpd) * wpd;  // the warps of this thread's head
                const float* inv = scratch + 512;
                float* red = scratch;  // [4 warps][8 tokens] per-head sums of squares
                // per-token position and KV row base, written by the kernel before the reduction
                const int* tok_pos = reinterpret_cast<const int*>(scratch) + 256;
                const int* tok_kv = tok_pos + 128;
                const int kv_col = region == 0 ? 0 : (((region - 1) * e.kv_heads) + col / D) * e.block_size;
                const float inv_d = 1.0f / (float)D;  // D is a power of two: exact
                // 8 tokens at a time: RoPE table loads, head norms and stores of the 8 overlap;
                // two barriers per 8 tokens (norm sums, RoPE partner exchange through R)
                for (int c0 = 0; c0 < per; c0 += 8) {
                    float v[8], cs[8], sn[8], sq[8];
#pragma unroll
                    for (int k = 0; k < 8; ++k) {
                        const int i = c0 + k;
                        const bool ok = i < per && tile_m * BN + m0 + i < p.M;
                        cs[k] = 1.f;
                        sn[k] = 0.f;
                        if (region < 2 && ok) {
                            cs[k] = e.rope_cos[(size_t)tok_pos[i] * half + dd];
                            sn[k] = e.rope_sin[(size_t)tok_pos[i] * half + dd];
                        }
                        v[k] = ok ? R[(m0 + i) * 128 + t] * (p.nin.ss ? inv[i] : 1.f) : 0.f;
                        sq[k] = v[k] * v[k];
                    }
#pragma unroll
                    for (int off = 16; off > 0; off >>= 1)
#pragma unroll
                        for (int k = 0; k < 8; ++k) sq[k] += __shfl_xor_sync(0xffffffffu, sq[k], off);
                    if (lane == 0) {
#pragma unroll
                        for (int k = 0; k < 8; ++k) red[warp * 8 + k] = sq[k];
                    }
                    __syncthreads();
                    if (region < 2) {
#pragma unroll
                        for (int k = 0; k < 8; ++k) {
                            float tot = 0.f;
#pragma unroll
                            for (int w = 0; w < 4; ++w)  // head_dim <= 128: at most 4 warps per head
                                if (w < wpd) tot += red[(w0 + w) * 8 + k];
                            v[k] = v[k] * rsqrtf(tot * inv_d + e.rms_eps) * wn;
                        }
                    }
                    // each thread rewrites only its own elements of R, read by its RoPE partner
#pragma unroll
                    for (int k = 0; k < 8; ++k)
                        if (c0 + k < per) R[(m0 + c0 + k) * 128 + t] = v[k];
                    __syncthreads();
#pragma unroll
                    for (int k = 0; k < 8; ++k) {
                        const int i = c0 + k;
                        const int m_g = tile_m * BN + m0 + i;
                        if (i >= per || m_g >= p.M) continue;
                        float val = v[k];
                        if (region < 2) {
                            const float partner = R[(m0 + i) * 128 + partner_t];
                            val = d < half ? val * cs[k] - partner * sn[k] : val * cs[k] + partner * sn[k];
                        }
                        if (region == 0) {
                            reinterpret_cast<float*>(p.out)[(size_t)m_g * q_rows + col] = val;  // q stays fp32
                        } else if (tok_kv[i] >= 0) {
                            reinterpret_cast<kv_t*>(e.kv_pool)[(size_t)(tok_kv[i] + kv_col) * D + d] = to_kv(val);
                        }
                    }
                }
            }
            break;
        }
        case kEpiConv: {
            // Vectorised: thread = (channel quad cg, token lane tl).  Each token's
            // row index in the three views is computed once into shared memory,
            // and the residual loads of 8 tokens are issued before their stores.
            const ConvEpi& e = p.conv;
            int* tok_ok = reinterpret_cast<int*>(scratch);
            int* row_res = tok_ok + 128;
            int* row_o32 = row_res + 128;
            int* row_o16 = row_o32 + 128;
            for (int i = threadIdx.x; i < per; i += NT) {
                const int m_g = tile_m * BN + m0 + i;
                const int r = m_g < p.M ? m_g / e.T_rows : 0;
                const bool ok = m_g < p.M && (e.T_valid == 0 || m_g - r * e.T_rows < e.T_valid);
                const int t0 = ok ? (m_g - r * e.T_rows) * e.phases : 0;
                const int sl = (ok && e.row_slot) ? e.row_slot[r] : r;
                tok_ok[i] = ok;
                row_res[i] = (e.res.by_slot ? sl : r) * e.res.seq_rows + e.res.ctx + t0;
                row_o32[i] = (e.out32.by_slot ? sl : r) * e.out32.seq_rows + e.out32.ctx + t0;
                row_o16[i] = (e.out16.by_slot ? sl : r) * e.out16.seq_rows + e.out16.ctx + t0;
            }
            __syncthreads();
            constexpr int NTL = NT / 32;  // token lanes
            const int cg = threadIdx.x & 31, tl = threadIdx.x >> 5;
            const int n0 = tile_n * 128 + cg * 4;
            if (n0 >= e.n_valid) break;  // n_valid and C_o are multiples of 4
            const int ph = n0 / e.C_o, c0 = n0 - ph * e.C_o;
            float b4[4], s4[4], pa[4], pb[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                b4[k] = p.bias ? __bfloat162float(p.bias[n0 + k]) : 0.0f;
                s4[k] = e.scale ? __bfloat162float(e.scale[c0 + k]) : 1.0f;
                pa[k] = e.act == ACT_SNAKE ? e.act_p[c0 + k] : 0.f;
                pb[k] = e.act == ACT_SNAKE ? e.act_p[e.C_o + c0 + k] : 0.f;
            }
            const float* res = reinterpret_cast<const float*>(e.res.ptr);
            float* o32 = reinterpret_cast<float*>(e.out32.ptr);
            __nv_bfloat16* o16 = reinterpret_cast<__nv_bfloat16*>(e.out16.ptr);
            constexpr int B = 8;
            for (int i0 = tl; i0 < per; i0 += NTL * B) {
                float4 v[B];
                bool ok[B];
#pragma unroll
                for (int u = 0; u < B; ++u) {
                    const int i = i0 + NTL * u;
                    ok[u] = i < per && tok_ok[i];
                    v[u] = make_float4(0.f, 0.f, 0.f, 0.f);
                    if (ok[u]) {
                        const float4 a = *reinterpret_cast<const float4*>(R + (m0 + i) * 128 + cg * 4);
                        v[u] = make_float4(s4[0] * (a.x + b4[0]), s4[1] * (a.y + b4[1]), s4[2] * (a.z + b4[2]),
                                           s4[3] * (a.w + b4[3]));
                    }
                }
                if (res) {
                    float4 rv[B];
#pragma unroll
                    for (int u = 0; u < B; ++u) {
                        const int i = i0 + NTL * u;
                        const size_t ri = (size_t)(row_res[i] + ph) * e.res.ld + c0;
                        rv[u] = (ok[u] && view_ok(e.res, ri, 4, 16)) ? *reinterpret_cast<const float4*>(res + ri)
                                                                       : make_float4(0.f, 0.f, 0.f, 0.f);
                    }
#pragma unroll
                    for (int u = 0; u < B; ++u) {
                        v[u].x += rv[u].x;
                        v[u].y += rv[u].y;
                        v[u].z += rv[u].z;
                        v[u].w += rv[u].w;
                    }
                }
#pragma unroll
                for (int u = 0; u < B; ++u) {
                    if (!ok[u]) continue;
                    const int i = i0 + NTL * u;
                    if (o32) {
                        const size_t oi = (size_t)(row_o32[i] + ph) * e.out32.ld + c0;
                        if (view_ok(e.out32, oi, 4, 16)) *reinterpret_cast<float4*>(o32 + oi) = v[u];
                    }
                    if (o16) {
                        float a[4] = {v[u].x, v[u].y, v[u].z, v[u].w};
#pragma unroll
                        for (int k = 0; k < 4; ++k) {
                            if (e.act == ACT_SNAKE) {
                                const float sn = __sinf(a[k] * pa[k]);
                                a[k] = a[k] + sn * sn * pb[k];
                            } else if (e.act == ACT_GELU) {
                                a[k] = 0.5f * a[k] * (1.0f + erff(a[k] * 0.70710678118654752f));
                            }
                        }
                        const __nv_bfloat162 h01 = __floats2bfloat162_rn(a[0], a[1]);
                        const __nv_bfloat162 h23 = __floats2bfloat162_rn(a[2], a[3]);
                        uint2 pack;
                        pack.x = *reinterpret_cast<const uint32_t*>(&h01);
                        pack.y = *reinterpret_cast<const uint32_t*>(&h23);
                        const size_t hi16 = (size_t)(row_o16[i] + ph) * e.out16.ld + c0;
                        if (view_ok(e.out16, hi16, 2, 8)) *reinterpret_cast<uint2*>(o16 + hi16) = pack;
                    }
                }
            }
            break;
        }
        default:
            break;
    }
}

// Decode attention of a paired QKV launch (see PairAttn), run after the pair's epilogues have
// stored q (fp32, p.out) and this step's K/V into the pool: the eight warps of the pair take
// tokens gw, gw + 8, ... of the CTA's token slice; a warp loads the token's keys and values
// 0..nk-1 for KV head g (lane l owns dims 2l, 2l+1), scores both query heads, softmax, and
// writes the two heads' outputs as a bf16 hi/lo pair.  Same math as short_attn_kernel.
template <int BN>
__device__ void pair_attention(const GemmParams& p, int m0, int per, int tile_n, int tile_m, int pm,
                               const float* scratch) {
    const qtts_qkv_epilogue& e = p.qkv;
    const int* tok_kb = reinterpret_cast<const int*>(scratch) + 640;
    const int* tok_nk = tok_kb + 128;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = tile_n >> 1, h0 = 2 * g;
    const int q_cols = e.num_heads * 64;
    const kv_t* kv = reinterpret_cast<const kv_t*>(e.kv_pool);
    const float* q = reinterpret_cast<const float*>(p.out);
    for (int i = pm * 4 + warp; i < per; i += 8) {
        const int m_g = tile_m * BN + m0 + i;
        if (m_g >= p.M) break;
        const int nk = min(tok_nk[i], 16);
        const size_t orow = (size_t)m_g * q_cols + h0 * 64 + 2 * lane;
        if (nk <= 0) {
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                *reinterpret_cast<__nv_bfloat162*>(p.pair.out + orow + h * 64) = __floats2bfloat162_rn(0.f, 0.f);
                *reinterpret_cast<__nv_bfloat162*>(p.pair.out_lo + orow + h * 64) = __floats2bfloat162_rn(0.f, 0.f);
            }
            continue;
        }
        const size_t krow = (size_t)tok_kb[i] + (size_t)g * e.block_size;
        const size_t vrow = (size_t)tok_kb[i] + (size_t)(e.kv_heads + g) * e.block_size;
        __half2 kr[16], vr[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            // L2 loads (.cg): this step's rows were stored by the other CTA of the pair
            kr[j] = j < nk ? __ldcg(reinterpret_cast<const __half2*>(kv + (krow + j) * 64 + 2 * lane)) : __float2half2_rn(0.f);
            vr[j] = j < nk ? __ldcg(reinterpret_cast<const __half2*>(kv + (vrow + j) * 64 + 2 * lane)) : __float2half2_rn(0.f);
        }
        const float2 qa = __ldcg(reinterpret_cast<const float2*>(q + orow));
        const float2 qb = __ldcg(reinterpret_cast<const float2*>(q + orow + 64));
        float sa[16], sb[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            const float2 k = __half22float2(kr[j]);
            sa[j] = qa.x * k.x + qa.y * k.y;
            sb[j] = qb.x * k.x + qb.y * k.y;
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                sa[j] += __shfl_xor_sync(0xffffffffu, sa[j], off);
                sb[j] += __shfl_xor_sync(0xffffffffu, sb[j], off);
            }
        }
        float ma = -INFINITY, mb = -INFINITY;
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            sa[j] *= p.pair.scale_log2;
            sb[j] *= p.pair.scale_log2;
            if (j < nk) {
                ma = fmaxf(ma, sa[j]);
                mb = fmaxf(mb, sb[j]);
            }
        }
        float la = 0.f, lb = 0.f, oa0 = 0.f, oa1 = 0.f, ob0 = 0.f, ob1 = 0.f;
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            const float pa = j < nk ? exp2f(sa[j] - ma) : 0.f;
            const float pb = j < nk ? exp2f(sb[j] - mb) : 0.f;
            const float2 v = __half22float2(vr[j]);
            la += pa;
            lb += pb;
            oa0 += pa * v.x;
            oa1 += pa * v.y;
            ob0 += pb * v.x;
            ob1 += pb * v.y;
        }
        const float ia = 1.0f / la, ib = 1.0f / lb;
        const float o[4] = {oa0 * ia, oa1 * ia, ob0 * ib, ob1 * ib};
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const __nv_bfloat162 hi = __floats2bfloat162_rn(o[2 * h], o[2 * h + 1]);
            const float2 hf = __bfloat1622float2(hi);
            *reinterpret_cast<__nv_bfloat162*>(p.pair.out + orow + h * 64) = hi;
            *reinterpret_cast<__nv_bfloat162*>(p.pair.out_lo + orow + h * 64) =
                __floats2bfloat162_rn(o[2 * h] - hf.x, o[2 * h + 1] - hf.y);
        }
    }
}

// This CTA's slice of the L2 prefetch of the next GEMM's weights (GemmParams::l2_next):
// 4 KB-aligned slices, one bulk prefetch per 32 KB.  A hint: no data moves into the SM.
__device__ __forceinline__ void l2_prefetch_slice(const uint8_t* base, unsigned long long bytes, int cta, int ctas) {
    const unsigned long long per = ((bytes / (unsigned long long)ctas) + 4095ull) & ~4095ull;
    const unsigned long long b0 = (unsigned long long)cta * per;
    const unsigned long long b1 = b0 + per < bytes ? b0 + per : bytes;
    for (unsigned long long o = b0; o < b1; o += 32768ull) {
        const unsigned long long rest = b1 - o;
        const uint32_t n = (uint32_t)(rest < 32768ull ? rest : 32768ull) & ~15u;
        if (n) asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(base + o), "r"(n) : "memory");
    }
}

// ---------------------------------------------------------------------------
// pieces of a split-K tile shared by the per-launch kernel and the persistent
// code-predictor kernel (cp_persist.cuh)
// ---------------------------------------------------------------------------

// Per-token data the epilogue needs, gathered while the cluster reduction runs: the folded
// norm's inv_rms (scratch[512 + i], from the producer's per-tile sums of squares, read through
// L2 because a persistent kernel's earlier phase wrote them) and the QKV epilogue's token
// metadata.
template <int BN, int NT>
__device__ __forceinline__ void epilogue_meta(const GemmParams& p, float* scratch, int m0, int per, int tile_m) {
    if (p.nin.ss) {
        for (int i = threadIdx.x; i < per; i += NT) {
            const int m_g = tile_m * BN + m0 + i;
            float tot = 0.f;
            if (m_g < p.M) {
                const float* q = p.nin.ss + (size_t)m_g * p.nin.parts;
                for (int j = 0; j < p.nin.parts; ++j) tot += __ldcg(q + j);  // fixed order: deterministic
            }
            scratch[512 + i] = rsqrtf(tot / (float)p.nin.K + p.nin.eps);
        }
    }
    if (p.epilogue == QTTS_EPI_QKV_ROPE) {
        // token metadata of the QKV epilogue: clamped RoPE position, and the KV-pool row of
        // (block, layer, k, head 0, offset) for the token's slot (-1: not stored)
        const qtts_qkv_epilogue& e = p.qkv;
        int* tok_pos = reinterpret_cast<int*>(scratch) + 256;
        int* tok_kv = tok_pos + 128;
        for (int i = threadIdx.x; i < per; i += NT) {
            const int m_g = tile_m * BN + m0 + i;
            const int pos = m_g < p.M ? e.row_pos[m_g] : 0;
            const int slot = m_g < p.M ? e.slot_mapping[m_g] : -1;
            tok_pos[i] = pos < 0 ? 0 : (pos >= e.max_pos ? e.max_pos - 1 : pos);  // table bounds
            const int kb = slot < 0 ? 0 : ((slot / e.block_size) * e.num_layers + e.layer) * 2 * e.kv_heads * e.block_size;
            tok_kv[i] = slot < 0 ? -1 : kb + slot % e.block_size;
            if (p.pair.on) {  // the token's block (keys 0 .. its offset) for the pair's attention
                reinterpret_cast<int*>(scratch)[640 + i] = kb;
                reinterpret_cast<int*>(scratch)[768 + i] = slot < 0 ? 0 : slot % e.block_size + 1;
            }
        }
    }
}

// The residual epilogue's old values of this thread's row for up to 8 tokens, loaded early
// (through L2: the residual stream is rewritten by other CTAs between phases).
template <int BN, int NT>
__device__ __forceinline__ void residual_prefetch(const GemmParams& p, int m0, int per, int tile_n, int tile_m,
                                                  float (&pre_old)[8]) {
    const int t = threadIdx.x & 127, grp = threadIdx.x >> 7;
#pragma unroll
    for (int u = 0; u < 8; ++u) {
        const int i = grp + (NT / 128) * u;
        const int m_g = tile_m * BN + m0 + i;
        pre_old[u] = (i < per && m_g < p.M)
                         ? __ldcg(reinterpret_cast<const float*>(p.out) + (size_t)m_g * p.N + tile_n * 128 + t)
                         : 0.f;
    }
}

// Split-K reduction of this CTA's token slice [m0, m0 + per): the fp32 partials P[token][128]
// of the cluster's CTAs (each in its own shared memory) are summed in a fixed order into this
// CTA's P.  A cluster of `members` tiles x splits: the splits of member pm are ranks
// members * r + pm (paired QKV tiles: members 2).  The loads of two float4 chunks from every
// split are issued before any is consumed, so the remote-shared-memory latency is paid once
// per 16 loads.
template <int NT>
__device__ __forceinline__ void cluster_reduce_slice(float* P, int m0, int per, int splits, int members, int pm) {
    const uint32_t base = smem_u32(P + m0 * 128);
    for (int e = threadIdx.x; e < per * 32; e += 2 * NT) {
        const int e2 = e + NT;
        const bool two = e2 < per * 32;
        float4 v[2][8];
#pragma unroll
        for (int r = 0; r < 8; ++r) {
            if (r < splits) {
                const uint32_t peer = (uint32_t)(members * r + pm);
                v[0][r] = ld_dsmem_f32x4(map_to_rank(base + (uint32_t)e * 16u, peer));
                if (two) v[1][r] = ld_dsmem_f32x4(map_to_rank(base + (uint32_t)e2 * 16u, peer));
            }
        }
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            if (h == 1 && !two) break;
            float4 acc = v[h][0];
#pragma unroll
            for (int r = 1; r < 8; ++r) {  // fixed order: deterministic
                if (r < splits) {
                    acc.x += v[h][r].x;
                    acc.y += v[h][r].y;
                    acc.z += v[h][r].z;
                    acc.w += v[h][r].w;
                }
            }
            *reinterpret_cast<float4*>(P + m0 * 128 + (h ? e2 : e) * 4) = acc;
        }
    }
}

// ---------------------------------------------------------------------------
// the kernel
// ---------------------------------------------------------------------------
template <int BN, int STAGES, bool SPLIT, int NT, bool PUSH = false>
__global__ void __launch_bounds__(NT) gemm_tc_kernel(const __grid_constant__ CUtensorMap tmW,
                                                     const __grid_constant__ CUtensorMap tmX,
                                                     const __grid_constant__ CUtensorMap tmXlo,
                                                     const GemmParams p) {
    static_assert(NT == 128 || NT == 256, "128 or 256 threads");
    static_assert(!PUSH || (NT == 128 && BN == 64), "push reduction: BN 64, 128 threads");
    using L = GemmLayout<BN, STAGES, SPLIT, PUSH>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    float* scratch = reinterpret_cast<float*>(smem + L::BODY);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::BODY + L::SCRATCH_BYTES);
    uint64_t* empty = full + STAGES;
    uint64_t* accum = empty + STAGES;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accum + 1);
    int* flags = reinterpret_cast<int*>(tmem_slot + 1);  // [0] error, [1] loads issued, [2] loads consumed

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int tile_n = blockIdx.x, tile_m = blockIdx.z;
    // cluster (1, splits, 1): rank = split; paired QKV tiles: (2, splits, 1), rank = member + 2 * split
    const int crank = (int)cluster_ctarank();
    const int split = p.pair.on ? crank >> 1 : crank;
    const int pm = p.pair.on ? crank & 1 : 0;  // 0: the q tile of the pair, 1: the k|v tile
    const int per_split = p.kblocks / p.splits, rem = p.kblocks % p.splits;
    const int kb0 = split * per_split + min(split, rem);
    const int nkb = per_split + (split < rem ? 1 : 0);

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(accum, 1);
        flags[0] = 0;
        flags[1] = 0;
        flags[2] = 0;
        fence_mbar_init();
        tma_prefetch_desc(&tmW);
        tma_prefetch_desc(&tmX);
        if (SPLIT) tma_prefetch_desc(&tmXlo);
        // The weights do not depend on the previous kernel: start streaming the
        // first stages before waiting for it (programmatic dependent launch).
        for (int i = 0; i < nkb && i < STAGES; ++i) {
            mbar_arrive_expect_tx(&full[i], L::STAGE_BYTES);
            tma_load_2d(smem + i * L::STAGE_BYTES, &tmW, &full[i], (kb0 + i) * 64, tile_n * 128);
        }
    }
    if (p.l2_next && threadIdx.x == 96)  // warp 3 has no role before the epilogue
        l2_prefetch_slice(p.l2_next, p.l2_next_bytes,
                          (int)(blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z)),
                          (int)(gridDim.x * gridDim.y * gridDim.z));
    griddep_wait();  // activations, outputs and the KV pool belong to earlier kernels
    griddep_launch();
    if (warp == 2) {
        tmem_alloc(tmem_slot, SPLIT ? 2 * BN : BN);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0 && lane == 0) {
        // ---------------- TMA producer ----------------
        int issued = 0;
        int x_row0 = 0;  // implicit convolution: first history row of this row tile
        if (p.ix.on) {
            const int m0g = tile_m * BN, r = m0g / p.ix.T;
            x_row0 = p.ix.row_slot[r] * p.ix.seq_rows + (m0g - r * p.ix.T);
        }
        for (int i = 0; i < nkb; ++i) {
            const int s = i % STAGES;
            const uint32_t ph = (uint32_t)(i / STAGES) & 1u;
            if (i >= STAGES && !mbar_wait(&empty[s], ph ^ 1u, DEV_ERR_GEMM_PRODUCER)) {
                flags[0] = 1;
                break;
            }
            uint8_t* a = smem + s * L::STAGE_BYTES;
            uint8_t* b = a + L::A_BYTES;
            if (i >= STAGES) {  // the first stages' weight tiles are already in flight
                mbar_arrive_expect_tx(&full[s], L::STAGE_BYTES);
                tma_load_2d(a, &tmW, &full[s], (kb0 + i) * 64, tile_n * 128);
            }
            if (p.ix.on) {
                const int kb = kb0 + i, tap = kb / p.ix.cblocks, cb = kb - tap * p.ix.cblocks;
                tma_load_2d(b, &tmX, &full[s], cb * 64, x_row0 + tap * p.ix.dil);
            } else {
                tma_load_2d(b, &tmX, &full[s], (kb0 + i) * 64, tile_m * BN);
                if (SPLIT) tma_load_2d(b + L::B_BYTES, &tmXlo, &full[s], (kb0 + i) * 64, tile_m * BN);
            }
            ++issued;
        }
        flags[1] = issued;
    } else if (warp == 1 && lane == 0) {
        // ---------------- UMMA issuer ----------------
        // hi/lo operands: the lo tile sits right after the hi tile, so one UMMA of N = 2 BN
        // accumulates W·hi into columns [0, BN) and W·lo into [BN, 2 BN); staging adds them
        const uint32_t idesc = make_idesc_bf16(128, SPLIT ? 2 * BN : BN);
        int consumed = 0;
        for (int i = 0; i < nkb; ++i) {
            const int s = i % STAGES;
            const uint32_t ph = (uint32_t)(i / STAGES) & 1u;
            if (!mbar_wait(&full[s], ph, DEV_ERR_GEMM_MMA)) {
                flags[0] = 1;
                break;
            }
            tc_fence_after();
            const uint32_t a = smem_u32(smem + s * L::STAGE_BYTES);
            const uint64_t da = make_sw128_desc(a);
            const uint64_t db = make_sw128_desc(a + L::A_BYTES);
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)  // 4 x UMMA_K(16) = 64; +32 B per step inside the swizzle atom
                umma_bf16(tmem, da + 2 * kk, db + 2 * kk, idesc, (i > 0 || kk > 0) ? 1u : 0u);
            umma_commit(&empty[s]);
            ++consumed;
        }
        flags[2] = consumed;
        umma_commit(accum);
    }
    __syncwarp();

    // ---------------- epilogue: TMEM -> shared partial ----------------
    const bool ok = mbar_wait(accum, 0, DEV_ERR_GEMM_EPILOGUE);
    tc_fence_after();
    __syncthreads();
    if (threadIdx.x == 0 && (flags[0] || !ok)) {
        // drain: wait (bounded) for loads issued but never consumed before reusing their buffers
        for (int i = flags[2]; i < flags[1]; ++i)
            mbar_wait(&full[i % STAGES], (uint32_t)(i / STAGES) & 1u, DEV_ERR_DRAIN);
    }
    __syncthreads();
    float* P = reinterpret_cast<float*>(smem);
    const bool good = ok && flags[0] == 0;
    // this CTA's token slice of the reduction: [m0, m0 + per), slices differ by at most one
    // token when splits does not divide BN
    const int m0 = split * BN / p.splits;
    const int per = (split + 1) * BN / p.splits - m0;
    const bool push = PUSH && p.splits > 1;
    {
        // warp w reads TMEM lane quarter w % 4; with 256 threads warps w and w + 4
        // take one half of the columns each
        const int quarter = warp & 3, half = warp >> 2;
        constexpr int COLS = BN / (NT / 128);
        const int row = quarter * 32 + lane;
        // push: each 4-token group goes straight from registers to the receive buffer of
        // the CTA that owns those tokens, at [this split][row][token in its slice]
        const uint32_t recv_s = smem_u32(smem + L::RING) + (uint32_t)((split * 128 + row) * per) * 4u;
#pragma unroll 1
        for (int c = half * COLS; c < (half + 1) * COLS; c += 16) {
            float v[16];
            tmem_ld16(tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)c, v);
            if (SPLIT) {
                float vl[16];
                tmem_ld16(tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(c + BN), vl);
#pragma unroll
                for (int j = 0; j < 16; ++j) v[j] += vl[j];
            }
            if (push) {
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const int tok = c + 4 * q, dst = tok / per, i0 = tok - dst * per;
                    const uint32_t a = map_to_rank(recv_s + (uint32_t)i0 * 4u, (uint32_t)dst);
                    if (good)
                        st_dsmem_f32x4(a, v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
                    else
                        st_dsmem_f32x4(a, 0.f, 0.f, 0.f, 0.f);
                }
            } else {
#pragma unroll
                for (int j = 0; j < 16; ++j) P[(c + j) * 128 + row] = good ? v[j] : 0.0f;
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 2) tmem_dealloc(tmem, SPLIT ? 2 * BN : BN);

    // ---------------- split-K reduction across the cluster ----------------
    // pull: arrive = this CTA's partial is in its shared memory; push: arrive = this
    // CTA's stores into its peers' receive buffers are done
    if (p.splits > 1) cluster_arrive();
    // Loads the epilogue needs are issued between arriving at the cluster barrier
    // and waiting on it, so they overlap the barrier and the reduction: the old
    // residual (when the token slice is one batch) and the norm-in partial sums.
    epilogue_meta<BN, NT>(p, scratch, m0, per, tile_m);
    float pre_old[8];
    const bool prefetch = p.epilogue == QTTS_EPI_RESIDUAL && per <= 8 * (NT / 128);
    if (prefetch) residual_prefetch<BN, NT>(p, m0, per, tile_n, tile_m, pre_old);
    if (push) {
        cluster_wait();  // every peer's partial of this CTA's token slice has landed here
        const float* recv = reinterpret_cast<const float*>(smem + L::RING);
        const int t = threadIdx.x;  // weight row
        for (int i0 = 0; i0 < per; i0 += 4) {
            float4 acc = *reinterpret_cast<const float4*>(recv + (size_t)t * per + i0);
            for (int r = 1; r < p.splits; ++r) {  // fixed order: deterministic
                const float4 b = *reinterpret_cast<const float4*>(recv + ((size_t)r * 128 + t) * per + i0);
                acc.x += b.x;
                acc.y += b.y;
                acc.z += b.z;
                acc.w += b.w;
            }
            P[(m0 + i0) * 128 + t] = acc.x;
            P[(m0 + i0 + 1) * 128 + t] = acc.y;
            P[(m0 + i0 + 2) * 128 + t] = acc.z;
            P[(m0 + i0 + 3) * 128 + t] = acc.w;
        }
        __syncthreads();
    } else if (p.splits > 1) {
        cluster_wait();  // every CTA's partial is in its shared memory
        cluster_reduce_slice<NT>(P, m0, per, p.splits, p.pair.on ? 2 : 1, pm);
        if (!p.pair.on) cluster_arrive();  // done reading the peers' shared memory
        __syncthreads();
    } else if (p.nin.ss || p.epilogue == QTTS_EPI_QKV_ROPE) {
        __syncthreads();
    }
    gemm_epilogue<BN, NT>(p, P, m0, per, tile_n, tile_m, scratch, prefetch ? pre_old : nullptr);
    if (p.pair.on) {
        // both tiles' stores (q, pool K/V) reach the cluster before either reads them; this
        // barrier also covers "done reading the peers' shared memory"
        __syncthreads();
        cluster_arrive();
        cluster_wait();
        if constexpr (NT == 128) pair_attention<BN>(p, m0, per, tile_n, tile_m, pm, scratch);
    } else if (p.splits > 1 && !push) {
        cluster_wait();  // no CTA leaves while a peer may still read its shared memory
    }
}

// ---------------------------------------------------------------------------
// Persistent form for wide-row convolution GEMMs (conv epilogue, no split-K):
// one CTA per SM walks the (row tile, weight tile) list.  Warp 0 lane 0 streams
// weight and activation tiles through a 4-deep ring across tile borders, warp 1
// lane 0 issues the UMMAs into one of two 128-column TMEM accumulators, and
// warps 4-11 run the conv epilogue straight from TMEM (TMEM lane = output
// channel, so a warp's loads and stores of one token are 32 consecutive
// channels): the epilogue of tile i overlaps the loads and MMAs of tile i + 1.
// ---------------------------------------------------------------------------
constexpr int kPersistStages = 4;
constexpr int kPersistThreads = 384;  // 4 control warps + 8 epilogue warps
constexpr int kPersistEpiThreads = 256;

struct PersistLayout {
    static constexpr int A_BYTES = 128 * 64 * 2;
    static constexpr int B_BYTES = 128 * 64 * 2;
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr int RING = kPersistStages * STAGE_BYTES;
    static constexpr int META = 4 * 128 * 4;  // per token: valid flag, rows in the three views
    static constexpr int BAR_BYTES = 256;
    static constexpr int SMEM = 1024 + RING + META + BAR_BYTES;
};

// Named barrier 1 among the epilogue warps; returns whether any of them passed a non-zero flag.
__device__ __forceinline__ int epi_sync_or(int flag) {
    int r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.s32 p, %1, 0;\n\t"
        "bar.red.or.pred q, 1, %2, p;\n\t"
        "selp.s32 %0, 1, 0, q;\n\t}"
        : "=r"(r)
        : "r"(flag), "n"(kPersistEpiThreads)
        : "memory");
    return r;
}

__global__ void __launch_bounds__(kPersistThreads, 1)
    gemm_conv_persist_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX,
                             const GemmParams p) {
    using L = PersistLayout;
    constexpr int BN = 128, S = kPersistStages;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    int* meta = reinterpret_cast<int*>(smem + L::RING);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::RING + L::META);
    uint64_t* empty = full + S;
    uint64_t* tfull = empty + S;   // [2] accumulator ready
    uint64_t* tempty = tfull + 2;  // [2] accumulator read out by the epilogue
    uint64_t* done = tempty + 2;   // every UMMA of this CTA has completed
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
    int* flags = reinterpret_cast<int*>(tmem_slot + 1);  // [0] error, [1] loads issued, [2] loads consumed

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n_tiles_n = p.N / 128, n_tiles = n_tiles_n * ((p.M + BN - 1) / BN);
    const int nkb = p.kblocks;
    if (threadIdx.x == 0) {
        for (int i = 0; i < S; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&tfull[i], 1);
            mbar_init(&tempty[i], 1);
        }
        mbar_init(done, 1);
        flags[0] = flags[1] = flags[2] = 0;
        fence_mbar_init();
        tma_prefetch_desc(&tmW);
        tma_prefetch_desc(&tmX);
    }
    griddep_wait();  // activations and outputs belong to earlier kernels
    griddep_launch();
    if (warp == 1) {
        tmem_alloc(tmem_slot, 2 * BN);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0 && lane == 0) {
        // ---------------- producer: every k-block of every tile of this CTA ----------------
        int it = 0;
        bool ok = true;
        for (int tile = blockIdx.x; tile < n_tiles && ok; tile += gridDim.x) {
            const int tile_m = tile / n_tiles_n, tile_n = tile - tile_m * n_tiles_n;
            int x_row0 = tile_m * BN;
            if (p.ix.on) {
                const int r = x_row0 / p.ix.T;
                x_row0 = p.ix.row_slot[r] * p.ix.seq_rows + (x_row0 - r * p.ix.T);
            }
            for (int kb = 0; kb < nkb; ++kb, ++it) {
                const int s = it % S;
                if (it >= S && !mbar_wait(&empty[s], ((uint32_t)(it / S) & 1u) ^ 1u, DEV_ERR_GEMM_PRODUCER)) {
                    ok = false;
                    break;
                }
                uint8_t* a = smem + s * L::STAGE_BYTES;
                mbar_arrive_expect_tx(&full[s], L::STAGE_BYTES);
                tma_load_2d(a, &tmW, &full[s], kb * 64, tile_n * 128);
                if (p.ix.on) {
                    const int tap = kb / p.ix.cblocks, cb = kb - tap * p.ix.cblocks;
                    tma_load_2d(a + L::A_BYTES, &tmX, &full[s], cb * 64, x_row0 + tap * p.ix.dil);
                } else {
                    tma_load_2d(a + L::A_BYTES, &tmX, &full[s], kb * 64, x_row0);
                }
            }
        }
        flags[1] = it;
        if (!ok) atomicExch(&flags[0], 1);
    } else if (warp == 1 && lane == 0) {
        // ---------------- UMMA issuer ----------------
        const uint32_t idesc = make_idesc_bf16(128, BN);
        int it = 0, j = 0;
        bool ok = true;
        for (int tile = blockIdx.x; tile < n_tiles && ok; tile += gridDim.x, ++j) {
            const int buf = j & 1;
            if (j >= 2 && !mbar_wait(&tempty[buf], ((uint32_t)(j >> 1) & 1u) ^ 1u, DEV_ERR_GEMM_MMA)) {
                ok = false;
                break;
            }
            tc_fence_after();
            const uint32_t acc = tmem + (uint32_t)(buf * BN);
            for (int kb = 0; kb < nkb; ++kb, ++it) {
                const int s = it % S;
                if (!mbar_wait(&full[s], (uint32_t)(it / S) & 1u, DEV_ERR_GEMM_MMA)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t a = smem_u32(smem + s * L::STAGE_BYTES);
                const uint64_t da = make_sw128_desc(a);
                const uint64_t db = make_sw128_desc(a + L::A_BYTES);
#pragma unroll
                for (int kk = 0; kk < 4; ++kk)
                    umma_bf16(acc, da + 2 * kk, db + 2 * kk, idesc, (kb > 0 || kk > 0) ? 1u : 0u);
                umma_commit(&empty[s]);
            }
            umma_commit(&tfull[buf]);  // also after a failed wait, so the epilogue is not left waiting
        }
        flags[2] = it;
        if (!ok) atomicExch(&flags[0], 1);
        umma_commit(done);
    } else if (warp >= 4) {
        // ---------------- epilogue: thread = (TMEM lane = channel, half of the token columns) ----------------
        const ConvEpi& e = p.conv;
        const int t = threadIdx.x - 128;        // 0..255
        const int quarter = warp & 3;           // TMEM lanes 32*quarter .. +31
        const int half = (warp - 4) >> 2;       // token columns 64*half .. +63
        int* tok_ok = meta;
        int* row_res = meta + 128;
        int* row_o32 = meta + 256;
        int* row_o16 = meta + 384;
        const float* res = reinterpret_cast<const float*>(e.res.ptr);
        float* o32 = reinterpret_cast<float*>(e.out32.ptr);
        __nv_bfloat16* o16 = reinterpret_cast<__nv_bfloat16*>(e.out16.ptr);
        int j = 0;
        for (int tile = blockIdx.x; tile < n_tiles; tile += gridDim.x, ++j) {
            const int buf = j & 1;
            const int tile_m = tile / n_tiles_n, tile_n = tile - tile_m * n_tiles_n;
            if (t < 128) {  // the token rows of this tile in the three views
                const int m_g = tile_m * BN + t;
                const int r = m_g < p.M ? m_g / e.T_rows : 0;
                const bool okm = m_g < p.M && (e.T_valid == 0 || m_g - r * e.T_rows < e.T_valid);
                const int t0 = okm ? (m_g - r * e.T_rows) * e.phases : 0;
                const int sl = (okm && e.row_slot) ? e.row_slot[r] : r;
                tok_ok[t] = okm;
                row_res[t] = (e.res.by_slot ? sl : r) * e.res.seq_rows + e.res.ctx + t0;
                row_o32[t] = (e.out32.by_slot ? sl : r) * e.out32.seq_rows + e.out32.ctx + t0;
                row_o16[t] = (e.out16.by_slot ? sl : r) * e.out16.seq_rows + e.out16.ctx + t0;
            }
            const bool got = mbar_wait(&tfull[buf], (uint32_t)(j >> 1) & 1u, DEV_ERR_GEMM_EPILOGUE);
            tc_fence_after();
            // uniform decision: every epilogue warp leaves together or none does
            if (epi_sync_or(!got || flags[0] != 0)) break;
            const int n_g = tile_n * 128 + quarter * 32 + lane;
            const bool colok = n_g < e.n_valid;
            const int ph = colok ? n_g / e.C_o : 0, c = colok ? n_g - ph * e.C_o : 0;
            const float b = (colok && p.bias) ? __bfloat162float(p.bias[n_g]) : 0.f;
            const float sc = (colok && e.scale) ? __bfloat162float(e.scale[c]) : 1.f;
            const float pa = (colok && e.act == ACT_SNAKE) ? e.act_p[c] : 0.f;
            const float pb = (colok && e.act == ACT_SNAKE) ? e.act_p[e.C_o + c] : 0.f;
#pragma unroll 1
            for (int c0 = half * 64; c0 < half * 64 + 64; c0 += 32) {
                float v[32];
                tmem_ld16(tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(buf * BN + c0),
                          *reinterpret_cast<float(*)[16]>(v));
                tmem_ld16(tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(buf * BN + c0 + 16),
                          *reinterpret_cast<float(*)[16]>(v + 16));
                if (!colok) continue;
                if (res) {
                    float rv[32];
#pragma unroll
                    for (int u = 0; u < 32; ++u)
                        rv[u] = tok_ok[c0 + u] ? res[(size_t)(row_res[c0 + u] + ph) * e.res.ld + c] : 0.f;
#pragma unroll
                    for (int u = 0; u < 32; ++u) v[u] = rv[u] + sc * (v[u] + b);
                } else {
#pragma unroll
                    for (int u = 0; u < 32; ++u) v[u] = sc * (v[u] + b);
                }
#pragma unroll
                for (int u = 0; u < 32; ++u) {
                    const int i = c0 + u;
                    if (!tok_ok[i]) continue;
                    float a = v[u];
                    if (o32) o32[(size_t)(row_o32[i] + ph) * e.out32.ld + c] = a;
                    if (o16) {
                        if (e.act == ACT_SNAKE) {
                            const float sn = __sinf(a * pa);
                            a = a + sn * sn * pb;
                        } else if (e.act == ACT_GELU) {
                            a = 0.5f * a * (1.0f + erff(a * 0.70710678118654752f));
                        }
                        o16[(size_t)(row_o16[i] + ph) * e.out16.ld + c] = __float2bfloat16(a);
                    }
                }
            }
            tc_fence_before();
            epi_sync_or(0);  // every epilogue thread is done with this accumulator and the token rows
            if (t == 0) mbar_arrive(&tempty[buf]);
        }
    }
    __syncthreads();
    if (threadIdx.x == 32) mbar_wait(done, 0, DEV_ERR_DRAIN);  // no UMMA still writes TMEM
    if (threadIdx.x == 0 && flags[0]) {
        // loads issued but never consumed must land before the CTA's shared memory is released
        for (int i = flags[2]; i < flags[1]; ++i) mbar_wait(&full[i % S], (uint32_t)(i / S) & 1u, DEV_ERR_DRAIN);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tmem, 2 * BN);
}

// ---------------------------------------------------------------------------
// host side: tensor maps and launch
// ---------------------------------------------------------------------------
// 2-D bf16 row-major [rows, cols] map with a (64 x box_rows) box and 128-B swizzle.
inline int make_map_bf16(CUtensorMap* map, const void* ptr, uint64_t rows, uint64_t cols, uint32_t box_rows) {
    PFN_encodeTiled enc = get_encode_fn();
    if (!enc) {
        set_error("cuTensorMapEncodeTiled unavailable");
        return QTTS_ERR_CUDA;
    }
    if ((reinterpret_cast<uintptr_t>(ptr) & 15) != 0 || (cols * 2) % 16 != 0) {
        set_error("tensor map needs a 16-byte aligned base and row pitch");
        return QTTS_ERR_INVALID;
    }
    cuuint64_t dims[2] = {cols, rows};
    cuuint64_t strides[1] = {cols * 2};
    cuuint32_t box[2] = {64, box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        set_error("cuTensorMapEncodeTiled failed (%d)", (int)r);
        return QTTS_ERR_CUDA;
    }
    return QTTS_OK;
}

// Token-tile width.  With QTTS_GEMM_BN32=1 (opt-in), up to 64 tokens run as 32-token tiles:
// each weight tile is read by two CTAs but a CTA's split-K partial and its share of the cluster
// exchange halve.  Measured slower on the decode step (9 808 vs 10 142 frames/s).
inline bool gemm_bn32() {
    static const bool on = [] {
        const char* v = getenv("QTTS_GEMM_BN32");
        return v && *v == '1';
    }();
    return on;
}
// Rows up to QTTS_GEMM_BN64_MAX_M (default 128: the code predictor's two-row first stage, +2 %
// over 128-token tiles) use 64-token tiles; more rows use 128-token tiles.
inline int gemm_bn64_max_m() {
    static const int m = [] {
        const char* v = getenv("QTTS_GEMM_BN64_MAX_M");
        return (v && *v) ? atoi(v) : 128;
    }();
    return m;
}
inline int pick_bn(int M) { return M <= 64 ? (gemm_bn32() ? 32 : 64) : (M <= gemm_bn64_max_m() ? 64 : 128); }

// Persistent conv GEMMs for wide rows: opt-in (QTTS_GEMM_PERSIST=1).  At the decoder's
// sizes they measured slower than the two-CTAs-per-SM form (2.43 vs 1.64 ms per
// 64-stream step): eight epilogue warps per SM issue 4x the memory instructions
// of the smem-staged float4 epilogue, and a 4-stage ring holds less in flight.
inline bool gemm_persist_enabled() {
    static const bool on = [] {
        const char* v = getenv("QTTS_GEMM_PERSIST");
        return v && *v == '1';
    }();
    return on;
}

// Paired QKV launches use clusters of 2 x splits CTAs; above 8 (portable) the kernel opts in to
// non-portable cluster sizes (up to 16).  QTTS_GEMM_PAIR_SPLITS caps splits (default 8).
inline int gemm_pair_max_splits() {
    static const int s = [] {
        const char* v = getenv("QTTS_GEMM_PAIR_SPLITS");
        const int x = (v && *v) ? atoi(v) : 8;
        return x < 1 ? 1 : (x > 8 ? 8 : x);
    }();
    return s;
}

inline bool gemm_push_enabled() {
    static const bool on = [] {
        const char* v = getenv("QTTS_GEMM_PUSH");
        return v && *v == '1';
    }();
    return on;
}

// Tuning knobs read once from the environment (defaults are the measured best; a 2-stage ring,
// globally or only for CTAs with at most two k-blocks, measured 2-3 % slower on the decode step):
// QTTS_GEMM_STAGES (pipeline depth of the hi/lo kernel at BN = 64) and
// QTTS_GEMM_MAX_SPLITS (largest split-K cluster), QTTS_GEMM_CTAS_PER_SM (split-K target).
inline int env_int(const char* name, int dflt) {
    const char* v = getenv(name);
    return (v && *v) ? atoi(v) : dflt;
}
inline int gemm_stages() {
    static const int s = env_int("QTTS_GEMM_STAGES", 3);
    return s;
}
inline int gemm_max_splits() {
    static const int s = env_int("QTTS_GEMM_MAX_SPLITS", 8);
    return s;
}
inline int gemm_ctas_per_sm() {
    static const int s = env_int("QTTS_GEMM_CTAS_PER_SM", 2);
    return s;
}

// Split-K factor: powers of two up to about `ctas_per_sm` CTAs per SM, at least two k-blocks
// per CTA.  Filling every SM with exactly two CTAs measured slower: splits of 3 (talker
// gate/up, 288 CTAs) 23.8 vs 17.8 us with 2, splits of 6 (code-predictor gate/up) 14.4 vs
// 9.6 us with 4.  (The kernel takes any factor: token slices differ by at most one.)
inline int pick_splits(int N, int M, int K, int BN) {
    const int tiles = (N / 128) * ceil_div(M, BN);
    const int kb = K / 64;
    const int target = gemm_ctas_per_sm() * num_sms();
    int s = 1;
    while (s * 2 <= gemm_max_splits() && tiles * s * 2 <= target + target / 5 && kb / (s * 2) >= 2 &&
           BN / (s * 2) >= 4)
        s *= 2;
    return s;
}

template <int BN, int STAGES, bool SPLIT, int NT = 128, bool PUSH = false>
inline int launch_gemm_t(const CUtensorMap& mw, const CUtensorMap& mx, const CUtensorMap& mxlo, const GemmParams& p,
                         cudaStream_t st) {
    using L = GemmLayout<BN, STAGES, SPLIT, PUSH>;
    auto kern = gemm_tc_kernel<BN, STAGES, SPLIT, NT, PUSH>;
    QTTS_CHECK_CUDA((func_attr_once<gemm_tc_kernel<BN, STAGES, SPLIT, NT, PUSH>>(L::SMEM, /*nonportable_cluster=*/true)));
    QTTS_CHECK_CUDA(launch_pdl(kern, dim3(p.N / 128, p.splits, ceil_div(p.M, BN)), dim3(NT, 1, 1), L::SMEM, st,
                               dim3(p.pair.on ? 2 : 1, p.splits, 1), mw, mx, mxlo, p));
    return QTTS_OK;
}

// Prepared GEMM: tensor maps built once (two token-tile heights, optional lo operand), reused every step.
struct GemmPlan {
    CUtensorMap mw, mx32, mx64, mx128, mlo32, mlo64, mlo128;
    GemmParams p;
    bool split;
    const void* w;       // the weight matrix [N][K] bf16
    size_t w_bytes;
};

// Prefetch `next`'s weights into L2 from the launches of `g` (see GemmParams::l2_next).
inline void gemm_chain_l2(GemmPlan& g, const GemmPlan& next) {
    g.p.l2_next = reinterpret_cast<const uint8_t*>(next.w);
    g.p.l2_next_bytes = next.w_bytes;
}

inline int gemm_plan(GemmPlan* g, const void* X, int rows, int K, const void* W, int N, int epilogue, void* out,
                     const void* bias, const qtts_qkv_epilogue* qkv, const void* X_lo = nullptr,
                     void* out_lo = nullptr) {
    if (N % 128 != 0 || K % 64 != 0 || rows <= 0) {
        set_error("gemm: need N %% 128 == 0, K %% 64 == 0, rows > 0 (N=%d K=%d rows=%d)", N, K, rows);
        return QTTS_ERR_UNSUPPORTED;
    }
    if (epilogue == QTTS_EPI_QKV_ROPE && (!qkv || qkv->head_dim % 32 != 0 || 128 % qkv->head_dim != 0)) {
        set_error("gemm: QKV epilogue needs head_dim in {32, 64, 128}");
        return QTTS_ERR_UNSUPPORTED;
    }
    int rc = make_map_bf16(&g->mw, W, (uint64_t)N, (uint64_t)K, 128);
    if (rc) return rc;
    rc = make_map_bf16(&g->mx32, X, (uint64_t)rows, (uint64_t)K, 32);
    if (rc) return rc;
    rc = make_map_bf16(&g->mx64, X, (uint64_t)rows, (uint64_t)K, 64);
    if (rc) return rc;
    rc = make_map_bf16(&g->mx128, X, (uint64_t)rows, (uint64_t)K, 128);
    if (rc) return rc;
    g->split = X_lo != nullptr;
    if (g->split) {
        rc = make_map_bf16(&g->mlo32, X_lo, (uint64_t)rows, (uint64_t)K, 32);
        if (rc) return rc;
        rc = make_map_bf16(&g->mlo64, X_lo, (uint64_t)rows, (uint64_t)K, 64);
        if (rc) return rc;
        rc = make_map_bf16(&g->mlo128, X_lo, (uint64_t)rows, (uint64_t)K, 128);
        if (rc) return rc;
    } else {
        g->mlo32 = g->mx32;
        g->mlo64 = g->mx64;
        g->mlo128 = g->mx128;
    }
    g->w = W;
    g->w_bytes = (size_t)N * K * sizeof(__nv_bfloat16);
    GemmParams& p = g->p;
    memset(&p, 0, sizeof(p));
    p.M = rows;
    p.N = N;
    p.K = K;
    p.kblocks = K / 64;
    p.splits = 1;
    p.epilogue = epilogue;
    p.out = out;
    p.out_lo = out_lo;
    p.bias = reinterpret_cast<const __nv_bfloat16*>(bias);
    if (qkv) p.qkv = *qkv;
    return QTTS_OK;
}

// Implicit-convolution plan: X is a slot-indexed history buffer H [(slots) * seq_rows][cpad]
// (bf16, cpad % 64 == 0), K = taps * cpad; a launch needs rows per stream (ix.T) % 128 == 0,
// which callers reach by padding each stream's rows (ConvEpi::T_valid marks the real ones).
inline int gemm_plan_implicit(GemmPlan* g, const void* H, int total_rows, int cpad, int taps, int dil, int T,
                              int seq_rows, int max_rows, const void* W, int N, const void* bias, const ConvEpi& e) {
    if (cpad % 64 != 0 || N % 128 != 0) {
        set_error("implicit conv: need channels %% 64 == 0, N %% 128 == 0");
        return QTTS_ERR_UNSUPPORTED;
    }
    const int K = taps * cpad;
    int rc = make_map_bf16(&g->mw, W, (uint64_t)N, (uint64_t)K, 128);
    if (rc) return rc;
    rc = make_map_bf16(&g->mx128, H, (uint64_t)total_rows, (uint64_t)cpad, 128);
    if (rc) return rc;
    g->mx32 = g->mx128;
    g->mx64 = g->mx128;
    g->mlo32 = g->mx128;
    g->mlo64 = g->mx128;
    g->mlo128 = g->mx128;
    g->split = false;
    GemmParams& p = g->p;
    memset(&p, 0, sizeof(p));
    p.M = max_rows;
    p.N = N;
    p.K = K;
    p.kblocks = K / 64;
    p.splits = 1;
    p.epilogue = kEpiConv;
    p.bias = reinterpret_cast<const __nv_bfloat16*>(bias);
    p.conv = e;
    p.ix.on = 1;
    p.ix.T = T;
    p.ix.seq_rows = seq_rows;
    p.ix.dil = dil;
    p.ix.cblocks = cpad / 64;
    return QTTS_OK;
}

// Worth it once every SM gets two or more tiles (QTTS_GEMM_PERSIST_MIN_TILES overrides the threshold).
inline bool gemm_persist_ok(const GemmPlan& g, int M) {
    static const int min_tiles = env_int("QTTS_GEMM_PERSIST_MIN_TILES", 2 * num_sms());
    const int tiles = (g.p.N / 128) * ceil_div(M, 128);
    return !g.split && g.p.epilogue == kEpiConv && tiles >= min_tiles;
}

inline int launch_gemm_persist(const GemmPlan& g, const GemmParams& p, cudaStream_t st) {
    using L = PersistLayout;
    QTTS_CHECK_CUDA((func_attr_once<gemm_conv_persist_kernel>(L::SMEM)));
    // QTTS_GEMM_PERSIST_CTAS caps the grid (e.g. to leave SMs to a concurrent stream)
    static const int cap = env_int("QTTS_GEMM_PERSIST_CTAS", num_sms());
    const int tiles = (p.N / 128) * ceil_div(p.M, 128);
    const int grid = tiles < cap ? tiles : cap;
    QTTS_CHECK_CUDA(launch_pdl(gemm_conv_persist_kernel, dim3(grid), dim3(kPersistThreads), L::SMEM, st,
                               dim3(1, 1, 1), g.mw, g.mx128, p));
    return QTTS_OK;
}

// Launch on the first M rows of the plan's X buffer(s).
inline int gemm_run(GemmPlan g, int M, cudaStream_t st, void* out = nullptr) {
    if (M <= 0) return QTTS_OK;
    const int bn = g.p.ix.on ? 128 : pick_bn(M);  // implicit convolutions tile whole 128-row stream blocks
    if (g.p.ix.on && (bn != 128 || M % g.p.ix.T != 0)) {
        set_error("implicit conv: rows must be whole streams of T >= 128 steps (M=%d T=%d)", M, g.p.ix.T);
        return QTTS_ERR_INVALID;
    }
    g.p.M = M;
    g.p.splits = pick_splits(g.p.N, M, g.p.K, bn);
    if (g.p.pair.on && g.p.splits > gemm_pair_max_splits()) g.p.splits = gemm_pair_max_splits();
    if (out) g.p.out = out;
    // Opt-in (QTTS_GEMM_PUSH=1): split-K launches that fit one CTA per SM reduce by
    // pushing partials from registers into the owner's receive buffer (5-stage ring +
    // 32 KB receive buffer).  Measured slower in the decode step (9.28 vs 7.65 ms): the
    // 196 KB footprint keeps the next kernel's CTAs off the SM until this one exits, so
    // programmatic dependent launch no longer overlaps their weight prefetch, and the
    // remote stores cost about what the pull's remote loads do.
    const bool push = bn == 64 && g.p.splits > 1 && 64 % g.p.splits == 0 && !g.p.pair.on && gemm_push_enabled() &&
                      (g.p.N / 128) * g.p.splits * ceil_div(M, bn) <= num_sms();
    if (push) {
        if (g.split) return launch_gemm_t<64, 5, true, 128, true>(g.mw, g.mx64, g.mlo64, g.p, st);
        return launch_gemm_t<64, 5, false, 128, true>(g.mw, g.mx64, g.mx64, g.p, st);
    }
    if (bn == 32) {
        if (g.split) return launch_gemm_t<32, 3, true>(g.mw, g.mx32, g.mlo32, g.p, st);
        return launch_gemm_t<32, 4, false>(g.mw, g.mx32, g.mx32, g.p, st);
    }
    if (g.split) {
        if (bn == 64) {
            switch (gemm_stages()) {
                case 2: return launch_gemm_t<64, 2, true>(g.mw, g.mx64, g.mlo64, g.p, st);
                case 4: return launch_gemm_t<64, 4, true>(g.mw, g.mx64, g.mlo64, g.p, st);
                case 6: return launch_gemm_t<64, 6, true>(g.mw, g.mx64, g.mlo64, g.p, st);
                default: return launch_gemm_t<64, 3, true>(g.mw, g.mx64, g.mlo64, g.p, st);
            }
        }
        return launch_gemm_t<128, 3, true>(g.mw, g.mx128, g.mlo128, g.p, st);
    }
    if (bn == 64) return launch_gemm_t<64, 4, false>(g.mw, g.mx64, g.mx64, g.p, st);
    if (gemm_persist_enabled() && gemm_persist_ok(g, M)) {
        g.p.splits = 1;
        return launch_gemm_persist(g, g.p, st);
    }
    // wide-row (convolution) GEMMs: 3 x 32 KB stages keep two CTAs per SM, so one
    // CTA's epilogue overlaps the other's main loop, and 8 warps share the epilogue
    if (g.p.epilogue == QTTS_EPI_QKV_ROPE) return launch_gemm_t<128, 3, false, 128>(g.mw, g.mx128, g.mx128, g.p, st);
    return launch_gemm_t<128, 3, false, 256>(g.mw, g.mx128, g.mx128, g.p, st);
}

}  // namespace qtts
