// Paged GQA attention over the block pool (decode and chunked prefill rows).
//
// One CTA per (query row, kv head, split of QTTS_ATTN_SPLIT_BLOCKS blocks).
// Each of the 4 warps owns every 4th KV block of the split and streams it
// through its own STAGES-deep ring in shared memory: lane 0 issues two bulk
// copies (K chunk and V chunk of one block, head, layer: block_size x D bf16,
// contiguous in the pool) completing on the stage's mbarrier.
//
// With 2 query heads per kv head and 16-token blocks a block has exactly 32
// (head, token) score pairs.  Each lane computes partial dot products over its
// D/32 dimensions for all 32 pairs, then a 5-step butterfly reduce-scatter
// leaves lane l with the full score of pair l (head l>>4, token l&15): 31
// shuffles per block instead of 160.  Online softmax runs in the log2 domain;
// P·V broadcasts each probability with one shuffle.  The four warps merge in
// shared memory, and the split partials (unnormalised o, running max, sum)
// go to a caller-provided workspace that attn_combine_kernel folds.
//
// Semantics: softmax(q k^T / sqrt(D)) v over the row's first row_ctx keys —
// talker_unified_modules.py:192-200 with the padding bias of
// batch_helper.py:48-66 and the causal mask of talker_unified_modules.py:282-288
// expressed as a per-row key count.
#pragma once

#include "common.cuh"

namespace qtts {

struct AttnParams {
    const float* q;  // [R][num_heads][D] fp32
    const kv_t* kv;
    int num_heads, kv_heads;
    int layer, num_layers, block_size, num_blocks;
    const int32_t* block_table;
    int mbps;
    const int32_t* row_slot;
    const int32_t* row_ctx;
    int max_splits;
    float scale_log2;  // log2(e) / sqrt(D)
    float* ws_o;
    float* ws_ml;
    __nv_bfloat16* out;
    __nv_bfloat16* out_lo;  // bf16 residual of the output (hi/lo GEMM operand), or NULL
    int R;
};

constexpr int kAttnStages = 3;

template <int D>
struct AttnLayout {
    static constexpr int CHUNK = 16 * D * 2;  // one block's K (or V) for one head, bytes
    static constexpr int STAGE = 2 * CHUNK;
    static constexpr int WARP_BYTES = kAttnStages * STAGE;
    static constexpr int SMEM = 128 + 4 * WARP_BYTES + 4 * kAttnStages * 8;
};

template <int D>
__device__ __forceinline__ void load_row(const kv_t* base, int lane, float (&v)[D / 32]) {
    if constexpr (D == 128) {
        const uint2 raw = *reinterpret_cast<const uint2*>(base + lane * 4);
        const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&raw.x));
        const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&raw.y));
        v[0] = a.x;
        v[1] = a.y;
        v[2] = b.x;
        v[3] = b.y;
    } else if constexpr (D == 64) {
        const float2 a = __half22float2(*reinterpret_cast<const __half2*>(base + lane * 2));
        v[0] = a.x;
        v[1] = a.y;
    } else {
        v[0] = __half2float(base[lane]);
    }
}

template <int D>
__global__ void __launch_bounds__(128) paged_attn_kernel(const AttnParams p) {
    using L = AttnLayout<D>;
    constexpr int DPL = D / 32;  // dims per lane
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~uintptr_t(127));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + 4 * L::WARP_BYTES);

    const int r = blockIdx.x, g = blockIdx.y, sp = blockIdx.z;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    griddep_wait();
    griddep_launch();
    const int ctx = p.row_ctx[r];
    const int nbt = (ctx + 15) >> 4;
    const int b_start = sp * QTTS_ATTN_SPLIT_BLOCKS;
    const int b_end = min(nbt, b_start + QTTS_ATTN_SPLIT_BLOCKS);
    if (b_start >= b_end) {  // uniform for the CTA
        if (nbt == 0 && sp == 0) {  // a row with no keys (only after a scheduler error): zero output
            for (int i = threadIdx.x; i < 2 * D; i += blockDim.x) {
                const size_t o = ((size_t)r * p.num_heads + g * 2) * D + i;
                p.out[o] = __float2bfloat16(0.f);
                if (p.out_lo) p.out_lo[o] = __float2bfloat16(0.f);
            }
        }
        return;
    }
    const int slot = p.row_slot[r];

    // q for the two heads of this kv group, pre-scaled into the log2 domain
    float q0[DPL], q1[DPL];
    {
        const float* qb = p.q + ((size_t)r * p.num_heads + g * 2) * D;
#pragma unroll
        for (int j = 0; j < DPL; ++j) {
            q0[j] = qb[lane * DPL + j] * p.scale_log2;
            q1[j] = qb[D + lane * DPL + j] * p.scale_log2;
        }
    }

    uint8_t* wbuf = smem + warp * L::WARP_BYTES;
    uint64_t* wbar = bars + warp * kAttnStages;
    if (lane == 0)
        for (int s = 0; s < kAttnStages; ++s) mbar_init(&wbar[s], 1);
    __syncwarp();
    fence_mbar_init();

    const int n_mine = b_end - b_start > warp ? (b_end - b_start - warp + 3) / 4 : 0;
    const size_t head_stride = (size_t)16 * D;
    auto issue = [&](int i) {
        const int jb = b_start + warp + 4 * i;
        const int s = i % kAttnStages;
        int blk = jb < p.mbps ? p.block_table[(size_t)slot * p.mbps + jb] : -1;
        if (blk < 0 || blk >= p.num_blocks) {
            record_error(DEV_ERR_ATTN_WAIT);
            blk = 0;  // stay in bounds; the error word reports the bad table entry
        }
        const kv_t* kp =
            p.kv + ((((size_t)blk * p.num_layers + p.layer) * 2 + 0) * p.kv_heads + g) * head_stride;
        const kv_t* vp = kp + (size_t)p.kv_heads * head_stride;
        uint8_t* dst = wbuf + s * L::STAGE;
        mbar_arrive_expect_tx(&wbar[s], L::STAGE);
        bulk_load(dst, kp, L::CHUNK, &wbar[s]);
        bulk_load(dst + L::CHUNK, vp, L::CHUNK, &wbar[s]);
    };

    int issued = 0;
    if (lane == 0) {
        for (int i = 0; i < n_mine && i < kAttnStages; ++i) issue(i);
        issued = min(n_mine, kAttnStages);
    }
    issued = __shfl_sync(0xffffffffu, issued, 0);

    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
    float o0[DPL], o1[DPL];
#pragma unroll
    for (int j = 0; j < DPL; ++j) o0[j] = o1[j] = 0.f;

    int done = 0;
    bool failed = false;
    for (int i = 0; i < n_mine; ++i) {
        const int s = i % kAttnStages;
        if (!mbar_wait(&wbar[s], (uint32_t)(i / kAttnStages) & 1u, DEV_ERR_ATTN_WAIT)) {
            failed = true;
            break;
        }
        const kv_t* Kb = reinterpret_cast<const kv_t*>(wbuf + s * L::STAGE);
        const kv_t* Vb = Kb + 16 * D;
        const int jb = b_start + warp + 4 * i;

        // ---- scores: partials for 32 (head, token) pairs, then reduce-scatter
        float part[32];
#pragma unroll
        for (int t = 0; t < 16; ++t) {
            float k[DPL];
            load_row<D>(Kb + t * D, lane, k);
            float a = 0.f, b = 0.f;
#pragma unroll
            for (int j = 0; j < DPL; ++j) {
                a = fmaf(q0[j], k[j], a);
                b = fmaf(q1[j], k[j], b);
            }
            part[t] = a;
            part[16 + t] = b;
        }
#pragma unroll
        for (int w = 16; w >= 1; w >>= 1) {
            const bool upper = (lane & w) != 0;
#pragma unroll
            for (int i2 = 0; i2 < w; ++i2) {
                const float send = upper ? part[i2] : part[i2 + w];
                const float keep = upper ? part[i2 + w] : part[i2];
                part[i2] = keep + __shfl_xor_sync(0xffffffffu, send, w);
            }
        }
        const int tok = jb * 16 + (lane & 15);
        const float sc = tok < ctx ? part[0] : -INFINITY;

        // ---- online softmax (lanes 0-15: head 0, lanes 16-31: head 1)
        float mb = sc;
#pragma unroll
        for (int o = 8; o >= 1; o >>= 1) mb = fmaxf(mb, __shfl_xor_sync(0xffffffffu, mb, o));
        const float mb_other = __shfl_xor_sync(0xffffffffu, mb, 16);
        const float mb0 = lane < 16 ? mb : mb_other;
        const float mb1 = lane < 16 ? mb_other : mb;
        const float mn0 = fmaxf(m0, mb0), mn1 = fmaxf(m1, mb1);
        const float a0 = m0 == -INFINITY ? 0.f : exp2f(m0 - mn0);
        const float a1 = m1 == -INFINITY ? 0.f : exp2f(m1 - mn1);
        const float mine = lane < 16 ? mn0 : mn1;
        const float pr = sc == -INFINITY ? 0.f : exp2f(sc - mine);
        float ps = pr;
#pragma unroll
        for (int o = 8; o >= 1; o >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, o);
        const float ps_other = __shfl_xor_sync(0xffffffffu, ps, 16);
        l0 = l0 * a0 + (lane < 16 ? ps : ps_other);
        l1 = l1 * a1 + (lane < 16 ? ps_other : ps);
        m0 = mn0;
        m1 = mn1;
#pragma unroll
        for (int j = 0; j < DPL; ++j) {
            o0[j] *= a0;
            o1[j] *= a1;
        }
        // ---- P V
#pragma unroll
        for (int t = 0; t < 16; ++t) {
            const float p0 = __shfl_sync(0xffffffffu, pr, t);
            const float p1 = __shfl_sync(0xffffffffu, pr, 16 + t);
            float v[DPL];
            load_row<D>(Vb + t * D, lane, v);
#pragma unroll
            for (int j = 0; j < DPL; ++j) {
                o0[j] = fmaf(p0, v[j], o0[j]);
                o1[j] = fmaf(p1, v[j], o1[j]);
            }
        }
        ++done;
        __syncwarp();
        if (lane == 0 && i + kAttnStages < n_mine) {
            fence_proxy_async_smem();
            issue(i + kAttnStages);
            ++issued;
        }
        issued = __shfl_sync(0xffffffffu, issued, 0);
    }
    if (failed && lane == 0) {
        for (int i = done; i < issued; ++i)
            mbar_wait(&wbar[i % kAttnStages], (uint32_t)(i / kAttnStages) & 1u, DEV_ERR_DRAIN);
    }
    __syncthreads();

    // ---- merge the four warps (reuse the stage buffers)
    float* red = reinterpret_cast<float*>(smem);  // [4 warps][2 heads][D + 2]
    constexpr int RS = D + 2;
#pragma unroll
    for (int j = 0; j < DPL; ++j) {
        red[(warp * 2 + 0) * RS + lane * DPL + j] = o0[j];
        red[(warp * 2 + 1) * RS + lane * DPL + j] = o1[j];
    }
    if (lane == 0) {
        red[(warp * 2 + 0) * RS + D] = n_mine > 0 ? m0 : -INFINITY;
        red[(warp * 2 + 0) * RS + D + 1] = n_mine > 0 ? l0 : 0.f;
        red[(warp * 2 + 1) * RS + D] = n_mine > 0 ? m1 : -INFINITY;
        red[(warp * 2 + 1) * RS + D + 1] = n_mine > 0 ? l1 : 0.f;
    }
    __syncthreads();
    for (int idx = threadIdx.x; idx < 2 * D; idx += blockDim.x) {
        const int h = idx / D, d = idx % D;
        float M = -INFINITY;
        for (int w = 0; w < 4; ++w) M = fmaxf(M, red[(w * 2 + h) * RS + D]);
        float acc = 0.f, lsum = 0.f;
        for (int w = 0; w < 4; ++w) {
            const float mw = red[(w * 2 + h) * RS + D];
            const float f = mw == -INFINITY ? 0.f : exp2f(mw - M);
            acc += red[(w * 2 + h) * RS + d] * f;
            lsum += red[(w * 2 + h) * RS + D + 1] * f;
        }
        const size_t hrow = (size_t)r * p.num_heads + g * 2 + h;
        if (nbt <= QTTS_ATTN_SPLIT_BLOCKS) {
            // the row has a single split: finish here, the combine kernel skips it
            const float o = lsum > 0.f ? acc / lsum : 0.f;
            const __nv_bfloat16 hi = __float2bfloat16(o);
            p.out[hrow * D + d] = hi;
            if (p.out_lo) p.out_lo[hrow * D + d] = __float2bfloat16(o - __bfloat162float(hi));
            continue;
        }
        p.ws_o[(hrow * p.max_splits + sp) * D + d] = acc;
        if (d == 0) {
            p.ws_ml[(hrow * p.max_splits + sp) * 2 + 0] = M;
            p.ws_ml[(hrow * p.max_splits + sp) * 2 + 1] = lsum;
        }
    }
}

// Fold split partials: out = Σ_s o_s 2^(m_s - M) / Σ_s l_s 2^(m_s - M), bf16.
template <int D>
__global__ void attn_combine_kernel(const AttnParams p) {
    const int r = blockIdx.x, h = blockIdx.y, d = threadIdx.x;
    griddep_wait();
    griddep_launch();
    const int ctx = p.row_ctx[r];
    const int nbt = (ctx + 15) >> 4;
    const int ns = min(p.max_splits, (nbt + QTTS_ATTN_SPLIT_BLOCKS - 1) / QTTS_ATTN_SPLIT_BLOCKS);
    if (ns <= 1) return;  // single-split (and empty) rows were finished by paged_attn_kernel
    const size_t hrow = (size_t)r * p.num_heads + h;
    float M = -INFINITY;
    for (int s = 0; s < ns; ++s) M = fmaxf(M, p.ws_ml[(hrow * p.max_splits + s) * 2]);
    float acc = 0.f, lsum = 0.f;
    for (int s = 0; s < ns; ++s) {
        const float ms = p.ws_ml[(hrow * p.max_splits + s) * 2];
        const float f = ms == -INFINITY ? 0.f : exp2f(ms - M);
        acc += p.ws_o[(hrow * p.max_splits + s) * D + d] * f;
        lsum += p.ws_ml[(hrow * p.max_splits + s) * 2 + 1] * f;
    }
    const float o = lsum > 0.f ? acc / lsum : 0.f;
    const __nv_bfloat16 hi = __float2bfloat16(o);
    p.out[hrow * D + d] = hi;
    if (p.out_lo) p.out_lo[hrow * D + d] = __float2bfloat16(o - __bfloat162float(hi));
}

inline int attn_max_splits(int max_ctx) {
    const int nb = (max_ctx + 15) / 16;
    const int s = (nb + QTTS_ATTN_SPLIT_BLOCKS - 1) / QTTS_ATTN_SPLIT_BLOCKS;
    return s > 1 ? s : 1;
}

template <int D>
inline int launch_attention_d(const AttnParams& p, cudaStream_t st) {
    using L = AttnLayout<D>;
    static bool attr = false;
    if (!attr) {
        QTTS_CHECK_CUDA(cudaFuncSetAttribute(paged_attn_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, L::SMEM));
        attr = true;
    }
    QTTS_LAUNCH(paged_attn_kernel<D>, dim3(p.R, p.kv_heads, p.max_splits), dim3(128), L::SMEM, st, p);
    if (p.max_splits > 1)  // otherwise every row finished inside paged_attn_kernel
        QTTS_LAUNCH(attn_combine_kernel<D>, dim3(p.R, p.num_heads), dim3(D), 0, st, p);
    return QTTS_OK;
}

inline int launch_attention(const AttnParams& p, int head_dim, cudaStream_t st) {
    if (p.R <= 0) return QTTS_OK;
    switch (head_dim) {
        case 128: return launch_attention_d<128>(p, st);
        case 64: return launch_attention_d<64>(p, st);
        case 32: return launch_attention_d<32>(p, st);
        default:
            set_error("paged attention: head_dim %d not supported (32, 64 or 128)", head_dim);
            return QTTS_ERR_UNSUPPORTED;
    }
}

}  // namespace qtts
