// Paged GQA attention over the block pool (decode and chunked prefill rows).
//
// One CTA per (query row, kv head, split of split_blocks KV blocks).
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
    int split_blocks;  // KV blocks per split (QTTS_ATTN_SPLIT_BLOCKS unless a caller sizes its scratch for another)
    float scale_log2;  // log2(e) / sqrt(D)
    float* ws_o;
    float* ws_ml;
    __nv_bfloat16* out;
    __nv_bfloat16* out_lo;  // bf16 residual of the output (hi/lo GEMM operand), or NULL
    int R;
    int static_meta;  // row_slot / row_ctx / block_table are not written by earlier kernels of the
                      // stream, so a kernel may read them before waiting on its predecessor
    int rows_per_stream;  // chunked prefill: rows come as R / rows_per_stream streams of this many
                          // consecutive query tokens (0 or 1: independent rows)
    int meta_settled;  // decode rows whose row_slot / row_ctx / block_table and every key but each
                       // row's newest were written at least two launches earlier: the row kernel
                       // reads them and starts its first loads before waiting on its predecessor
};

// Ring depth per warp (QTTS_ATTN_STAGES, default below): 3 stages x 8 KB x 4
// warps hold 2 CTAs per SM; 2 stages hold 3.
inline int attn_stages() {
    static const int s = [] {
        const char* v = getenv("QTTS_ATTN_STAGES");
        const int x = (v && *v) ? atoi(v) : 2;
        return (x == 2 || x == 3 || x == 4) ? x : 2;
    }();
    return s;
}

template <int D, int STAGES>
struct AttnLayout {
    static constexpr int CHUNK = 16 * D * 2;  // one block's K (or V) for one head, bytes
    static constexpr int STAGE = 2 * CHUNK;
    static constexpr int WARP_BYTES = STAGES * STAGE;
    static constexpr int SMEM = 128 + 4 * WARP_BYTES + 4 * STAGES * 8;
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

template <int D, int kAttnStages>
__global__ void __launch_bounds__(128) paged_attn_kernel(const AttnParams p) {
    using L = AttnLayout<D, kAttnStages>;
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
    const int b_start = sp * p.split_blocks;
    const int b_end = min(nbt, b_start + p.split_blocks);
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
        if (nbt <= p.split_blocks) {
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

// ---------------------------------------------------------------------------
// head_dim 128: one warp per (split, row, kv head) work item, each with its own
// ring of whole blocks and no cross-warp merge, so a CTA is four independent
// streams and a layer's items fit in about one wave; the per-block math runs on
// the tensor pipe (warp-level mma.sync, m16n8k16, fp16 inputs, fp32
// accumulators).
//
// The K and V chunks of a block come in by TMA as two 16 x 64 boxes each with
// the 128-B swizzle, so the ldmatrix row reads below hit eight different
// bank groups.  Per 16-token block and warp:
//   S^T[16 tok][8] = K[16][128] · Q^T[128][8]   (8 k-steps; Q^T columns 0, 1 =
//                     the two q heads, carried as an fp16 hi/lo pair so the
//                     scores keep ~fp32 accuracy; columns 2..7 zero)
//   online softmax on the 32 real scores (lanes 4k hold tokens k, k+8)
//   O^T[128][8] += V^T[128][16] · P^T[16][8]    (8 m-tiles; P as fp16 hi/lo)
// ~130 instructions per block instead of ~900 for the same math on FMAs.
// ---------------------------------------------------------------------------
constexpr int kTcBox = 16 * 128;         // one 16-token x 64-dim fp16 box, bytes
constexpr int kTcStage = 4 * kTcBox;     // K dims 0-63, K 64-127, V 0-63, V 64-127

template <int S>
struct AttnTcLayout {
    static constexpr int WARP_BYTES = S * kTcStage;
    static constexpr int SMEM = 1024 + 4 * WARP_BYTES + 4 * S * 8;
};

// byte address (shared window) of the 16-B chunk holding (row, dim..dim+7) of a
// [16 rows][128 dims] tile stored as two swizzled 16 x 64 boxes
__device__ __forceinline__ uint32_t tc_sw128(uint32_t tile, int row, int dim) {
    return tile + (uint32_t)((dim >> 6) * kTcBox + row * 128 + ((((dim & 63) >> 3) ^ (row & 7)) << 4));
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t (&r)[4]) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t (&r)[4]) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}

__device__ __forceinline__ void mma_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack_h2(float a, float b) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
}

// (hi, lo) fp16 pairs of two floats: hi = fp16(x), lo = fp16(x - hi)
__device__ __forceinline__ void split_h2(float a, float b, uint32_t& hi, uint32_t& lo) {
    const __half2 h = __floats2half2_rn(a, b);
    const float2 hf = __half22float2(h);
    hi = *reinterpret_cast<const uint32_t*>(&h);
    lo = pack_h2(a - hf.x, b - hf.y);
}

template <int S>
__global__ void __launch_bounds__(128) paged_attn_tc_kernel(const __grid_constant__ CUtensorMap tmKV,
                                                            const AttnParams p) {
    constexpr int D = 128;
    using L = AttnTcLayout<S>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + 4 * L::WARP_BYTES);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int gq = lane >> 2, qq = lane & 3;  // mma fragment coordinates
    griddep_wait();
    griddep_launch();
    // work item of this warp: (split, row, kv head), heads fastest, so the four warps
    // of a CTA share a row and have the same amount of work
    const int item = blockIdx.x * 4 + warp;
    if (item >= p.R * p.kv_heads * p.max_splits) return;  // warp-uniform
    const int g = item % p.kv_heads;
    const int r = (item / p.kv_heads) % p.R;
    const int sp = item / (p.kv_heads * p.R);
    const int ctx = p.row_ctx[r];
    const int nbt = (ctx + 15) >> 4;
    const int b_start = sp * p.split_blocks;
    const int b_end = min(nbt, b_start + p.split_blocks);
    const size_t hrow0 = (size_t)r * p.num_heads + g * 2;
    if (b_start >= b_end) {
        if (nbt == 0 && sp == 0) {  // a row with no keys (only after a scheduler error): zero output
            for (int i = lane; i < 2 * D; i += 32) {
                p.out[hrow0 * D + i] = __float2bfloat16(0.f);
                if (p.out_lo) p.out_lo[hrow0 * D + i] = __float2bfloat16(0.f);
            }
        }
        return;
    }
    const int slot = p.row_slot[r];

    // Q^T fragments (B operand): lane (gq, qq) holds head gq's dims 16s + 2qq (+1) and +8 (+9)
    uint32_t qh[8][2], ql[8][2];
    {
        const float* qb = p.q + (hrow0 + (gq < 2 ? gq : 0)) * D;
#pragma unroll
        for (int s = 0; s < 8; ++s) {
            const int d0 = 16 * s + 2 * qq;
            float v[4] = {0.f, 0.f, 0.f, 0.f};
            if (gq < 2) {
                v[0] = qb[d0] * p.scale_log2;
                v[1] = qb[d0 + 1] * p.scale_log2;
                v[2] = qb[d0 + 8] * p.scale_log2;
                v[3] = qb[d0 + 9] * p.scale_log2;
            }
            split_h2(v[0], v[1], qh[s][0], ql[s][0]);
            split_h2(v[2], v[3], qh[s][1], ql[s][1]);
        }
    }

    uint8_t* wbuf = smem + warp * L::WARP_BYTES;
    uint64_t* wbar = bars + warp * S;
    if (lane == 0) {
        for (int s = 0; s < S; ++s) mbar_init(&wbar[s], 1);
        tma_prefetch_desc(&tmKV);
        fence_mbar_init();
    }
    __syncwarp();

    const int n_mine = b_end - b_start;
    auto issue = [&](int i) {
        const int jb = b_start + i;
        const int s = i % S;
        int blk = jb < p.mbps ? p.block_table[(size_t)slot * p.mbps + jb] : -1;
        if (blk < 0 || blk >= p.num_blocks) {
            record_error(DEV_ERR_ATTN_WAIT);
            blk = 0;  // stay in bounds; the error word reports the bad table entry
        }
        const int krow = (((blk * p.num_layers + p.layer) * 2 + 0) * p.kv_heads + g) * 16;
        const int vrow = krow + p.kv_heads * 16;
        uint8_t* dst = wbuf + s * kTcStage;
        mbar_arrive_expect_tx(&wbar[s], kTcStage);
        tma_load_2d(dst, &tmKV, &wbar[s], 0, krow);
        tma_load_2d(dst + kTcBox, &tmKV, &wbar[s], 64, krow);
        tma_load_2d(dst + 2 * kTcBox, &tmKV, &wbar[s], 0, vrow);
        tma_load_2d(dst + 3 * kTcBox, &tmKV, &wbar[s], 64, vrow);
    };

    int issued = 0;
    if (lane == 0) {
        for (int i = 0; i < n_mine && i < S; ++i) issue(i);
        issued = min(n_mine, S);
    }
    issued = __shfl_sync(0xffffffffu, issued, 0);

    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
    float o[8][4];
#pragma unroll
    for (int mt = 0; mt < 8; ++mt) o[mt][0] = o[mt][1] = o[mt][2] = o[mt][3] = 0.f;

    // ldmatrix row addresses: lane supplies row (lane & 7) of matrix (lane >> 3)
    const int mi = lane >> 3, rr = lane & 7;
    const int k_tok = (mi & 1) * 8 + rr, k_dim = (mi >> 1) * 8;  // K as the A operand (rows = tokens)
    const int v_tok = (mi >> 1) * 8 + rr, v_dim = (mi & 1) * 8;  // V^T as the A operand (transposed load)

    int done = 0;
    bool failed = false;
    for (int i = 0; i < n_mine; ++i) {
        const int s = i % S;
        if (!mbar_wait(&wbar[s], (uint32_t)(i / S) & 1u, DEV_ERR_ATTN_WAIT)) {
            failed = true;
            break;
        }
        const uint32_t kb = smem_u32(wbuf + s * kTcStage);
        const uint32_t vb = kb + 2 * kTcBox;
        const int jb = b_start + i;

        // ---- S^T = K Q^T, four independent accumulator chains (hi / lo x even / odd k-slices)
        float sc4[4][4] = {};
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {
            uint32_t a[4];
            ldsm_x4(tc_sw128(kb, k_tok, 16 * ks + k_dim), a);
            mma_16816(sc4[ks & 1], a, qh[ks][0], qh[ks][1]);
            mma_16816(sc4[2 + (ks & 1)], a, ql[ks][0], ql[ks][1]);
        }
        float sc[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) sc[e] = (sc4[0][e] + sc4[1][e]) + (sc4[2][e] + sc4[3][e]);
        // lanes with qq == 0: sc[0] = (tok gq, head 0), sc[1] = (tok gq, head 1), sc[2], sc[3] = tok gq + 8
        const int tA = jb * 16 + gq, tB = tA + 8;
        const float s00 = tA < ctx ? sc[0] : -INFINITY, s01 = tA < ctx ? sc[1] : -INFINITY;
        const float s10 = tB < ctx ? sc[2] : -INFINITY, s11 = tB < ctx ? sc[3] : -INFINITY;
        float bm0 = fmaxf(s00, s10), bm1 = fmaxf(s01, s11);
#pragma unroll
        for (int off = 4; off <= 16; off <<= 1) {
            bm0 = fmaxf(bm0, __shfl_xor_sync(0xffffffffu, bm0, off));
            bm1 = fmaxf(bm1, __shfl_xor_sync(0xffffffffu, bm1, off));
        }
        // every processed block has at least one visible key, so bm0/bm1 are finite
        const float mn0 = fmaxf(m0, bm0), mn1 = fmaxf(m1, bm1);
        float a0 = m0 == -INFINITY ? 0.f : exp2f(m0 - mn0);
        float a1 = m1 == -INFINITY ? 0.f : exp2f(m1 - mn1);
        const float p00 = s00 == -INFINITY ? 0.f : exp2f(s00 - mn0);
        const float p01 = s01 == -INFINITY ? 0.f : exp2f(s01 - mn1);
        const float p10 = s10 == -INFINITY ? 0.f : exp2f(s10 - mn0);
        const float p11 = s11 == -INFINITY ? 0.f : exp2f(s11 - mn1);
        float ps0 = p00 + p10, ps1 = p01 + p11;
#pragma unroll
        for (int off = 4; off <= 16; off <<= 1) {
            ps0 += __shfl_xor_sync(0xffffffffu, ps0, off);
            ps1 += __shfl_xor_sync(0xffffffffu, ps1, off);
        }
        l0 = l0 * a0 + ps0;
        l1 = l1 * a1 + ps1;
        m0 = mn0;
        m1 = mn1;
        if (qq != 0) a0 = a1 = 0.f;  // these lanes' O^T columns are padding heads (kept at zero)
#pragma unroll
        for (int mt = 0; mt < 8; ++mt) {
            o[mt][0] *= a0;
            o[mt][1] *= a1;
            o[mt][2] *= a0;
            o[mt][3] *= a1;
        }
        // ---- P^T fragments: lane (gq = head, qq) needs P[gq][2qq], [2qq+1], [2qq+8], [2qq+9];
        // P[h][k] sits in lane 4k (k < 8) or 4(k-8) (k >= 8)
        const int src1 = 8 * qq, src2 = 8 * qq + 4;
        const float x0 = __shfl_sync(0xffffffffu, p00, src1), x1 = __shfl_sync(0xffffffffu, p01, src1);
        const float y0 = __shfl_sync(0xffffffffu, p00, src2), y1 = __shfl_sync(0xffffffffu, p01, src2);
        const float z0 = __shfl_sync(0xffffffffu, p10, src1), z1 = __shfl_sync(0xffffffffu, p11, src1);
        const float w0 = __shfl_sync(0xffffffffu, p10, src2), w1 = __shfl_sync(0xffffffffu, p11, src2);
        float pa = 0.f, pb = 0.f, pc = 0.f, pd = 0.f;
        if (gq == 0) {
            pa = x0; pb = y0; pc = z0; pd = w0;
        } else if (gq == 1) {
            pa = x1; pb = y1; pc = z1; pd = w1;
        }
        uint32_t bh0, bl0, bh1, bl1;
        split_h2(pa, pb, bh0, bl0);
        split_h2(pc, pd, bh1, bl1);
        // ---- O^T += V^T P^T
#pragma unroll
        for (int mt = 0; mt < 8; ++mt) {
            uint32_t a[4];
            ldsm_x4_t(tc_sw128(vb, v_tok, 16 * mt + v_dim), a);
            mma_16816(o[mt], a, bh0, bh1);
            mma_16816(o[mt], a, bl0, bl1);
        }
        ++done;
        __syncwarp();
        if (lane == 0 && i + S < n_mine) {
            fence_proxy_async_smem();
            issue(i + S);
            ++issued;
        }
        issued = __shfl_sync(0xffffffffu, issued, 0);
    }
    if (failed && lane == 0) {
        for (int i = done; i < issued; ++i) mbar_wait(&wbar[i % S], (uint32_t)(i / S) & 1u, DEV_ERR_DRAIN);
    }

    // ---- finish: lanes with qq == 0 hold O^T[dims 16mt + gq (+8)][heads 0, 1]
    if (nbt <= p.split_blocks) {  // a single split: final output
        if (qq == 0) {
            const float i0 = l0 > 0.f ? 1.f / l0 : 0.f, i1 = l1 > 0.f ? 1.f / l1 : 0.f;
#pragma unroll
            for (int mt = 0; mt < 8; ++mt) {
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int h = e & 1, d = 16 * mt + gq + (e >> 1) * 8;
                    const float ov = o[mt][e] * (h ? i1 : i0);
                    const __nv_bfloat16 hi = __float2bfloat16(ov);
                    p.out[(hrow0 + h) * D + d] = hi;
                    if (p.out_lo) p.out_lo[(hrow0 + h) * D + d] = __float2bfloat16(ov - __bfloat162float(hi));
                }
            }
        }
        return;
    }
    if (qq == 0) {
#pragma unroll
        for (int mt = 0; mt < 8; ++mt) {
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int h = e & 1, d = 16 * mt + gq + (e >> 1) * 8;
                p.ws_o[((hrow0 + h) * p.max_splits + sp) * D + d] = o[mt][e];
            }
        }
    }
    if (lane == 0) {
        p.ws_ml[((hrow0 + 0) * p.max_splits + sp) * 2 + 0] = m0;
        p.ws_ml[((hrow0 + 0) * p.max_splits + sp) * 2 + 1] = l0;
        p.ws_ml[((hrow0 + 1) * p.max_splits + sp) * 2 + 0] = m1;
        p.ws_ml[((hrow0 + 1) * p.max_splits + sp) * 2 + 1] = l1;
    }
}

// fp16 KV pool as a 2-D tensor [blocks*layers*2*kv_heads*16 rows][128] with 16 x 64 swizzled boxes
inline int make_kv_map(CUtensorMap* map, const AttnParams& p) {
    const uint64_t rows = (uint64_t)p.num_blocks * p.num_layers * 2 * p.kv_heads * 16;
    if (rows >= (1ull << 31)) {
        set_error("paged attention: pool too large for 32-bit tensor-map rows");
        return QTTS_ERR_UNSUPPORTED;
    }
    PFN_encodeTiled enc = get_encode_fn();
    if (!enc) {
        set_error("cuTensorMapEncodeTiled unavailable");
        return QTTS_ERR_CUDA;
    }
    if ((reinterpret_cast<uintptr_t>(p.kv) & 15) != 0) {
        set_error("paged attention: KV pool must be 16-byte aligned");
        return QTTS_ERR_INVALID;
    }
    cuuint64_t dims[2] = {128, rows};
    cuuint64_t strides[1] = {256};
    cuuint32_t box[2] = {64, 16};
    cuuint32_t estr[2] = {1, 1};
    CUresult rc = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<kv_t*>(p.kv), dims, strides, box, estr,
                      CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (rc != CUDA_SUCCESS) {
        set_error("cuTensorMapEncodeTiled (KV pool) failed (%d)", (int)rc);
        return QTTS_ERR_CUDA;
    }
    return QTTS_OK;
}

// ---------------------------------------------------------------------------
// Decode attention without split partials: one CTA per (row, kv head); its W warps take the
// row's KV blocks w, w + W, w + 2W, ... (each with its own TMA ring, the math of
// paged_attn_tc_kernel), and the W partial softmax states (max, sum, unnormalised O) are
// folded in shared memory into the final output.  No workspace and no combine launch.
// ---------------------------------------------------------------------------
template <int S, int W>
struct AttnRowLayout {
    static constexpr int RING = W * S * kTcStage;
    static constexpr int COMB = W * (4 + 2 * 128) * 4;  // per warp: m0 m1 l0 l1, O [2 heads][128]
    static constexpr int SMEM = 1024 + RING + COMB + W * S * 8;
};

template <int S, int W>
__global__ void __launch_bounds__(W * 32) paged_attn_tc_row_kernel(const __grid_constant__ CUtensorMap tmKV,
                                                                   const AttnParams p) {
    constexpr int D = 128;
    using L = AttnRowLayout<S, W>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    float* comb = reinterpret_cast<float*>(smem + L::RING);
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::RING + L::COMB);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int gq = lane >> 2, qq = lane & 3;  // mma fragment coordinates
    const bool early = p.meta_settled != 0;  // metadata and past keys may be read before the wait
    if (!early) {
        griddep_wait();
        griddep_launch();
    }
    const int g = blockIdx.x % p.kv_heads;  // CTA-uniform
    const int r = blockIdx.x / p.kv_heads;
    if (r >= p.R) return;
    const int ctx = __ldcg(p.row_ctx + r);
    const int nbt = (ctx + 15) >> 4;
    const size_t hrow0 = (size_t)r * p.num_heads + g * 2;
    const int slot = __ldcg(p.row_slot + r);
    if (nbt <= 0 || slot < 0) {  // CTA-uniform: a row with no keys (only after a scheduler error)
        if (early) {
            griddep_wait();
            griddep_launch();
        }
        for (int i = threadIdx.x; i < 2 * D; i += W * 32) {
            p.out[hrow0 * D + i] = __float2bfloat16(0.f);
            if (p.out_lo) p.out_lo[hrow0 * D + i] = __float2bfloat16(0.f);
        }
        return;
    }
    const int n_mine = warp < nbt ? (nbt - warp + W - 1) / W : 0;  // blocks warp, warp + W, ...

    uint8_t* wbuf = smem + warp * S * kTcStage;
    uint64_t* wbar = bars + warp * S;
    if (lane == 0) {
        for (int s2 = 0; s2 < S; ++s2) mbar_init(&wbar[s2], 1);
        tma_prefetch_desc(&tmKV);
        fence_mbar_init();
    }
    __syncwarp();

    // the table entry of this warp's block i (lane 0 reads the next one while a block is worked
    // on, so the read's latency stays off the refill)
    auto raw_block = [&](int i) -> int {
        const int jb = warp + W * i;
        return jb < p.mbps ? __ldcg(p.block_table + (size_t)slot * p.mbps + jb) : -1;
    };
    auto issue = [&](int i, int blk) {
        const int s2 = i % S;
        if (blk < 0 || blk >= p.num_blocks) {
            record_error(DEV_ERR_ATTN_WAIT);
            blk = 0;  // stay in bounds; the error word reports the bad table entry
        }
        const int krow = (((blk * p.num_layers + p.layer) * 2 + 0) * p.kv_heads + g) * 16;
        const int vrow = krow + p.kv_heads * 16;
        uint8_t* dst = wbuf + s2 * kTcStage;
        mbar_arrive_expect_tx(&wbar[s2], kTcStage);
        tma_load_2d(dst, &tmKV, &wbar[s2], 0, krow);
        tma_load_2d(dst + kTcBox, &tmKV, &wbar[s2], 64, krow);
        tma_load_2d(dst + 2 * kTcBox, &tmKV, &wbar[s2], 0, vrow);
        tma_load_2d(dst + 3 * kTcBox, &tmKV, &wbar[s2], 64, vrow);
    };

    // the first S loads; with settled metadata they go out before the wait on the preceding
    // kernel (the QKV projection), except the block holding the row's newest key, which that
    // kernel writes
    int issued = 0;
    int next_raw = -1;  // lane 0: table entry of block `issued`
    int deferred = -1;  // lane 0: the first-S block that waits for the preceding kernel
    if (lane == 0) {
        const int newest = (ctx - 1) >> 4;
        for (int i = 0; i < n_mine && i < S; ++i) {
            if (early && warp + W * i == newest) deferred = i;
            else issue(i, raw_block(i));
        }
        issued = min(n_mine, S);
        if (issued < n_mine) next_raw = raw_block(issued);
    }
    issued = __shfl_sync(0xffffffffu, issued, 0);
    if (early) {
        griddep_wait();
        griddep_launch();
        if (lane == 0 && deferred >= 0) issue(deferred, raw_block(deferred));
    }

    // Q^T fragments (B operand): lane (gq, qq) holds head gq's dims 16s + 2qq (+1) and +8 (+9)
    uint32_t qh[8][2], ql[8][2];
    {
        const float* qb = p.q + (hrow0 + (gq < 2 ? gq : 0)) * D;
#pragma unroll
        for (int s2 = 0; s2 < 8; ++s2) {
            const int d0 = 16 * s2 + 2 * qq;
            float v[4] = {0.f, 0.f, 0.f, 0.f};
            if (gq < 2) {
                v[0] = qb[d0] * p.scale_log2;
                v[1] = qb[d0 + 1] * p.scale_log2;
                v[2] = qb[d0 + 8] * p.scale_log2;
                v[3] = qb[d0 + 9] * p.scale_log2;
            }
            split_h2(v[0], v[1], qh[s2][0], ql[s2][0]);
            split_h2(v[2], v[3], qh[s2][1], ql[s2][1]);
        }
    }

    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
    float o[8][4];
#pragma unroll
    for (int mt = 0; mt < 8; ++mt) o[mt][0] = o[mt][1] = o[mt][2] = o[mt][3] = 0.f;

    const int mi = lane >> 3, rr = lane & 7;
    const int k_tok = (mi & 1) * 8 + rr, k_dim = (mi >> 1) * 8;  // K as the A operand (rows = tokens)
    const int v_tok = (mi >> 1) * 8 + rr, v_dim = (mi & 1) * 8;  // V^T as the A operand (transposed load)

    int done = 0;
    bool failed = false;
    for (int i = 0; i < n_mine; ++i) {
        const int s2 = i % S;
        if (!mbar_wait(&wbar[s2], (uint32_t)(i / S) & 1u, DEV_ERR_ATTN_WAIT)) {
            failed = true;
            break;
        }
        const uint32_t kb = smem_u32(wbuf + s2 * kTcStage);
        const uint32_t vb = kb + 2 * kTcBox;
        const int jb = warp + W * i;

        // four independent accumulator chains (hi / lo x even / odd k-slices), summed at the end:
        // the 16 MMAs of a block would otherwise wait on one another
        float sc4[4][4] = {};
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {
            uint32_t a[4];
            ldsm_x4(tc_sw128(kb, k_tok, 16 * ks + k_dim), a);
            mma_16816(sc4[ks & 1], a, qh[ks][0], qh[ks][1]);
            mma_16816(sc4[2 + (ks & 1)], a, ql[ks][0], ql[ks][1]);
        }
        float sc[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) sc[e] = (sc4[0][e] + sc4[1][e]) + (sc4[2][e] + sc4[3][e]);
        const int tA = jb * 16 + gq, tB = tA + 8;
        const float s00 = tA < ctx ? sc[0] : -INFINITY, s01 = tA < ctx ? sc[1] : -INFINITY;
        const float s10 = tB < ctx ? sc[2] : -INFINITY, s11 = tB < ctx ? sc[3] : -INFINITY;
        float bm0 = fmaxf(s00, s10), bm1 = fmaxf(s01, s11);
#pragma unroll
        for (int off = 4; off <= 16; off <<= 1) {
            bm0 = fmaxf(bm0, __shfl_xor_sync(0xffffffffu, bm0, off));
            bm1 = fmaxf(bm1, __shfl_xor_sync(0xffffffffu, bm1, off));
        }
        const float mn0 = fmaxf(m0, bm0), mn1 = fmaxf(m1, bm1);
        float a0 = m0 == -INFINITY ? 0.f : exp2f(m0 - mn0);
        float a1 = m1 == -INFINITY ? 0.f : exp2f(m1 - mn1);
        const float p00 = s00 == -INFINITY ? 0.f : exp2f(s00 - mn0);
        const float p01 = s01 == -INFINITY ? 0.f : exp2f(s01 - mn1);
        const float p10 = s10 == -INFINITY ? 0.f : exp2f(s10 - mn0);
        const float p11 = s11 == -INFINITY ? 0.f : exp2f(s11 - mn1);
        float ps0 = p00 + p10, ps1 = p01 + p11;
#pragma unroll
        for (int off = 4; off <= 16; off <<= 1) {
            ps0 += __shfl_xor_sync(0xffffffffu, ps0, off);
            ps1 += __shfl_xor_sync(0xffffffffu, ps1, off);
        }
        l0 = l0 * a0 + ps0;
        l1 = l1 * a1 + ps1;
        m0 = mn0;
        m1 = mn1;
        if (qq != 0) a0 = a1 = 0.f;  // these lanes' O^T columns are padding heads (kept at zero)
#pragma unroll
        for (int mt = 0; mt < 8; ++mt) {
            o[mt][0] *= a0;
            o[mt][1] *= a1;
            o[mt][2] *= a0;
            o[mt][3] *= a1;
        }
        const int src1 = 8 * qq, src2 = 8 * qq + 4;
        const float x0 = __shfl_sync(0xffffffffu, p00, src1), x1 = __shfl_sync(0xffffffffu, p01, src1);
        const float y0 = __shfl_sync(0xffffffffu, p00, src2), y1 = __shfl_sync(0xffffffffu, p01, src2);
        const float z0 = __shfl_sync(0xffffffffu, p10, src1), z1 = __shfl_sync(0xffffffffu, p11, src1);
        const float w0 = __shfl_sync(0xffffffffu, p10, src2), w1 = __shfl_sync(0xffffffffu, p11, src2);
        float pa = 0.f, pb = 0.f, pc = 0.f, pd = 0.f;
        if (gq == 0) {
            pa = x0; pb = y0; pc = z0; pd = w0;
        } else if (gq == 1) {
            pa = x1; pb = y1; pc = z1; pd = w1;
        }
        uint32_t bh0, bl0, bh1, bl1;
        split_h2(pa, pb, bh0, bl0);
        split_h2(pc, pd, bh1, bl1);
#pragma unroll
        for (int mt = 0; mt < 8; ++mt) {
            uint32_t a[4];
            ldsm_x4_t(tc_sw128(vb, v_tok, 16 * mt + v_dim), a);
            mma_16816(o[mt], a, bh0, bh1);
            mma_16816(o[mt], a, bl0, bl1);
        }
        ++done;
        __syncwarp();
        if (lane == 0 && i + S < n_mine) {
            fence_proxy_async_smem();
            issue(i + S, next_raw);
            ++issued;
            if (issued < n_mine) next_raw = raw_block(issued);
        }
        issued = __shfl_sync(0xffffffffu, issued, 0);
    }
    if (failed && lane == 0) {
        for (int i = done; i < issued; ++i) mbar_wait(&wbar[i % S], (uint32_t)(i / S) & 1u, DEV_ERR_DRAIN);
    }

    // ---- this warp's partial state into shared memory; lanes with qq == 0 hold
    // O^T[dims 16 mt + gq (+8)][heads 0, 1]
    float* cw = comb + warp * (4 + 2 * D);
    if (lane == 0) {
        cw[0] = failed ? -INFINITY : m0;
        cw[1] = failed ? -INFINITY : m1;
        cw[2] = l0;
        cw[3] = l1;
    }
    if (qq == 0) {
#pragma unroll
        for (int mt = 0; mt < 8; ++mt) {
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int h = e & 1, d = 16 * mt + gq + (e >> 1) * 8;
                cw[4 + h * D + d] = o[mt][e];
            }
        }
    }
    __syncthreads();
    // ---- fold the W partial states (fixed order): out = Σ o_w 2^(m_w - M) / Σ l_w 2^(m_w - M)
    for (int t = threadIdx.x; t < 2 * D; t += W * 32) {
        const int h = t / D, d = t - h * D;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < W; ++w) M = fmaxf(M, comb[w * (4 + 2 * D) + h]);
        float num = 0.f, den = 0.f;
        if (M != -INFINITY) {
#pragma unroll
            for (int w = 0; w < W; ++w) {
                const float* cv = comb + w * (4 + 2 * D);
                const float mw = cv[h];
                if (mw == -INFINITY) continue;
                const float sc = exp2f(mw - M);
                num += cv[4 + h * D + d] * sc;
                den += cv[2 + h] * sc;
            }
        }
        const float ov = den > 0.f ? num / den : 0.f;
        const __nv_bfloat16 hi = __float2bfloat16(ov);
        p.out[(hrow0 + h) * D + d] = hi;
        if (p.out_lo) p.out_lo[(hrow0 + h) * D + d] = __float2bfloat16(ov - __bfloat162float(hi));
    }
}

// warps per (row, kv head) CTA of the row form (QTTS_ATTN_ROW_WARPS: 2, 3, 4 or 8).  Three
// with the default 2-stage rings (52 KB of shared memory) keep 4 CTAs on an SM, so the 512 CTAs
// of a 64-row step fit in one wave; four (69 KB) fit only 3 per SM.
inline int attn_row_warps() {
    static const int w = [] {
        const char* v = getenv("QTTS_ATTN_ROW_WARPS");
        const int x = v ? atoi(v) : 3;
        return (x == 2 || x == 4 || x == 8) ? x : 3;
    }();
    return w;
}

template <int S, int W>
inline int launch_attention_tc_rows_w(const AttnParams& p, cudaStream_t st) {
    using L = AttnRowLayout<S, W>;
    CUtensorMap map;
    const int rc = make_kv_map(&map, p);
    if (rc) return rc;
    auto kern = paged_attn_tc_row_kernel<S, W>;
    QTTS_CHECK_CUDA((func_attr_once<paged_attn_tc_row_kernel<S, W>>(L::SMEM)));
    QTTS_LAUNCH(kern, dim3(p.R * p.kv_heads), dim3(W * 32), L::SMEM, st, map, p);
    return QTTS_OK;
}

template <int S>
inline int launch_attention_tc_rows(const AttnParams& p, cudaStream_t st) {
    switch (attn_row_warps()) {
        case 2: return launch_attention_tc_rows_w<S, 2>(p, st);
        case 4: return launch_attention_tc_rows_w<S, 4>(p, st);
        case 8: return launch_attention_tc_rows_w<S, 8>(p, st);
        default: return launch_attention_tc_rows_w<S, 3>(p, st);
    }
}

// head_dim 128 decode attention as one CTA per (row, kv head), no split partials or combine
// launch (QTTS_ATTN_ROWS=0: the split form, paged_attn_tc_kernel + attn_combine_kernel).
// Measured per layer, 64 rows: 14.95 vs 17.0 us at mean context 247 (the benchmark's start),
// 23.0 vs 26.5 us at 346 without prefix sharing, equal (18.85 vs 18.82 us) at the benchmark's
// context 346 with its shared prefix, where the longest rows' warps set the time.
inline bool attn_rows() {
    static const bool on = [] {
        const char* v = getenv("QTTS_ATTN_ROWS");
        return !(v && *v == '0');
    }();
    return on;
}

// Fold split partials: out = Σ_s o_s 2^(m_s - M) / Σ_s l_s 2^(m_s - M), bf16.
template <int D>
__global__ void attn_combine_kernel(const AttnParams p) {
    const int r = blockIdx.x, h = blockIdx.y, d = threadIdx.x;
    griddep_wait();
    griddep_launch();
    const int ctx = p.row_ctx[r];
    const int nbt = (ctx + 15) >> 4;
    const int ns = min(p.max_splits, (nbt + p.split_blocks - 1) / p.split_blocks);
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

// KV blocks per split in the engine's decode step (QTTS_ATTN_SPLIT to override)
// The decode engine's split size: 8 blocks measured best on the 64-stream decode step
// (contexts U[16, 512] + a 96-token prefix: 8581 frames/s vs 8301 with 16); QTTS_ATTN_SPLIT overrides.
constexpr int kEngineAttnSplit = 8;
inline int attn_engine_split() {
    static const int s = [] {
        const char* v = getenv("QTTS_ATTN_SPLIT");
        const int x = (v && *v) ? atoi(v) : kEngineAttnSplit;
        return (x >= 1 && x <= 64) ? x : kEngineAttnSplit;
    }();
    return s;
}

// ---------------------------------------------------------------------------
// Short rows (at most one 16-token block of keys, e.g. the code predictor's
// per-frame cache): one warp per query head, keys read straight from the pool
// (lane l scores key l), softmax with warp reductions, P·V with one broadcast
// per key.  No staging ring: the whole row is 2-4 KB per head.
// ---------------------------------------------------------------------------
template <int D>
__global__ void __launch_bounds__(128) short_attn_kernel(const AttnParams p) {
    static_assert(D % 32 == 0 && D <= 128, "head_dim 32, 64 or 128");
    constexpr int PER = D / 32;
    __shared__ float qs[4][D];
    const int r = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int h = blockIdx.y * 4 + warp;
    const bool head_ok = h < p.num_heads;
    // row metadata (static for the code predictor's stages: read before the wait)
    int n = 0, blk = 0;
    if (p.static_meta && head_ok) {
        n = min(p.row_ctx[r], 16);
        blk = p.block_table[(size_t)p.row_slot[r] * p.mbps];
    }
    griddep_wait();
    griddep_launch();
    if (!head_ok) return;
    if (!p.static_meta) {
        n = min(p.row_ctx[r], 16);
        blk = p.block_table[(size_t)p.row_slot[r] * p.mbps];
    }
    const int g = h / (p.num_heads / p.kv_heads);
    const size_t orow = ((size_t)r * p.num_heads + h) * D;
    if (n <= 0) {
        for (int d = lane; d < D; d += 32) {
            p.out[orow + d] = __float2bfloat16(0.f);
            if (p.out_lo) p.out_lo[orow + d] = __float2bfloat16(0.f);
        }
        return;
    }
    if (blk < 0 || blk >= p.num_blocks) {
        record_error(DEV_ERR_ATTN_WAIT);
        blk = 0;
    }
    const size_t head = (size_t)16 * D;
    const kv_t* K = p.kv + ((((size_t)blk * p.num_layers + p.layer) * 2 + 0) * p.kv_heads + g) * head;
    const kv_t* V = K + (size_t)p.kv_heads * head;
    // every load of the kernel in flight together: this lane's key row, q, and the V
    // elements this lane accumulates for all 16 keys
    uint4 kraw[D / 8];
    if (lane < n) {
#pragma unroll
        for (int j = 0; j < D / 8; ++j) kraw[j] = *reinterpret_cast<const uint4*>(K + (size_t)lane * D + j * 8);
    }
    float vv[16][PER];
#pragma unroll
    for (int k = 0; k < 16; ++k) {
#pragma unroll
        for (int e = 0; e < PER; ++e) vv[k][e] = k < n ? __half2float(V[(size_t)k * D + lane * PER + e]) : 0.f;
    }
    for (int d = lane; d < D; d += 32) qs[warp][d] = p.q[orow + d] * p.scale_log2;
    __syncwarp();
    float sc = -INFINITY;
    if (lane < n) {
        float acc[4] = {0.f, 0.f, 0.f, 0.f};  // independent chains
#pragma unroll
        for (int j = 0; j < D / 8; ++j) {
            const __half2* hp = reinterpret_cast<const __half2*>(&kraw[j]);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const float2 f = __half22float2(hp[e]);
                acc[e] += f.x * qs[warp][j * 8 + 2 * e] + f.y * qs[warp][j * 8 + 2 * e + 1];
            }
        }
        sc = (acc[0] + acc[1]) + (acc[2] + acc[3]);
    }
    const float mx = warp_max(sc);
    const float pr = lane < n ? exp2f(sc - mx) : 0.f;
    const float inv = 1.0f / warp_sum(pr);
    float o[PER];
#pragma unroll
    for (int e = 0; e < PER; ++e) o[e] = 0.f;
#pragma unroll
    for (int k = 0; k < 16; ++k) {
        const float pk = __shfl_sync(0xffffffffu, pr, k);  // 0 beyond n
#pragma unroll
        for (int e = 0; e < PER; ++e) o[e] += pk * vv[k][e];
    }
#pragma unroll
    for (int e = 0; e < PER; ++e) {
        const float v = o[e] * inv;
        const __nv_bfloat16 hi = __float2bfloat16(v);
        p.out[orow + lane * PER + e] = hi;
        if (p.out_lo) p.out_lo[orow + lane * PER + e] = __float2bfloat16(v - __bfloat162float(hi));
    }
}

// rows whose keys fit one 16-token block (p.mbps == 1)
inline int launch_short_attention(const AttnParams& p, int head_dim, cudaStream_t st) {
    if (p.R <= 0) return QTTS_OK;
    const dim3 grid(p.R, ceil_div(p.num_heads, 4));
    switch (head_dim) {
        case 128: QTTS_LAUNCH(short_attn_kernel<128>, grid, dim3(128), 0, st, p); return QTTS_OK;
        case 64: QTTS_LAUNCH(short_attn_kernel<64>, grid, dim3(128), 0, st, p); return QTTS_OK;
        case 32: QTTS_LAUNCH(short_attn_kernel<32>, grid, dim3(128), 0, st, p); return QTTS_OK;
        default:
            set_error("short attention: head_dim %d not supported (32, 64 or 128)", head_dim);
            return QTTS_ERR_UNSUPPORTED;
    }
}

inline int attn_max_splits(int max_ctx, int split_blocks = QTTS_ATTN_SPLIT_BLOCKS) {
    const int nb = (max_ctx + 15) / 16;
    const int s = (nb + split_blocks - 1) / split_blocks;
    return s > 1 ? s : 1;
}

template <int D, int S>
inline int launch_attention_s(const AttnParams& p, cudaStream_t st) {
    using L = AttnLayout<D, S>;
    auto kern = paged_attn_kernel<D, S>;
    QTTS_CHECK_CUDA((func_attr_once<paged_attn_kernel<D, S>>(L::SMEM)));
    QTTS_LAUNCH(kern, dim3(p.R, p.kv_heads, p.max_splits), dim3(128), L::SMEM, st, p);
    return QTTS_OK;
}

template <int S>
inline int launch_attention_tc(const AttnParams& p, cudaStream_t st) {
    using L = AttnTcLayout<S>;
    CUtensorMap map;
    const int rc = make_kv_map(&map, p);
    if (rc) return rc;
    auto kern = paged_attn_tc_kernel<S>;
    QTTS_CHECK_CUDA((func_attr_once<paged_attn_tc_kernel<S>>(L::SMEM)));
    const int items = p.R * p.kv_heads * p.max_splits;  // one (split, row, kv head) per warp
    QTTS_LAUNCH(kern, dim3(ceil_div(items, 4)), dim3(128), L::SMEM, st, map, p);
    return QTTS_OK;
}

// ---------------------------------------------------------------------------
// Chunked prefill, head_dim 128: the rows of a prefill step are streams of
// rows_per_stream consecutive query tokens, each row seeing its first row_ctx
// keys (the causal mask of talker_unified_modules.py:282-288 over the chunk,
// after the stream's earlier KV).  One warp per work item (8-token query tile of
// one stream, kv head, split of split_blocks KV blocks): each KV block is staged
// once (TMA, 128-B swizzle, the decode kernel's ring) and serves the tile's 8
// queries x 2 heads, instead of being read again for every query row.
//
// Per 16-token block, on the tensor pipe (mma.sync m16n8k16, fp16 in, fp32 acc):
//   S[16][16] = Q[16 rows][128] · K^T[128][16 keys]   rows = (query i, head h):
//       row i for head 0, row 8 + i for head 1; Q carried as an fp16 hi/lo pair
//   masked per (query, key), online softmax per row in the log2 domain
//   O[16][128] += P[16][16] · V[16][128]               P as an fp16 hi/lo pair,
//       taken straight from S's accumulator layout (no shuffles)
// Output per row as the decode kernel: final when the row has one split of keys,
// otherwise (o, max, sum) partials that attn_combine_kernel folds.
// ---------------------------------------------------------------------------
constexpr int kPrefillTile = 8;  // query tokens per warp work item

template <int S>
__global__ void __launch_bounds__(128) paged_prefill_tc_kernel(const __grid_constant__ CUtensorMap tmKV,
                                                               const AttnParams p) {
    constexpr int D = 128;
    using L = AttnTcLayout<S>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + 4 * L::WARP_BYTES);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int gq = lane >> 2, qq = lane & 3;  // mma fragment coordinates
    griddep_wait();
    griddep_launch();
    const int SPS = p.rows_per_stream;
    const int n_streams = p.R / SPS;
    const int n_tiles = (SPS + kPrefillTile - 1) / kPrefillTile;
    const int item = blockIdx.x * 4 + warp;
    if (item >= n_streams * n_tiles * p.kv_heads * p.max_splits) return;  // warp-uniform
    int rest = item;
    const int g = rest % p.kv_heads;
    rest /= p.kv_heads;
    const int tile = rest % n_tiles;
    rest /= n_tiles;
    const int b = rest % n_streams;
    const int sp = rest / n_streams;
    const int r0 = b * SPS + tile * kPrefillTile;
    const int nq = min(kPrefillTile, SPS - tile * kPrefillTile);
    // this lane's query (row gq of the tile) and its key count; the tile reads up to the largest
    const bool q_ok = gq < nq;
    const int ctx_q = q_ok ? p.row_ctx[r0 + gq] : 0;
    int ctx_max = ctx_q;
#pragma unroll
    for (int off = 4; off <= 16; off <<= 1) ctx_max = max(ctx_max, __shfl_xor_sync(0xffffffffu, ctx_max, off));
    const int nbt = (ctx_max + 15) >> 4;
    const int b_start = sp * p.split_blocks;
    const int b_end = min(nbt, b_start + p.split_blocks);
    const int nbt_q = (ctx_q + 15) >> 4;
    const int ns_q = min(p.max_splits, (nbt_q + p.split_blocks - 1) / p.split_blocks);  // splits of this query
    const size_t hrow0 = (size_t)(r0 + gq) * p.num_heads + g * 2;  // head 0 of this lane's query
    if (b_start >= b_end) {
        if (sp == 0 && q_ok && ctx_q <= 0 && qq == 0) {  // no keys (only after a scheduler error): zeros
            for (int i = 0; i < 2 * D; ++i) {
                p.out[hrow0 * D + i] = __float2bfloat16(0.f);
                if (p.out_lo) p.out_lo[hrow0 * D + i] = __float2bfloat16(0.f);
            }
        }
        return;
    }
    const int slot = p.row_slot[r0];
    // self-check: the rows' buffers hold R rows; a slot outside the table is skipped
    const size_t qo_limit = (size_t)p.R * p.num_heads * D;
    const size_t ws_limit = (size_t)p.R * p.num_heads * p.max_splits;
    if (slot < 0 || r0 + nq > p.R) {
        if (lane == 0) record_error(DEV_ERR_ATTN_BOUNDS);
        return;
    }

    // Q fragments (A operand): lane (gq, qq) holds rows gq (head 0) and gq + 8 (head 1) of
    // query gq, dims 16 ks + 2 qq (+1) and + 8 (+9), scaled into the log2 domain
    uint32_t qh[8][4], ql[8][4];
    {
        const float* q0p = p.q + hrow0 * D;
        const float* q1p = q0p + D;
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {
            const int d0 = 16 * ks + 2 * qq;
            float v[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
            if (q_ok) {
                v[0] = q0p[d0] * p.scale_log2;
                v[1] = q0p[d0 + 1] * p.scale_log2;
                v[2] = q1p[d0] * p.scale_log2;
                v[3] = q1p[d0 + 1] * p.scale_log2;
                v[4] = q0p[d0 + 8] * p.scale_log2;
                v[5] = q0p[d0 + 9] * p.scale_log2;
                v[6] = q1p[d0 + 8] * p.scale_log2;
                v[7] = q1p[d0 + 9] * p.scale_log2;
            }
#pragma unroll
            for (int j = 0; j < 4; ++j) split_h2(v[2 * j], v[2 * j + 1], qh[ks][j], ql[ks][j]);
        }
    }

    uint8_t* wbuf = smem + warp * L::WARP_BYTES;
    uint64_t* wbar = bars + warp * S;
    if (lane == 0) {
        for (int s = 0; s < S; ++s) mbar_init(&wbar[s], 1);
        tma_prefetch_desc(&tmKV);
        fence_mbar_init();
    }
    __syncwarp();

    const int n_mine = b_end - b_start;
    auto issue = [&](int i) {
        const int jb = b_start + i;
        const int s = i % S;
        int blk = jb < p.mbps ? p.block_table[(size_t)slot * p.mbps + jb] : -1;
        if (blk < 0 || blk >= p.num_blocks) {
            record_error(DEV_ERR_ATTN_WAIT);
            blk = 0;  // stay in bounds; the error word reports the bad table entry
        }
        const int krow = (((blk * p.num_layers + p.layer) * 2 + 0) * p.kv_heads + g) * 16;
        const int vrow = krow + p.kv_heads * 16;
        uint8_t* dst = wbuf + s * kTcStage;
        mbar_arrive_expect_tx(&wbar[s], kTcStage);
        tma_load_2d(dst, &tmKV, &wbar[s], 0, krow);
        tma_load_2d(dst + kTcBox, &tmKV, &wbar[s], 64, krow);
        tma_load_2d(dst + 2 * kTcBox, &tmKV, &wbar[s], 0, vrow);
        tma_load_2d(dst + 3 * kTcBox, &tmKV, &wbar[s], 64, vrow);
    };

    int issued = 0;
    if (lane == 0) {
        for (int i = 0; i < n_mine && i < S; ++i) issue(i);
        issued = min(n_mine, S);
    }
    issued = __shfl_sync(0xffffffffu, issued, 0);

    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;  // rows (query gq, head 0 / 1)
    float o[16][4];
#pragma unroll
    for (int dt = 0; dt < 16; ++dt) o[dt][0] = o[dt][1] = o[dt][2] = o[dt][3] = 0.f;

    // ldmatrix row addresses: lane supplies row (lane & 7) of matrix (lane >> 3)
    const int mi = lane >> 3, rr = lane & 7;
    const int kb_key = (mi >> 1) * 8 + rr, kb_dim = (mi & 1) * 8;  // K^T as the B operand (rows = keys)
    const int vb_key = (mi & 1) * 8 + rr, vb_dim = (mi >> 1) * 8;  // V as the B operand (transposed load)

    int done = 0;
    bool failed = false;
    for (int i = 0; i < n_mine; ++i) {
        const int s = i % S;
        if (!mbar_wait(&wbar[s], (uint32_t)(i / S) & 1u, DEV_ERR_ATTN_WAIT)) {
            failed = true;
            break;
        }
        const uint32_t kb = smem_u32(wbuf + s * kTcStage);
        const uint32_t vb = kb + 2 * kTcBox;
        const int jb = b_start + i;

        // ---- S = Q K^T: two 8-key n-tiles, hi and lo in separate accumulator chains
        float sc[2][4] = {}, sl[2][4] = {};
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {
            uint32_t kf[4];
            ldsm_x4(tc_sw128(kb, kb_key, 16 * ks + kb_dim), kf);
            mma_16816(sc[0], qh[ks], kf[0], kf[1]);
            mma_16816(sl[0], ql[ks], kf[0], kf[1]);
            mma_16816(sc[1], qh[ks], kf[2], kf[3]);
            mma_16816(sl[1], ql[ks], kf[2], kf[3]);
        }
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
#pragma unroll
            for (int e = 0; e < 4; ++e) sc[nt][e] += sl[nt][e];
        // sc[nt][0,1] = (head 0, keys 16 jb + 8 nt + 2 qq, +1), sc[nt][2,3] = head 1, same keys
        float bm0 = -INFINITY, bm1 = -INFINITY;
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) {
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int key = jb * 16 + nt * 8 + 2 * qq + (e & 1);
                if (key >= ctx_q) sc[nt][e] = -INFINITY;
            }
            bm0 = fmaxf(bm0, fmaxf(sc[nt][0], sc[nt][1]));
            bm1 = fmaxf(bm1, fmaxf(sc[nt][2], sc[nt][3]));
        }
#pragma unroll
        for (int off = 1; off <= 2; off <<= 1) {
            bm0 = fmaxf(bm0, __shfl_xor_sync(0xffffffffu, bm0, off));
            bm1 = fmaxf(bm1, __shfl_xor_sync(0xffffffffu, bm1, off));
        }
        const float mn0 = fmaxf(m0, bm0), mn1 = fmaxf(m1, bm1);
        const float a0 = m0 == -INFINITY ? 0.f : exp2f(m0 - mn0);
        const float a1 = m1 == -INFINITY ? 0.f : exp2f(m1 - mn1);
        float pr[2][4];
        float ps0 = 0.f, ps1 = 0.f;
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) {
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const float mref = e < 2 ? mn0 : mn1;
                pr[nt][e] = sc[nt][e] == -INFINITY ? 0.f : exp2f(sc[nt][e] - mref);
            }
            ps0 += pr[nt][0] + pr[nt][1];
            ps1 += pr[nt][2] + pr[nt][3];
        }
#pragma unroll
        for (int off = 1; off <= 2; off <<= 1) {
            ps0 += __shfl_xor_sync(0xffffffffu, ps0, off);
            ps1 += __shfl_xor_sync(0xffffffffu, ps1, off);
        }
        l0 = l0 * a0 + ps0;
        l1 = l1 * a1 + ps1;
        m0 = mn0;
        m1 = mn1;
#pragma unroll
        for (int dt = 0; dt < 16; ++dt) {
            o[dt][0] *= a0;
            o[dt][1] *= a0;
            o[dt][2] *= a1;
            o[dt][3] *= a1;
        }
        // ---- P as the A operand, straight from the accumulator layout: rows gq / gq + 8,
        // keys 2 qq (+1) in regs 0 / 1 and 8 + 2 qq (+1) in regs 2 / 3
        uint32_t ph[4], pl[4];
        split_h2(pr[0][0], pr[0][1], ph[0], pl[0]);
        split_h2(pr[0][2], pr[0][3], ph[1], pl[1]);
        split_h2(pr[1][0], pr[1][1], ph[2], pl[2]);
        split_h2(pr[1][2], pr[1][3], ph[3], pl[3]);
        // ---- O += P V: 16 dim tiles of 8, two per transposed ldmatrix
#pragma unroll
        for (int dp = 0; dp < 8; ++dp) {
            uint32_t vf[4];
            ldsm_x4_t(tc_sw128(vb, vb_key, 16 * dp + vb_dim), vf);
            mma_16816(o[2 * dp], ph, vf[0], vf[1]);
            mma_16816(o[2 * dp], pl, vf[0], vf[1]);
            mma_16816(o[2 * dp + 1], ph, vf[2], vf[3]);
            mma_16816(o[2 * dp + 1], pl, vf[2], vf[3]);
        }
        ++done;
        __syncwarp();
        if (lane == 0 && i + S < n_mine) {
            fence_proxy_async_smem();
            issue(i + S);
            ++issued;
        }
        issued = __shfl_sync(0xffffffffu, issued, 0);
    }
    if (failed && lane == 0) {
        for (int i = done; i < issued; ++i) mbar_wait(&wbar[i % S], (uint32_t)(i / S) & 1u, DEV_ERR_DRAIN);
    }
    if (!q_ok || sp >= ns_q) return;  // padding query, or a split without keys of this query
    if ((hrow0 + 2) * D > qo_limit || (hrow0 + 2) * p.max_splits > ws_limit) {
        record_error(DEV_ERR_ATTN_BOUNDS);
        return;
    }

    // ---- rows (query gq, heads 0 / 1): dims 8 dt + 2 qq (+1)
    if (ns_q == 1) {  // all of this query's keys were in this split: final output
        const float i0 = l0 > 0.f ? 1.f / l0 : 0.f, i1 = l1 > 0.f ? 1.f / l1 : 0.f;
#pragma unroll
        for (int dt = 0; dt < 16; ++dt) {
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int h = e >> 1, d = 8 * dt + 2 * qq + (e & 1);
                const float ov = o[dt][e] * (h ? i1 : i0);
                const __nv_bfloat16 hi = __float2bfloat16(ov);
                p.out[(hrow0 + h) * D + d] = hi;
                if (p.out_lo) p.out_lo[(hrow0 + h) * D + d] = __float2bfloat16(ov - __bfloat162float(hi));
            }
        }
        return;
    }
#pragma unroll
    for (int dt = 0; dt < 16; ++dt) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int h = e >> 1, d = 8 * dt + 2 * qq + (e & 1);
            p.ws_o[((hrow0 + h) * p.max_splits + sp) * D + d] = o[dt][e];
        }
    }
    if (qq == 0) {
        p.ws_ml[((hrow0 + 0) * p.max_splits + sp) * 2 + 0] = m0;
        p.ws_ml[((hrow0 + 0) * p.max_splits + sp) * 2 + 1] = l0;
        p.ws_ml[((hrow0 + 1) * p.max_splits + sp) * 2 + 0] = m1;
        p.ws_ml[((hrow0 + 1) * p.max_splits + sp) * 2 + 1] = l1;
    }
}

template <int S>
inline int launch_prefill_tc(const AttnParams& p, cudaStream_t st) {
    using L = AttnTcLayout<S>;
    CUtensorMap map;
    const int rc = make_kv_map(&map, p);
    if (rc) return rc;
    auto kern = paged_prefill_tc_kernel<S>;
    QTTS_CHECK_CUDA((func_attr_once<paged_prefill_tc_kernel<S>>(L::SMEM)));
    const int n_tiles = (p.rows_per_stream + kPrefillTile - 1) / kPrefillTile;
    const int items = (p.R / p.rows_per_stream) * n_tiles * p.kv_heads * p.max_splits;
    QTTS_LAUNCH(kern, dim3(ceil_div(items, 4)), dim3(128), L::SMEM, st, map, p);
    return QTTS_OK;
}

// ---------------------------------------------------------------------------
// Chunked prefill on the tcgen05 tensor pipe (head_dim 128, two query heads per KV head).
// One CTA per (stream, kv head, group of 64 query rows): the group's 64 queries x 2 heads are
// the 128 rows of the UMMA M side (row = head * 64 + query), keys arrive in tiles of 64 (four
// 16-token blocks, TMA with the 128-B swizzle, a 4-stage ring), and per tile i
//   S[128][64]  = Q · K^T     TMEM, two buffers (columns 0..63 / 192..255); a UMMA warp
//                             issues S(i + 1) while the softmax warps work on tile i (a TMA
//                             warp keeps the ring two tiles ahead)
//   softmax     8 warps, two threads per row (TMEM lane): each takes 32 keys and 64 columns of
//               O; causal mask (keys < row_ctx), online max in the log2 domain shared by the
//               pair through shared memory; O is rescaled in TMEM only when the max grows by
//               more than 8 (P = 2^(s - m) stays below 256, exact enough as an fp16 pair)
//   P -> shared memory as an fp16 hi/lo pair (K-major, swizzled)
//   O[128][128] += P · V      TMEM columns 64..191; two passes, hi and lo; V is read where TMA
//                             put it, as an MN-major operand (keys are its K rows, dims its N);
//                             in the last tile, V rows past the group's keys are zeroed first
// then O / l per row, written as a bf16 hi/lo pair.  Q is an fp16 hi/lo pair too, so both
// products keep about 22 bits.  No key splits: the group's keys run in one CTA (prefill chunks
// are at most max_prefill_rows long).  Every wait is bounded.
// ---------------------------------------------------------------------------
constexpr int kPfuQ = 64;        // queries per CTA
constexpr int kPfuKeys = 64;     // keys per tile
constexpr int kPfuStages = 4;
constexpr int kPfuSoftmaxWarps = 8;                        // two per TMEM lane quadrant
constexpr int kPfuThreads = (kPfuSoftmaxWarps + 2) * 32;   // + the UMMA warp and the TMA warp

struct PfuLayout {
    static constexpr int QH = 0;                      // Q hi: 2 halves [128 rows][64 dims] fp16
    static constexpr int QL = QH + 2 * 128 * 128;     // Q lo
    static constexpr int RING = QL + 2 * 128 * 128;   // stages: K half 0/1, V half 0/1 [64 keys][64 dims]
    static constexpr int STAGE = 4 * 64 * 128;
    static constexpr int PH = RING + kPfuStages * STAGE;  // P hi [128 rows][64 keys]
    static constexpr int PL = PH + 128 * 128;         // P lo
    static constexpr int BAR = PL + 128 * 128;        // kv_full[4], s_full[2], pv_done, drain, tmem slot
    static constexpr int XCH = BAR + 128;             // [2][128] floats: a row's pair exchange
    static constexpr int SMEM = 1024 + XCH + 2 * 128 * 4;
};
static_assert(PfuLayout::SMEM <= 227 * 1024, "prefill tile exceeds shared memory");

// byte offset of (row, col) (col < 64 fp16) in a K-major tile of 128-B rows with the 128-B swizzle
__device__ __forceinline__ uint32_t sw128_off(int row, int col) {
    return (uint32_t)(row * 128 + ((((col >> 3) ^ (row & 7)) << 4)) + (col & 7) * 2);
}

__device__ __forceinline__ void stsm_x4(uint32_t addr, const uint32_t (&r)[4]) {
    asm volatile("stmatrix.sync.aligned.m8n8.x4.shared.b16 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(r[0]),
                 "r"(r[1]), "r"(r[2]), "r"(r[3])
                 : "memory");
}

// 32 lanes x 32 bits, 32 consecutive columns (one wait)
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// Shared-memory descriptor of an MN-major operand with the 128-B swizzle: 128-B rows (64
// fp16 along MN) are the K rows, 8-row groups 1024 B apart (SBO), and the next 64 MN elements
// start `mn_block_bytes` further on (LBO).
__device__ __forceinline__ uint64_t make_sw128_mn_desc(uint32_t smem_addr, uint32_t mn_block_bytes) {
    uint64_t d = 0;
    d |= (uint64_t)((smem_addr >> 4) & 0x3FFF);
    d |= (uint64_t)((mn_block_bytes >> 4) & 0x3FFF) << 16;  // LBO: next 64 MN elements
    d |= (uint64_t)(1024 >> 4) << 32;                       // SBO: next 8 K rows
    d |= (uint64_t)1 << 46;                                 // descriptor version (Blackwell)
    d |= (uint64_t)2 << 61;                                 // SWIZZLE_128B
    return d;
}

__device__ __forceinline__ float ex2_approx(float x) {  // 2^x; 0 for -inf
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// optional per-window timestamps of the tcgen05 prefill (a profiling build defines PFU_STAMP;
// role 0 = the UMMA warp, 1 / 2 = a softmax thread of each half)
#ifndef PFU_STAMP
#define PFU_STAMP(role, point)
#endif

// the two warps that share a TMEM lane quadrant (w and w + 4) meet at barrier 1 + w % 4
__device__ __forceinline__ void pair_sync(int warp) {
    asm volatile("bar.sync %0, 64;" ::"r"(1 + (warp & 3)) : "memory");
}

__global__ void __launch_bounds__(kPfuThreads, 1) paged_prefill_umma_kernel(const __grid_constant__ CUtensorMap tmKV,
                                                                             const AttnParams p) {
    constexpr int D = 128;
    using L = PfuLayout;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* kv_full = reinterpret_cast<uint64_t*>(smem + L::BAR);
    uint64_t* s_full = kv_full + kPfuStages;  // [2]: S buffer b holds its tile's scores
    uint64_t* pv_done = s_full + 2;
    uint64_t* drain = pv_done + 1;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
    float* xch = reinterpret_cast<float*>(smem + L::XCH);

    const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
    const bool mma_w = warp == kPfuSoftmaxWarps;      // issues the UMMAs (and owns TMEM)
    const bool tma_w = warp == kPfuSoftmaxWarps + 1;  // issues the KV loads
    const bool ctrl = mma_w || tma_w;
    griddep_wait();
    griddep_launch();
    const int SPS = p.rows_per_stream;
    const int n_streams = p.R / SPS;
    const int n_groups = (SPS + kPfuQ - 1) / kPfuQ;
    int rest = blockIdx.x;  // CTA-uniform
    const int g = rest % p.kv_heads;
    rest /= p.kv_heads;
    const int grp = rest % n_groups;
    rest /= n_groups;
    const int b = rest % n_streams;
    const int sp = rest / n_streams;  // key split sp of max_splits: a contiguous share of the group's tiles
    if (sp >= p.max_splits) return;
    const int nsplit = p.max_splits;
    const int q0 = grp * kPfuQ;                        // first query of the group within the stream
    const int nq = min(kPfuQ, SPS - q0);
    const int row = t & 127, ch = (t >> 7) & 1;        // softmax threads: TMEM lane and half
    const int h = row >> 6, qi = row & 63;
    const bool row_ok = !ctrl && qi < nq;
    const int r = b * SPS + q0 + qi;                   // row of the call
    const int ctx_row = row_ok ? p.row_ctx[r] : 0;
    const int slot = p.row_slot[b * SPS];
    // the group's keys: the largest key count of its rows (CTA-uniform through shared memory)
    __shared__ int s_ctx;
    if (t == 0) s_ctx = 0;
    __syncthreads();
    if (row_ok && ch == 0) atomicMax(&s_ctx, ctx_row);
    __syncthreads();
    const int ctx_max = s_ctx;
    const size_t out_row = (size_t)r * p.num_heads + g * 2 + h;
    const size_t part_row = (size_t)out_row * nsplit + sp;  // this row's partial (several splits)
    if (ctx_max <= 0 || slot < 0) {  // CTA-uniform: nothing to attend (only after a scheduler error)
        if (ctx_max > 0 && t == 0 && sp == 0) record_error(DEV_ERR_ATTN_BOUNDS);
        if (row_ok && nsplit == 1)
            for (int d = ch * 64; d < ch * 64 + 64; ++d) {
                p.out[out_row * D + d] = __float2bfloat16(0.f);
                if (p.out_lo) p.out_lo[out_row * D + d] = __float2bfloat16(0.f);
            }
        if (row_ok && nsplit > 1 && ch == 0) {  // an empty partial: prefill_combine_kernel writes zeros
            p.ws_ml[part_row * 2 + 0] = -INFINITY;
            p.ws_ml[part_row * 2 + 1] = 0.f;
        }
        return;
    }
    const int nbt = (ctx_max + 15) >> 4;               // 16-token blocks the group reads
    const int ntiles = (ctx_max + kPfuKeys - 1) / kPfuKeys;
    const int t0 = (int)(((long long)sp * ntiles) / nsplit);
    const int nt = (int)(((long long)(sp + 1) * ntiles) / nsplit) - t0;  // this CTA's tiles: t0 .. t0 + nt - 1
    if (nt <= 0) {  // CTA-uniform: fewer tiles than splits; this split is empty for every row
        if (row_ok && ch == 0) {
            p.ws_ml[part_row * 2 + 0] = -INFINITY;
            p.ws_ml[part_row * 2 + 1] = 0.f;
        }
        return;
    }

    // Block j of tile `tile` as the table holds it (lanes 0..3 of the TMA warp each fetch
    // one, a window before the block is loaded, so the read's latency is hidden); past the
    // group's keys any valid block stands in (its keys are masked and its V zeroed).
    auto tile_block_raw = [&](int tile, int j) -> int {
        int jb = tile * 4 + j;
        if (jb >= nbt) jb = 0;
        return jb < p.mbps ? p.block_table[(size_t)slot * p.mbps + jb] : -1;
    };
    auto checked = [&](int blk) -> int {
        if (blk < 0 || blk >= p.num_blocks) {
            record_error(DEV_ERR_ATTN_BOUNDS);
            blk = 0;  // stay in bounds; the error word reports the bad table entry
        }
        return blk;
    };
    // TMA warp, converged: local tile li's K and V, both dim halves, one box per lane 0..15
    // (lane = 4 j + 2 kind + half); lanes 0..3 hold the four block ids.
    auto issue = [&](int li, int nb, bool go) {
        const int s2 = li % kPfuStages;
        uint8_t* st = smem + L::RING + s2 * L::STAGE;
        const int blk = __shfl_sync(0xffffffffu, nb, (lane >> 2) & 3);
        if (!go) return;
        if (lane == 0) mbar_arrive_expect_tx(&kv_full[s2], L::STAGE);
        __syncwarp();
        if (lane < 16) {
            const int j = lane >> 2, kind = (lane >> 1) & 1, half = lane & 1;
            const int row = (((blk * p.num_layers + p.layer) * 2 + kind) * p.kv_heads + g) * 16;
            tma_load_2d(st + (kind * 2 + half) * 8192 + j * 2048, &tmKV, &kv_full[s2], half * 64, row);
        }
    };

    int issued = 0;   // TMA lane 0: tiles whose loads were issued
    int nb_next = 0;  // TMA lanes 0..3: block ids (as read) of the next tile to load
    if (t == 0) {
        for (int s2 = 0; s2 < kPfuStages; ++s2) mbar_init(&kv_full[s2], 1);
        mbar_init(&s_full[0], 1);
        mbar_init(&s_full[1], 1);
        mbar_init(pv_done, 1);
        mbar_init(drain, 1);
        fence_mbar_init();
    }
    __syncthreads();
    if (mma_w) {
        tmem_alloc(tmem_slot, 256);
        tmem_relinquish();
    } else if (tma_w) {
        if (lane == 0) tma_prefetch_desc(&tmKV);
        // the first two tiles' loads; the third's block ids stay in lanes 0..3
        for (int li = 0; li < 2 && li < nt; ++li)
            issue(li, lane < 4 ? checked(tile_block_raw(t0 + li, lane)) : 0, true);
        issued = min(nt, 2);
        nb_next = (lane < 4 && 2 < nt) ? tile_block_raw(t0 + 2, lane) : 0;
    } else {
        // ---- Q rows (x scale_log2) as an fp16 hi/lo pair: this thread's half of the dims
        const float4* qp = reinterpret_cast<const float4*>(p.q + out_row * D + ch * 64);
        const float sc = p.scale_log2;
#pragma unroll 2
        for (int c = 0; c < 8; ++c) {  // 16-B chunk c of the half: dims 64 ch + 8c .. + 7
            float4 x0 = make_float4(0.f, 0.f, 0.f, 0.f), x1 = x0;
            if (row_ok) {
                x0 = qp[2 * c];
                x1 = qp[2 * c + 1];
            }
            uint32_t hi[4], lo[4];
            split_h2(x0.x * sc, x0.y * sc, hi[0], lo[0]);
            split_h2(x0.z * sc, x0.w * sc, hi[1], lo[1]);
            split_h2(x1.x * sc, x1.y * sc, hi[2], lo[2]);
            split_h2(x1.z * sc, x1.w * sc, hi[3], lo[3]);
            const uint32_t off = (uint32_t)ch * (128 * 128) + sw128_off(row, c * 8);
            *reinterpret_cast<uint4*>(smem + L::QH + off) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
            *reinterpret_cast<uint4*>(smem + L::QL + off) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
        }
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
    // O's B operand (V) is MN-major: bit 16 of the instruction descriptor
    const uint32_t idesc_s = make_idesc_f16(128, kPfuKeys), idesc_o = make_idesc_f16(128, D) | (1u << 16);

    // UMMA lane 0: S of local tile li = Q K^T into buffer li & 1, once the tile's K has landed
    auto issue_s = [&](int li) -> bool {
        if (!mbar_wait(&kv_full[li % kPfuStages], (uint32_t)(li / kPfuStages) & 1u, DEV_ERR_ATTN_WAIT))
            return false;
        tc_fence_after();
        const uint32_t st = smem_u32(smem + L::RING + (li % kPfuStages) * L::STAGE);
        const uint32_t d = tmem + ((li & 1) ? 192u : 0u);
#pragma unroll
        for (int part = 0; part < 2; ++part) {
            const uint32_t qb = smem_u32(smem + (part ? L::QL : L::QH));
#pragma unroll
            for (int hd = 0; hd < 2; ++hd)
#pragma unroll
                for (int kk = 0; kk < 4; ++kk)
                    umma_bf16(d, make_sw128_desc(qb + hd * 16384) + 2 * kk, make_sw128_desc(st + hd * 8192) + 2 * kk,
                              idesc_s, (part | hd | kk) ? 1u : 0u);
        }
        umma_commit(&s_full[li & 1]);
        return true;
    };
    // UMMA lane 0: O (+)= P V of the tile whose P is in shared memory (V in its stage; a
    // K step of 16 keys is two 8-row groups, 2048 B)
    auto issue_pv = [&](int li) {
        const uint32_t vb = smem_u32(smem + L::RING + (li % kPfuStages) * L::STAGE) + 2 * 8192;
#pragma unroll
        for (int part = 0; part < 2; ++part) {
            const uint32_t pb = smem_u32(smem + (part ? L::PL : L::PH));
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
                umma_bf16(tmem + 64u, make_sw128_desc(pb) + 2 * kk, make_sw128_mn_desc(vb + kk * 2048, 8192), idesc_o,
                          (li > 0 || part > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(pv_done);
    };

    bool fail = false;  // this thread saw a wait run out; the CTA leaves the loop together
    if (mma_w && lane == 0) fail = !issue_s(0);
    float m_ref = -INFINITY, l = 0.f;
    int li = 0;
    // Window li (between two CTA barriers; local tile li = tile t0 + li): the softmax warps turn
    // S(li) into P(li); the UMMA warp issues PV(li - 1) and S(li + 1) (into the S buffer li - 1
    // left) back to back; the TMA warp issues the loads of li + 2 (into the stage of li - 2, whose
    // PV the softmax warps saw finish in window li - 1) and reads the block ids of li + 3.
    for (; li < nt; ++li) {
        const int i = t0 + li;  // the tile: keys 64 i .. 64 i + 63
        if (mma_w) {
            PFU_STAMP(0, 0);
            if (lane == 0 && !fail && li > 0) issue_pv(li - 1);
            PFU_STAMP(0, 1);
            if (lane == 0 && !fail && li + 1 < nt) fail = !issue_s(li + 1);
            __syncwarp();
            PFU_STAMP(0, 2);
        } else if (tma_w) {
            if (li + 2 < nt) {
                issue(li + 2, lane < 4 ? checked(nb_next) : 0, true);
                if (lane == 0) ++issued;
                nb_next = (lane < 4 && li + 3 < nt) ? tile_block_raw(i + 3, lane) : 0;
            }
            __syncwarp();
        } else {
            PFU_STAMP(1, 0);
            // ---- this thread's 32 scores of tile i
            fail |= !mbar_wait(&s_full[li & 1], (uint32_t)(li >> 1) & 1u, DEV_ERR_ATTN_WAIT);
            __syncwarp();
            tc_fence_after();
            PFU_STAMP(1, 1);
            float sv[32];
            tmem_ld32(tmem + lane_base + ((li & 1) ? 192u : 0u) + (uint32_t)(ch * 32), sv);
            PFU_STAMP(1, 2);
            const int lim = ctx_row - (i * kPfuKeys + ch * 32);  // keys of the row in this half-tile
            if (lim < 32)
#pragma unroll
                for (int k = 0; k < 32; ++k) sv[k] = k < lim ? sv[k] : -INFINITY;
            float mt = sv[0];
#pragma unroll
            for (int k = 1; k < 32; ++k) mt = fmaxf(mt, sv[k]);
            xch[ch * 128 + row] = mt;
            pair_sync(warp);
            mt = fmaxf(mt, xch[(ch ^ 1) * 128 + row]);
            PFU_STAMP(1, 3);
            float alpha = 1.f;
            bool rescale = false;
            if (mt != -INFINITY) {
                if (m_ref == -INFINITY) {
                    m_ref = mt;
                } else if (mt > m_ref + 8.f) {
                    alpha = ex2_approx(m_ref - mt);
                    l *= alpha;
                    m_ref = mt;
                    rescale = true;
                }
            }
            const float m_use = m_ref == -INFINITY ? 0.f : m_ref;  // a row with no keys yet: P = 0
            // ---- P = 2^(s - m) of this thread's 32 keys; written after the previous PV finished
            uint32_t ph[16], pl[16];
            float psum = 0.f;
#pragma unroll
            for (int k = 0; k < 16; ++k) {
                const float a = ex2_approx(sv[2 * k] - m_use), b2 = ex2_approx(sv[2 * k + 1] - m_use);
                psum += a + b2;
                split_h2(a, b2, ph[k], pl[k]);
            }
            l += psum;
            PFU_STAMP(1, 4);
            if (li > 0) fail |= !mbar_wait(pv_done, (uint32_t)(li - 1) & 1u, DEV_ERR_ATTN_WAIT);
            __syncwarp();
            tc_fence_after();
            PFU_STAMP(1, 5);
            if (__any_sync(0xffffffffu, rescale)) {  // warp-collective TMEM read-modify-write of O
#pragma unroll 1
                for (int c = 0; c < 64; c += 16) {
                    const uint32_t ta = tmem + lane_base + 64u + (uint32_t)(ch * 64 + c);
                    float v[16];
                    tmem_ld16(ta, v);
#pragma unroll
                    for (int k = 0; k < 16; ++k) v[k] *= alpha;
                    tmem_st16(ta, v);
                }
            }
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                const uint32_t off = sw128_off(row, ch * 32 + 8 * c);
                *reinterpret_cast<uint4*>(smem + L::PH + off) =
                    make_uint4(ph[4 * c], ph[4 * c + 1], ph[4 * c + 2], ph[4 * c + 3]);
                *reinterpret_cast<uint4*>(smem + L::PL + off) =
                    make_uint4(pl[4 * c], pl[4 * c + 1], pl[4 * c + 2], pl[4 * c + 3]);
            }
            // ---- the last tile's keys past the group's last one read whatever the pool holds
            // there: their V rows are zeroed so that P = 0 meets a finite V
            const int first_stale = ctx_max - i * kPfuKeys;
            if (i == ntiles - 1 && first_stale < kPfuKeys) {
                fail |= !mbar_wait(&kv_full[li % kPfuStages], (uint32_t)(li / kPfuStages) & 1u, DEV_ERR_ATTN_WAIT);
                uint8_t* vst = smem + L::RING + (li % kPfuStages) * L::STAGE + 2 * 8192;
                for (int c = t; c < (kPfuKeys - first_stale) * 16; c += kPfuSoftmaxWarps * 32) {
                    const int key = first_stale + (c >> 4), half = (c >> 3) & 1, chunk = c & 7;
                    *reinterpret_cast<uint4*>(vst + half * 8192 + key * 128 + chunk * 16) = make_uint4(0u, 0u, 0u, 0u);
                }
            }
            PFU_STAMP(1, 6);
        }
        fence_proxy_async_smem();
        tc_fence_before();
        const int any_fail = __syncthreads_or(fail ? 1 : 0);  // CTA-uniform
        tc_fence_after();
        if (any_fail) {
            fail = true;
            break;
        }
    }
    if (mma_w && lane == 0 && !fail) issue_pv(nt - 1);
    if (!ctrl) {
        // ---- after the last PV: O / l -> out (bf16 hi/lo) with one split, else O, the max and
        // the sum -> this split's partial (max -inf: no keys of the row here); the pair adds its
        // halves of l
        const bool good = !fail && mbar_wait(pv_done, (uint32_t)(nt - 1) & 1u, DEV_ERR_ATTN_WAIT);
        __syncwarp();
        tc_fence_after();
        xch[ch * 128 + row] = l;
        pair_sync(warp);
        const float l_row = l + xch[(ch ^ 1) * 128 + row];
        const bool final_out = nsplit == 1;
        const bool has_keys = good && m_ref != -INFINITY;
        const bool partial = !final_out && has_keys;  // its O goes to the workspace
        const float inv = final_out ? ((good && l_row > 0.f) ? 1.f / l_row : 0.f) : 1.f;
        if (row_ok && !final_out && ch == 0) {
            p.ws_ml[part_row * 2 + 0] = has_keys ? m_ref : -INFINITY;
            p.ws_ml[part_row * 2 + 1] = has_keys ? l_row : 0.f;
        }
#pragma unroll 1
        for (int c = 0; c < 64; c += 16) {
            float v[16];
            tmem_ld16(tmem + lane_base + 64u + (uint32_t)(ch * 64 + c), v);
            if (!good)
#pragma unroll
                for (int k = 0; k < 16; ++k) v[k] = 0.f;
            if (row_ok && partial) {
                float4* wo = reinterpret_cast<float4*>(p.ws_o + part_row * D + ch * 64 + c);
#pragma unroll
                for (int k = 0; k < 4; ++k) wo[k] = make_float4(v[4 * k], v[4 * k + 1], v[4 * k + 2], v[4 * k + 3]);
            }
            if (row_ok && final_out) {
                uint32_t hw[8], lw[8];
#pragma unroll
                for (int k = 0; k < 8; ++k) {
                    const float a = v[2 * k] * inv, b2 = v[2 * k + 1] * inv;
                    const __nv_bfloat162 hb = __floats2bfloat162_rn(a, b2);
                    const float2 hf = __bfloat1622float2(hb);
                    const __nv_bfloat162 lb = __floats2bfloat162_rn(a - hf.x, b2 - hf.y);
                    hw[k] = *reinterpret_cast<const uint32_t*>(&hb);
                    lw[k] = *reinterpret_cast<const uint32_t*>(&lb);
                }
                uint4* oh = reinterpret_cast<uint4*>(p.out + out_row * D + ch * 64 + c);
                oh[0] = make_uint4(hw[0], hw[1], hw[2], hw[3]);
                oh[1] = make_uint4(hw[4], hw[5], hw[6], hw[7]);
                if (p.out_lo) {
                    uint4* ol = reinterpret_cast<uint4*>(p.out_lo + out_row * D + ch * 64 + c);
                    ol[0] = make_uint4(lw[0], lw[1], lw[2], lw[3]);
                    ol[1] = make_uint4(lw[4], lw[5], lw[6], lw[7]);
                }
            }
        }
    } else if (lane == 0 && fail) {
        // after a failure: the loads in flight land and every UMMA finishes before TMEM is released
        if (tma_w)
            for (int j = issued > kPfuStages ? issued - kPfuStages : 0; j < issued; ++j)
                mbar_wait(&kv_full[j % kPfuStages], (uint32_t)(j / kPfuStages) & 1u, DEV_ERR_DRAIN);
        if (mma_w) {
            umma_commit(drain);
            mbar_wait(drain, 0, DEV_ERR_DRAIN);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (mma_w) tmem_dealloc(tmem, 256);
}


// ---------------------------------------------------------------------------
// The same attention with 128-key tiles and both UMMA A operands in TMEM: Q (fp16 hi/lo, 128
// columns) for S = Q K^T, P (fp16 hi/lo, 128 columns) for O += P V, so a 128-key tile takes
// 16 + 16 UMMAs of N = 128 instead of 2 x (16 of N = 64 + 8 of N = 128), and shared memory
// holds only the KV rings: K in 3 slots (its tile is loaded two windows ahead, as soon as the
// S that read the slot is done), V in 2 (loaded one window ahead, once the PV that read the
// slot is done). TMEM columns: Q hi 0..63, Q lo 64..127, S 128..255, P hi 256..319, P lo
// 320..383, O 384..511. Per window li: the softmax warps read S(li) and release it (s_free),
// the UMMA warp then issues S(li + 1) while they compute P(li), which they store to TMEM once
// PV(li - 1) is done; after the window's barrier the UMMA warp issues PV(li).
// ---------------------------------------------------------------------------
constexpr int kPf2Keys = 128;
constexpr int kPf2KSlots = 3, kPf2VSlots = 2;

struct Pf2Layout {
    static constexpr int SLOT = 2 * 128 * 128;                // 128 keys x 2 dim halves x 128 B
    static constexpr int KRING = 0;
    static constexpr int VRING = KRING + kPf2KSlots * SLOT;
    static constexpr int BAR = VRING + kPf2VSlots * SLOT;     // k_full[3], v_full[2], s_full, s_free, pv_done, drain, slot
    static constexpr int XCH = BAR + 128;
    static constexpr int SMEM = 1024 + XCH + 2 * 128 * 4;
};
static_assert(Pf2Layout::SMEM <= 227 * 1024, "prefill tile exceeds shared memory");

// D[tmem] (+)= A[tmem] * B[smem desc]^T, kind::f16 (A: M rows = TMEM lanes, two 16-bit
// elements per 32-bit column along K)
__device__ __forceinline__ void umma_ts_f16(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// 32 lanes x 32 bits, 16 consecutive columns of packed words (waits for the store)
__device__ __forceinline__ void tmem_st16_u(uint32_t taddr, const uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
            taddr),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]),
        "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
        : "memory");
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

__global__ void __launch_bounds__(kPfuThreads, 1) paged_prefill_umma128_kernel(const __grid_constant__ CUtensorMap tmKV,
                                                                                const AttnParams p) {
    constexpr int D = 128;
    using L = Pf2Layout;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* k_full = reinterpret_cast<uint64_t*>(smem + L::BAR);
    uint64_t* v_full = k_full + kPf2KSlots;
    uint64_t* s_full = v_full + kPf2VSlots;  // S(li) is in TMEM
    uint64_t* s_free = s_full + 1;           // the softmax threads have read S(li)
    uint64_t* pv_done = s_free + 1;
    uint64_t* drain = pv_done + 1;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
    float* xch = reinterpret_cast<float*>(smem + L::XCH);
    constexpr uint32_t kQ = 0, kS = 128, kP = 256, kO = 384;  // TMEM columns

    const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
    const bool mma_w = warp == kPfuSoftmaxWarps;      // issues the UMMAs (and owns TMEM)
    const bool tma_w = warp == kPfuSoftmaxWarps + 1;  // issues the KV loads
    const bool ctrl = mma_w || tma_w;
    griddep_wait();
    griddep_launch();
    const int SPS = p.rows_per_stream;
    const int n_streams = p.R / SPS;
    const int n_groups = (SPS + kPfuQ - 1) / kPfuQ;
    int rest = blockIdx.x;  // CTA-uniform
    const int g = rest % p.kv_heads;
    rest /= p.kv_heads;
    const int grp = rest % n_groups;
    rest /= n_groups;
    const int b = rest % n_streams;
    const int sp = rest / n_streams;  // key split sp of max_splits: a contiguous share of the group's tiles
    if (sp >= p.max_splits) return;
    const int nsplit = p.max_splits;
    const int q0 = grp * kPfuQ;
    const int nq = min(kPfuQ, SPS - q0);
    const int row = t & 127, ch = (t >> 7) & 1;  // softmax threads: TMEM lane and half
    const int h = row >> 6, qi = row & 63;
    const bool row_ok = !ctrl && qi < nq;
    const int r = b * SPS + q0 + qi;
    const int ctx_row = row_ok ? p.row_ctx[r] : 0;
    const int slot = p.row_slot[b * SPS];
    __shared__ int s_ctx;
    if (t == 0) s_ctx = 0;
    __syncthreads();
    if (row_ok && ch == 0) atomicMax(&s_ctx, ctx_row);
    __syncthreads();
    const int ctx_max = s_ctx;
    const size_t out_row = (size_t)r * p.num_heads + g * 2 + h;
    const size_t part_row = (size_t)out_row * nsplit + sp;
    if (ctx_max <= 0 || slot < 0) {  // CTA-uniform: nothing to attend (only after a scheduler error)
        if (ctx_max > 0 && t == 0 && sp == 0) record_error(DEV_ERR_ATTN_BOUNDS);
        if (row_ok && nsplit == 1)
            for (int d = ch * 64; d < ch * 64 + 64; ++d) {
                p.out[out_row * D + d] = __float2bfloat16(0.f);
                if (p.out_lo) p.out_lo[out_row * D + d] = __float2bfloat16(0.f);
            }
        if (row_ok && nsplit > 1 && ch == 0) {
            p.ws_ml[part_row * 2 + 0] = -INFINITY;
            p.ws_ml[part_row * 2 + 1] = 0.f;
        }
        return;
    }
    const int nbt = (ctx_max + 15) >> 4;
    const int ntiles = (ctx_max + kPf2Keys - 1) / kPf2Keys;
    const int t0 = (int)(((long long)sp * ntiles) / nsplit);
    const int nt = (int)(((long long)(sp + 1) * ntiles) / nsplit) - t0;
    if (nt <= 0) {
        if (row_ok && ch == 0) {
            p.ws_ml[part_row * 2 + 0] = -INFINITY;
            p.ws_ml[part_row * 2 + 1] = 0.f;
        }
        return;
    }

    // block j (0..7) of tile `tile` as the table holds it; past the group's keys any valid
    // block stands in (its keys are masked, its V zeroed)
    auto tile_block_raw = [&](int tile, int j) -> int {
        int jb = tile * 8 + j;
        if (jb >= nbt) jb = 0;
        return jb < p.mbps ? p.block_table[(size_t)slot * p.mbps + jb] : -1;
    };
    auto checked = [&](int blk) -> int {
        if (blk < 0 || blk >= p.num_blocks) {
            record_error(DEV_ERR_ATTN_BOUNDS);
            blk = 0;
        }
        return blk;
    };
    // TMA warp, converged: K (kind 0) or V (kind 1) of local tile li into its slot, one box per
    // lane 0..15 (lane = 2 j + half); lanes 0..7 hold the eight block ids
    auto issue_kv = [&](int kind, int li, int nb) {
        const int nslots = kind ? kPf2VSlots : kPf2KSlots;
        const int s2 = li % nslots;
        uint64_t* bar = kind ? &v_full[s2] : &k_full[s2];
        uint8_t* dst = smem + (kind ? L::VRING : L::KRING) + s2 * L::SLOT;
        const int blk = __shfl_sync(0xffffffffu, nb, (lane >> 1) & 7);
        if (lane == 0) mbar_arrive_expect_tx(bar, L::SLOT);
        __syncwarp();
        if (lane < 16) {
            const int j = lane >> 1, half = lane & 1;
            const int krow = (((blk * p.num_layers + p.layer) * 2 + kind) * p.kv_heads + g) * 16;
            tma_load_2d(dst + half * (128 * 128) + j * 2048, &tmKV, bar, half * 64, krow);
        }
    };

    int k_issued = 0, v_issued = 0;  // TMA lane 0
    int id_v = 0, id_k = 0;          // TMA lanes 0..7: checked ids of the next V tile, raw ids of the next K tile
    if (t == 0) {
        for (int s2 = 0; s2 < kPf2KSlots; ++s2) mbar_init(&k_full[s2], 1);
        for (int s2 = 0; s2 < kPf2VSlots; ++s2) mbar_init(&v_full[s2], 1);
        mbar_init(s_full, 1);
        mbar_init(s_free, kPfuSoftmaxWarps * 32);
        mbar_init(pv_done, 1);
        mbar_init(drain, 1);
        fence_mbar_init();
    }
    __syncthreads();
    if (mma_w) {
        tmem_alloc(tmem_slot, 512);
        tmem_relinquish();
    } else if (tma_w) {
        if (lane == 0) tma_prefetch_desc(&tmKV);
        const int id0 = lane < 8 ? checked(tile_block_raw(t0, lane)) : 0;
        issue_kv(0, 0, id0);
        issue_kv(1, 0, id0);
        k_issued = v_issued = 1;
        if (nt > 1) {
            const int id1 = lane < 8 ? checked(tile_block_raw(t0 + 1, lane)) : 0;
            issue_kv(0, 1, id1);
            k_issued = 2;
            id_v = id1;
        }
        id_k = (lane < 8 && nt > 2) ? tile_block_raw(t0 + 2, lane) : 0;
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
    if (!ctrl) {
        // ---- Q rows (x scale_log2) as an fp16 hi/lo pair into TMEM: dims 64 ch .. 64 ch + 63
        // are columns 32 ch .. 32 ch + 31 of each (two dims per column, the even one low)
        const float4* qp = reinterpret_cast<const float4*>(p.q + out_row * D + ch * 64);
        const float sc = p.scale_log2;
#pragma unroll
        for (int c = 0; c < 2; ++c) {  // 32 dims -> 16 columns
            uint32_t hi[16], lo[16];
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                const float4 x = row_ok ? qp[c * 8 + k] : make_float4(0.f, 0.f, 0.f, 0.f);
                split_h2(x.x * sc, x.y * sc, hi[2 * k], lo[2 * k]);
                split_h2(x.z * sc, x.w * sc, hi[2 * k + 1], lo[2 * k + 1]);
            }
            tmem_st16_u(tmem + lane_base + kQ + (uint32_t)(ch * 32 + c * 16), hi);
            tmem_st16_u(tmem + lane_base + kQ + 64u + (uint32_t)(ch * 32 + c * 16), lo);
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    // O's B operand (V) is MN-major: bit 16 of the instruction descriptor
    const uint32_t idesc_s = make_idesc_f16(128, kPf2Keys), idesc_o = make_idesc_f16(128, D) | (1u << 16);

    // UMMA lane 0: S(li) = Q K^T, A = Q from TMEM (k step kk: dims 16 kk .. : columns 8 kk ..)
    auto issue_s = [&](int li) -> bool {
        if (!mbar_wait(&k_full[li % kPf2KSlots], (uint32_t)(li / kPf2KSlots) & 1u, DEV_ERR_ATTN_WAIT)) return false;
        tc_fence_after();
        const uint32_t kb = smem_u32(smem + L::KRING + (li % kPf2KSlots) * L::SLOT);
#pragma unroll
        for (int part = 0; part < 2; ++part)
#pragma unroll
            for (int kk = 0; kk < 8; ++kk)
                umma_ts_f16(tmem + kS, tmem + kQ + (uint32_t)(part * 64 + kk * 8),
                            make_sw128_desc(kb + (kk >> 2) * (128 * 128)) + 2 * (kk & 3), idesc_s,
                            (part | kk) ? 1u : 0u);
        umma_commit(s_full);
        return true;
    };
    // UMMA lane 0: O (+)= P V, A = P from TMEM (16 keys per step: 8 columns), B = V MN-major in
    // its slot (LBO: the second 64 dims 16 KB on, 16 keys = 2048 B)
    auto issue_pv = [&](int li) -> bool {
        if (!mbar_wait(&v_full[li % kPf2VSlots], (uint32_t)(li / kPf2VSlots) & 1u, DEV_ERR_ATTN_WAIT)) return false;
        tc_fence_after();
        const uint32_t vb = smem_u32(smem + L::VRING + (li % kPf2VSlots) * L::SLOT);
#pragma unroll
        for (int part = 0; part < 2; ++part)
#pragma unroll
            for (int kk = 0; kk < 8; ++kk)
                umma_ts_f16(tmem + kO, tmem + kP + (uint32_t)(part * 64 + kk * 8),
                            make_sw128_mn_desc(vb + kk * 2048, 128 * 128), idesc_o,
                            (li > 0 || part > 0 || kk > 0) ? 1u : 0u);
        umma_commit(pv_done);
        return true;
    };

    bool fail = false;
    if (mma_w && lane == 0) fail = !issue_s(0);
    float m_ref = -INFINITY, l = 0.f;
    int li = 0;
    for (; li < nt; ++li) {
        const int i = t0 + li;  // the tile: keys 128 i .. 128 i + 127
        if (mma_w) {
            PFU_STAMP(0, 0);
            if (lane == 0 && !fail && li > 0) fail = !issue_pv(li - 1);
            PFU_STAMP(0, 1);
            if (lane == 0 && !fail && li + 1 < nt) {
                // S(li + 1) overwrites S(li): after the softmax threads have read it
                fail = !mbar_wait(s_free, (uint32_t)li & 1u, DEV_ERR_ATTN_WAIT);
                tc_fence_after();
                PFU_STAMP(0, 2);
                if (!fail) fail = !issue_s(li + 1);
            }
            __syncwarp();
            PFU_STAMP(0, 3);
        } else if (tma_w) {
            const bool dead = __shfl_sync(0xffffffffu, fail, 0);
            if (li + 2 < nt && !dead) {  // K of li + 2 into the slot S(li - 1) read
                const int idc = lane < 8 ? checked(id_k) : 0;
                issue_kv(0, li + 2, idc);
                if (lane == 0) ++k_issued;
                id_k = (lane < 8 && li + 3 < nt) ? tile_block_raw(i + 3, lane) : 0;
                if (li + 1 < nt) {
                    // V of li + 1 into the slot PV(li - 1) reads: once that PV is done
                    if (li > 0 && lane == 0) fail = !mbar_wait(pv_done, (uint32_t)(li - 1) & 1u, DEV_ERR_ATTN_WAIT);
                    if (!__shfl_sync(0xffffffffu, fail, 0)) {
                        issue_kv(1, li + 1, id_v);
                        if (lane == 0) ++v_issued;
                    }
                }
                id_v = idc;
            } else if (li + 1 < nt && !dead) {
                if (li > 0 && lane == 0) fail = !mbar_wait(pv_done, (uint32_t)(li - 1) & 1u, DEV_ERR_ATTN_WAIT);
                if (!__shfl_sync(0xffffffffu, fail, 0)) {
                    issue_kv(1, li + 1, id_v);
                    if (lane == 0) ++v_issued;
                }
            }
            __syncwarp();
        } else {
            PFU_STAMP(1, 0);
            // ---- this thread's 64 scores of tile i: columns 64 ch .. 64 ch + 63 of S
            fail |= !mbar_wait(s_full, (uint32_t)li & 1u, DEV_ERR_ATTN_WAIT);
            __syncwarp();
            tc_fence_after();
            PFU_STAMP(1, 1);
            float sv[64];
            {
                float a32[32];
                tmem_ld32(tmem + lane_base + kS + (uint32_t)(ch * 64), a32);
#pragma unroll
                for (int k = 0; k < 32; ++k) sv[k] = a32[k];
                tmem_ld32(tmem + lane_base + kS + (uint32_t)(ch * 64 + 32), a32);
#pragma unroll
                for (int k = 0; k < 32; ++k) sv[32 + k] = a32[k];
            }
            tc_fence_before();
            mbar_arrive(s_free);  // S may be overwritten: the UMMA warp issues S(li + 1)
            PFU_STAMP(1, 2);
            const int lim = ctx_row - (i * kPf2Keys + ch * 64);  // keys of the row in this half-tile
            if (lim < 64)
#pragma unroll
                for (int k = 0; k < 64; ++k) sv[k] = k < lim ? sv[k] : -INFINITY;
            float mt = sv[0];
#pragma unroll
            for (int k = 1; k < 64; ++k) mt = fmaxf(mt, sv[k]);
            xch[ch * 128 + row] = mt;
            pair_sync(warp);
            mt = fmaxf(mt, xch[(ch ^ 1) * 128 + row]);
            PFU_STAMP(1, 3);
            float alpha = 1.f;
            bool rescale = false;
            if (mt != -INFINITY) {
                if (m_ref == -INFINITY) {
                    m_ref = mt;
                } else if (mt > m_ref + 8.f) {
                    alpha = ex2_approx(m_ref - mt);
                    l *= alpha;
                    m_ref = mt;
                    rescale = true;
                }
            }
            const float m_use = m_ref == -INFINITY ? 0.f : m_ref;
            // ---- P = 2^(s - m), an fp16 hi/lo pair per key, two keys per column (even one low);
            // the first 32 keys' words are formed while PV(li - 1) still reads P(li - 1)
            float psum = 0.f;
            uint32_t wh[16], wl[16];
#pragma unroll
            for (int k = 0; k < 16; ++k) {
                const float a = ex2_approx(sv[2 * k] - m_use), b2 = ex2_approx(sv[2 * k + 1] - m_use);
                psum += a + b2;
                split_h2(a, b2, wh[k], wl[k]);
            }
            // P(li) replaces P(li - 1) in TMEM and O is rescaled: both once PV(li - 1) is done
            if (li > 0) fail |= !mbar_wait(pv_done, (uint32_t)(li - 1) & 1u, DEV_ERR_ATTN_WAIT);
            __syncwarp();
            tc_fence_after();
            PFU_STAMP(1, 4);
            if (__any_sync(0xffffffffu, rescale)) {  // warp-collective TMEM read-modify-write of O
#pragma unroll 1
                for (int c = 0; c < 64; c += 16) {
                    const uint32_t ta = tmem + lane_base + kO + (uint32_t)(ch * 64 + c);
                    float v[16];
                    tmem_ld16(ta, v);
#pragma unroll
                    for (int k = 0; k < 16; ++k) v[k] *= alpha;
                    tmem_st16(ta, v);
                }
            }
            tmem_st16_u(tmem + lane_base + kP + (uint32_t)(ch * 32), wh);
            tmem_st16_u(tmem + lane_base + kP + 64u + (uint32_t)(ch * 32), wl);
#pragma unroll
            for (int k = 0; k < 16; ++k) {
                const float a = ex2_approx(sv[32 + 2 * k] - m_use), b2 = ex2_approx(sv[33 + 2 * k] - m_use);
                psum += a + b2;
                split_h2(a, b2, wh[k], wl[k]);
            }
            tmem_st16_u(tmem + lane_base + kP + (uint32_t)(ch * 32 + 16), wh);
            tmem_st16_u(tmem + lane_base + kP + 64u + (uint32_t)(ch * 32 + 16), wl);
            l += psum;
            PFU_STAMP(1, 5);
            // ---- the last tile's keys past the group's last one: V rows zeroed (P = 0 meets a
            // finite V)
            const int first_stale = ctx_max - i * kPf2Keys;
            if (i == ntiles - 1 && first_stale < kPf2Keys) {
                fail |= !mbar_wait(&v_full[li % kPf2VSlots], (uint32_t)(li / kPf2VSlots) & 1u, DEV_ERR_ATTN_WAIT);
                uint8_t* vst = smem + L::VRING + (li % kPf2VSlots) * L::SLOT;
                for (int c = t; c < (kPf2Keys - first_stale) * 16; c += kPfuSoftmaxWarps * 32) {
                    const int key = first_stale + (c >> 4), half = (c >> 3) & 1, chunk = c & 7;
                    *reinterpret_cast<uint4*>(vst + half * (128 * 128) + key * 128 + chunk * 16) =
                        make_uint4(0u, 0u, 0u, 0u);
                }
            }
            PFU_STAMP(1, 6);
        }
        fence_proxy_async_smem();
        tc_fence_before();
        const int any_fail = __syncthreads_or(fail ? 1 : 0);
        tc_fence_after();
        if (any_fail) {
            fail = true;
            break;
        }
    }
    if (mma_w && lane == 0 && !fail) fail = !issue_pv(nt - 1);
    if (!ctrl) {
        const bool good = !fail && mbar_wait(pv_done, (uint32_t)(nt - 1) & 1u, DEV_ERR_ATTN_WAIT);
        __syncwarp();
        tc_fence_after();
        xch[ch * 128 + row] = l;
        pair_sync(warp);
        const float l_row = l + xch[(ch ^ 1) * 128 + row];
        const bool final_out = nsplit == 1;
        const bool has_keys = good && m_ref != -INFINITY;
        const bool partial = !final_out && has_keys;
        const float inv = final_out ? ((good && l_row > 0.f) ? 1.f / l_row : 0.f) : 1.f;
        if (row_ok && !final_out && ch == 0) {
            p.ws_ml[part_row * 2 + 0] = has_keys ? m_ref : -INFINITY;
            p.ws_ml[part_row * 2 + 1] = has_keys ? l_row : 0.f;
        }
#pragma unroll 1
        for (int c = 0; c < 64; c += 16) {
            float v[16];
            tmem_ld16(tmem + lane_base + kO + (uint32_t)(ch * 64 + c), v);
            if (!good)
#pragma unroll
                for (int k = 0; k < 16; ++k) v[k] = 0.f;
            if (row_ok && partial) {
                float4* wo = reinterpret_cast<float4*>(p.ws_o + part_row * D + ch * 64 + c);
#pragma unroll
                for (int k = 0; k < 4; ++k) wo[k] = make_float4(v[4 * k], v[4 * k + 1], v[4 * k + 2], v[4 * k + 3]);
            }
            if (row_ok && final_out) {
                uint32_t hw[8], lw[8];
#pragma unroll
                for (int k = 0; k < 8; ++k) {
                    const float a = v[2 * k] * inv, b2 = v[2 * k + 1] * inv;
                    const __nv_bfloat162 hb = __floats2bfloat162_rn(a, b2);
                    const float2 hf = __bfloat1622float2(hb);
                    const __nv_bfloat162 lb = __floats2bfloat162_rn(a - hf.x, b2 - hf.y);
                    hw[k] = *reinterpret_cast<const uint32_t*>(&hb);
                    lw[k] = *reinterpret_cast<const uint32_t*>(&lb);
                }
                uint4* oh = reinterpret_cast<uint4*>(p.out + out_row * D + ch * 64 + c);
                oh[0] = make_uint4(hw[0], hw[1], hw[2], hw[3]);
                oh[1] = make_uint4(hw[4], hw[5], hw[6], hw[7]);
                if (p.out_lo) {
                    uint4* ol = reinterpret_cast<uint4*>(p.out_lo + out_row * D + ch * 64 + c);
                    ol[0] = make_uint4(lw[0], lw[1], lw[2], lw[3]);
                    ol[1] = make_uint4(lw[4], lw[5], lw[6], lw[7]);
                }
            }
        }
    } else if (lane == 0 && fail) {
        // after a failure: the loads in flight land and every UMMA finishes before TMEM is released
        if (tma_w) {
            for (int j = k_issued > kPf2KSlots ? k_issued - kPf2KSlots : 0; j < k_issued; ++j)
                mbar_wait(&k_full[j % kPf2KSlots], (uint32_t)(j / kPf2KSlots) & 1u, DEV_ERR_DRAIN);
            for (int j = v_issued > kPf2VSlots ? v_issued - kPf2VSlots : 0; j < v_issued; ++j)
                mbar_wait(&v_full[j % kPf2VSlots], (uint32_t)(j / kPf2VSlots) & 1u, DEV_ERR_DRAIN);
        }
        if (mma_w) {
            umma_commit(drain);
            mbar_wait(drain, 0, DEV_ERR_DRAIN);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (mma_w) tmem_dealloc(tmem, 512);
}

// Folds the key splits of paged_prefill_umma_kernel: one warp per (row, q head), lane d4 owns
// dims 4 d4 .. 4 d4 + 3; a partial whose max is -inf holds no keys and is skipped.
__global__ void __launch_bounds__(128) prefill_combine_kernel(const AttnParams p) {
    constexpr int D = 128;
    griddep_wait();
    griddep_launch();
    const int pair = blockIdx.x * 4 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (pair >= p.R * p.num_heads) return;
    const int k = p.max_splits;
    const float* ml = p.ws_ml + (size_t)pair * k * 2;
    float M = -INFINITY;
    for (int s2 = 0; s2 < k; ++s2) M = fmaxf(M, ml[2 * s2]);
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    float lsum = 0.f;
    if (M != -INFINITY)
        for (int s2 = 0; s2 < k; ++s2) {
            const float ms = ml[2 * s2];
            if (ms == -INFINITY) continue;
            const float f = exp2f(ms - M);
            const float4 o = reinterpret_cast<const float4*>(p.ws_o + ((size_t)pair * k + s2) * D)[lane];
            acc.x += o.x * f;
            acc.y += o.y * f;
            acc.z += o.z * f;
            acc.w += o.w * f;
            lsum += ml[2 * s2 + 1] * f;
        }
    const float inv = lsum > 0.f ? 1.f / lsum : 0.f;
    const float v[4] = {acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv};
    uint32_t hw[2], lw[2];
#pragma unroll
    for (int k2 = 0; k2 < 2; ++k2) {
        const __nv_bfloat162 hb = __floats2bfloat162_rn(v[2 * k2], v[2 * k2 + 1]);
        const float2 hf = __bfloat1622float2(hb);
        const __nv_bfloat162 lb = __floats2bfloat162_rn(v[2 * k2] - hf.x, v[2 * k2 + 1] - hf.y);
        hw[k2] = *reinterpret_cast<const uint32_t*>(&hb);
        lw[k2] = *reinterpret_cast<const uint32_t*>(&lb);
    }
    reinterpret_cast<uint2*>(p.out + (size_t)pair * D)[lane] = make_uint2(hw[0], hw[1]);
    if (p.out_lo) reinterpret_cast<uint2*>(p.out_lo + (size_t)pair * D)[lane] = make_uint2(lw[0], lw[1]);
}

// Key splits of the tcgen05 prefill: with fewer (stream, group, kv head) CTAs than half the SMs,
// each group's tiles are shared by up to floor(SMs / CTAs) CTAs (at most the workspace's
// max_splits and kPfuMaxSplits; QTTS_PREFILL_SPLITS caps it, 1 = never split).
constexpr int kPfuMaxSplits = 16;
inline int prefill_umma_split_cap() {
    static const int c = [] {
        const char* v = getenv("QTTS_PREFILL_SPLITS");
        const int x = (v && *v) ? atoi(v) : kPfuMaxSplits;
        return (x >= 1 && x <= kPfuMaxSplits) ? x : kPfuMaxSplits;
    }();
    return c;
}

// QTTS_PREFILL_UMMA: 1 = 64-key tiles (Q and P in shared memory), 2 = 128-key tiles with Q and P
// in TMEM, unset = 2 for chunks of 128 rows or more per stream (long chunks, whose pasts tend to
// be long too, gain from the wider tiles; short chunks lose to their partial last tile)
inline int attn_prefill_umma_form(int rows_per_stream) {
    static const int f = [] {
        const char* v = getenv("QTTS_PREFILL_UMMA");
        return (v && (*v == '1' || *v == '2')) ? (*v - '0') : 0;
    }();
    return f ? f : (rows_per_stream >= 128 ? 2 : 1);
}

inline int launch_prefill_umma(const AttnParams& p, cudaStream_t st) {
    CUtensorMap map;
    const int rc = make_kv_map(&map, p);
    if (rc) return rc;
    const bool wide = attn_prefill_umma_form(p.rows_per_stream) == 2;
    if (wide) QTTS_CHECK_CUDA((func_attr_once<paged_prefill_umma128_kernel>(Pf2Layout::SMEM)));
    else QTTS_CHECK_CUDA((func_attr_once<paged_prefill_umma_kernel>(PfuLayout::SMEM)));
    const int n_groups = (p.rows_per_stream + kPfuQ - 1) / kPfuQ;
    const int base = (p.R / p.rows_per_stream) * n_groups * p.kv_heads;
    const int sms = num_sms();
    int k = 1;
    const bool ws_ok = p.ws_o && p.ws_ml && (reinterpret_cast<uintptr_t>(p.ws_o) & 15) == 0;
    if (ws_ok && 2 * base <= sms) k = min(min(sms / base, p.max_splits), prefill_umma_split_cap());
    AttnParams q = p;
    q.max_splits = k > 1 ? k : 1;  // the workspace stride: k partials per (row, q head)
    if (wide)
        QTTS_LAUNCH(paged_prefill_umma128_kernel, dim3(base * q.max_splits), dim3(kPfuThreads), Pf2Layout::SMEM, st,
                    map, q);
    else
        QTTS_LAUNCH(paged_prefill_umma_kernel, dim3(base * q.max_splits), dim3(kPfuThreads), PfuLayout::SMEM, st,
                    map, q);
    if (q.max_splits > 1)
        QTTS_LAUNCH(prefill_combine_kernel, dim3(ceil_div(q.R * q.num_heads, 4)), dim3(128), 0, st, q);
    return QTTS_OK;
}

// Prefill attention on the tcgen05 tensor pipe (head_dim 128, 2 query heads per KV head) unless
// QTTS_PREFILL_UMMA=0 (the mma.sync query-tile kernel); 1 / 2 pick its form (above).
inline bool attn_prefill_umma() {
    static const bool on = [] {
        const char* v = getenv("QTTS_PREFILL_UMMA");
        return !(v && *v == '0');
    }();
    return on;
}

// The engine's prefill steps use the query-tile kernel unless QTTS_PREFILL_TILES=0 (one row per
// query through the decode kernel).
inline bool attn_prefill_tiles() {
    static const bool on = [] {
        const char* v = getenv("QTTS_PREFILL_TILES");
        return !(v && *v == '0');
    }();
    return on;
}

// Prefill rows (head_dim 128): query tiles share each KV block; the split partials fold as in decode.
inline int launch_prefill_attention(const AttnParams& p, cudaStream_t st) {
    if (p.R <= 0) return QTTS_OK;
    if (p.rows_per_stream < 1 || p.R % p.rows_per_stream != 0) {
        set_error("prefill attention: %d rows are not streams of %d tokens", p.R, p.rows_per_stream);
        return QTTS_ERR_INVALID;
    }
    const bool aligned = ((reinterpret_cast<uintptr_t>(p.q) | reinterpret_cast<uintptr_t>(p.out) |
                           reinterpret_cast<uintptr_t>(p.out_lo)) & 15) == 0;
    if (p.num_heads == 2 * p.kv_heads && aligned && attn_prefill_umma()) return launch_prefill_umma(p, st);
    const int rc = launch_prefill_tc<2>(p, st);
    if (rc) return rc;
    if (p.max_splits > 1) QTTS_LAUNCH(attn_combine_kernel<128>, dim3(p.R, p.num_heads), dim3(128), 0, st, p);
    return QTTS_OK;
}

// The engine's decode steps let the row kernel read its metadata and start its first loads
// before the wait on the preceding launch (AttnParams::meta_settled) unless QTTS_ATTN_EARLY=0.
inline bool attn_early() {
    static const bool on = [] {
        const char* v = getenv("QTTS_ATTN_EARLY");
        return !(v && *v == '0');
    }();
    return on;
}

// head_dim 128 runs on the tensor pipe unless QTTS_ATTN_TC=0
inline bool attn_use_tc() {
    static const bool on = [] {
        const char* v = getenv("QTTS_ATTN_TC");
        return !(v && *v == '0');
    }();
    return on;
}

template <int D>
inline int launch_attention_d(const AttnParams& p, cudaStream_t st) {
    int rc;
    if (D == 128 && attn_use_tc() && attn_rows())
        return attn_stages() == 3 ? launch_attention_tc_rows<3>(p, st) : launch_attention_tc_rows<2>(p, st);
    if (D == 128 && attn_use_tc()) {
        rc = attn_stages() == 3 ? launch_attention_tc<3>(p, st) : launch_attention_tc<2>(p, st);
        if (rc) return rc;
        if (p.max_splits > 1) QTTS_LAUNCH(attn_combine_kernel<D>, dim3(p.R, p.num_heads), dim3(D), 0, st, p);
        return QTTS_OK;
    }
    switch (attn_stages()) {
        case 3: rc = launch_attention_s<D, 3>(p, st); break;
        case 4: rc = launch_attention_s<D, 4>(p, st); break;
        default: rc = launch_attention_s<D, 2>(p, st); break;
    }
    if (rc) return rc;
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
