// Code-predictor stage in one launch: a thread-block cluster per 8 streams.
//
// A code-predictor stage s >= 1 (utils.py:1003-1042, KV-cached: one new token
// per stream at position s + 1) is 5 transformer layers + the stage's lm_head,
// about 24 MB of bf16 weights per layer, all resident in L2 across the 15
// stages.  Run as separate GEMM launches it is a chain of ~26 dependent
// kernels of ~8 us each, every one a few microseconds of launch / dependency
// latency around half a microsecond of work.  Here one cluster of 16 CTAs
// (one per SM, 512 threads) carries a group of 8 streams through the whole
// stage:
//
//  * the residual stream x [8][1024] fp32 is replicated in every CTA's shared
//    memory; each CTA computes the RMSNorm of all 8 rows itself and keeps the
//    GEMM operand as a bf16 hi/lo pair (hi = bf16(v), lo = bf16(v - hi)), so
//    the products keep ~16 mantissa bits of the fp32 activation;
//  * weights stream straight from L2 into registers in mma.sync A-fragment
//    order (packed once at load, 16 B per lane per 16 x 16 tile, coalesced),
//    a prefetch ring per warp, two m16n8k16 bf16 MMAs (hi, lo) per tile;
//  * QKV, O, gate/up and the lm_head split their output rows over the 16
//    CTAs; the down projection splits K by the SwiGLU features each CTA just
//    computed, and its partial sums are reduce-scattered through distributed
//    shared memory;
//  * q/k RMSNorm + RoPE, the new K/V row into the paged code-predictor cache,
//    attention over the stream's s + 2 keys, SwiGLU and the residual adds are
//    epilogues between phases; slices computed by one CTA reach the others
//    with st.shared::cluster stores, and phases are separated by hardware
//    cluster barriers (every CTA runs the same barrier sequence: there is no
//    early exit and no spin-wait in the kernel).
//
// The stage's logits [stream][2048] go to global memory for the sampling
// kernel, which forms the next stage's input as before.
#pragma once

#include "common.cuh"

namespace qtts {

constexpr int kCpcTok = 8;        // streams per cluster (the mma N dimension)
constexpr int kCpcCtas = 16;      // CTAs per cluster
constexpr int kCpcWarps = 16;
constexpr int kCpcThreads = kCpcWarps * 32;
constexpr int kCpcH = 1024, kCpcI = 3072, kCpcHq = 16, kCpcHkv = 8, kCpcD = 64, kCpcL = 5, kCpcV = 2048;
constexpr int kCpcQkv = (kCpcHq + 2 * kCpcHkv) * kCpcD;  // 2048 rows
constexpr int kCpcActLd = kCpcH + 8;                    // bf16 per operand row (16-B pad: conflict-free B loads)
constexpr int kCpcFeat = kCpcI / kCpcCtas;              // 192 SwiGLU features per CTA
constexpr int kCpcFeatLd = kCpcFeat + 8;
#ifndef CPC_PF
#define CPC_PF 4
#endif
constexpr int kCpcPf = CPC_PF;                          // weight tiles in flight per warp

// optional per-phase timestamps (a profiling build defines CPC_STAMP(i))
#ifndef CPC_STAMP
#define CPC_STAMP(i) \
    do {             \
    } while (0)
#endif

struct CpClusterParams {
    int nr;       // streams (rows of x_in / logits)
    int stage;    // s >= 1
    int bmax;     // rows of the KV cache
    const float* x_in;  // [nr][1024] the stage's input
    float* logits;      // [nr][2048]
    kv_t* kv;           // [bmax][5][2][8][16][64] fp16
    const uint4* w_qkv[kCpcL];   // packed [128 m-tiles][64 k-tiles][32 lanes]
    const uint4* w_o[kCpcL];     // packed [64][64][32]
    const uint4* w_gu[kCpcL];    // packed [384][64][32] (gate/up interleaved in 64-row groups)
    const uint4* w_down[kCpcL];  // packed per CTA: [16 ranks][64 m-tiles][12 k-tiles][32]
    const uint4* w_head;         // packed [128][64][32], this stage's lm_head
    const __nv_bfloat16* in_norm;    // [5][1024]
    const __nv_bfloat16* post_norm;  // [5][1024]
    const __nv_bfloat16* q_norm;     // [5][64]
    const __nv_bfloat16* k_norm;     // [5][64]
    const __nv_bfloat16* final_norm; // [1024]
    const float* rope_cos;  // [max_pos][32]
    const float* rope_sin;
    float eps;
};

// shared memory layout (bytes)
struct CpcSmem {
    static constexpr int XS = 0;                                           // float [8][1024]
    static constexpr int ACT_HI = XS + kCpcTok * kCpcH * 4;                // bf16 [8][1032]
    static constexpr int ACT_LO = ACT_HI + kCpcTok * kCpcActLd * 2;
    static constexpr int FEAT_HI = ACT_LO + kCpcTok * kCpcActLd * 2;       // bf16 [8][200]
    static constexpr int FEAT_LO = FEAT_HI + kCpcTok * kCpcFeatLd * 2;
    static constexpr int OUT = FEAT_LO + kCpcTok * kCpcFeatLd * 2;         // float [8][384]
    static constexpr int PART = OUT + kCpcTok * 384 * 4;                   // float [48 units][32][4]
    static constexpr int RECV = PART + 48 * 32 * 4 * 4;                    // float [16 src][8][64]
    static constexpr int QS = RECV + kCpcCtas * kCpcTok * 64 * 4;          // float [8][128]
    static constexpr int INV = QS + kCpcTok * 128 * 4;                     // float [8]
    static constexpr int BYTES = INV + 64;
};

__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], const uint4& a, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a.x), "r"(a.y), "r"(a.z), "r"(a.w), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint4 ldg_frag(const uint4* p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

// One m-tile (16 weight rows) x 8 tokens over nks k-tiles: weight fragments from global
// (packed, `wa` at the first k-tile, 32 uint4 per k-tile), operand tokens x k from shared
// memory as a bf16 hi/lo pair (row stride ld elements, starting at column k0).
__device__ __forceinline__ void cpc_mma_unit(const uint4* __restrict__ wa, int nks, const __nv_bfloat16* bhi,
                                             const __nv_bfloat16* blo, int ld, int k0, int lane, float (&acc)[4]) {
    const int gq = lane >> 2, qq = lane & 3;
    const __nv_bfloat16* ph = bhi + gq * ld + k0 + 2 * qq;
    const __nv_bfloat16* pl = blo + gq * ld + k0 + 2 * qq;
    uint4 ring[kCpcPf];
#pragma unroll
    for (int i = 0; i < kCpcPf; ++i) ring[i] = i < nks ? ldg_frag(wa + i * 32 + lane) : make_uint4(0, 0, 0, 0);
    for (int k0s = 0; k0s < nks; k0s += kCpcPf) {
#pragma unroll
        for (int j = 0; j < kCpcPf; ++j) {
            const int ks = k0s + j;
            if (ks < nks) {
                const uint4 a = ring[j];
                if (ks + kCpcPf < nks) ring[j] = ldg_frag(wa + (ks + kCpcPf) * 32 + lane);
                const uint32_t h0 = *reinterpret_cast<const uint32_t*>(ph + 16 * ks);
                const uint32_t h1 = *reinterpret_cast<const uint32_t*>(ph + 16 * ks + 8);
                const uint32_t l0 = *reinterpret_cast<const uint32_t*>(pl + 16 * ks);
                const uint32_t l1 = *reinterpret_cast<const uint32_t*>(pl + 16 * ks + 8);
                mma_bf16_16816(acc, a, h0, h1);
                mma_bf16_16816(acc, a, l0, l1);
            }
        }
    }
}

// C fragment of a unit -> the partial buffer (lane-major, 4 floats per lane)
__device__ __forceinline__ void cpc_store_part(float* part, int unit, int lane, const float (&acc)[4]) {
    *reinterpret_cast<float4*>(part + ((size_t)unit * 32 + lane) * 4) = make_float4(acc[0], acc[1], acc[2], acc[3]);
}

// sum of the P k-parts of local row `row` (of R_c) for token t -> out[t][row]
__device__ __forceinline__ float cpc_gather(const float* part, int P, int row, int t) {
    const int mt = row >> 4, i = row & 15;
    const int lane = (i & 7) * 4 + (t >> 1);
    const int e = (i >= 8 ? 2 : 0) + (t & 1);
    float s = 0.f;
    for (int p = 0; p < P; ++p) s += part[((size_t)(mt * P + p) * 32 + lane) * 4 + e];
    return s;
}

// GEMM phase: this CTA's R_c = 16 * n_mt rows over K = 16 * nks_total, split into P k-parts;
// weights for local m-tile m at global m-tile (mt0 + m) of a packed matrix with ks_total
// k-tiles per row; result (summed over k-parts) into out[t][row] (ld_out floats per token).
__device__ __forceinline__ void cpc_gemm_rows(const uint4* __restrict__ w, int mt0, int n_mt, int ks_total, int P,
                                              const __nv_bfloat16* bhi, const __nv_bfloat16* blo, int ld, float* part,
                                              float* out, int ld_out) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int units = n_mt * P, nks = ks_total / P;
    for (int u = warp; u < units; u += kCpcWarps) {
        const int m = u / P, p = u % P;
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
        cpc_mma_unit(w + ((size_t)(mt0 + m) * ks_total + (size_t)p * nks) * 32, nks, bhi, blo, ld, p * nks * 16, lane,
                     acc);
        cpc_store_part(part, u, lane, acc);
    }
    __syncthreads();
    const int R = n_mt * 16;
    for (int e = threadIdx.x; e < R * kCpcTok; e += kCpcThreads) {
        const int t = e / R, row = e % R;
        out[t * ld_out + row] = cpc_gather(part, P, row, t);
    }
    __syncthreads();
}

// x (fp32, shared, replicated) -> bf16 hi/lo operand of RMSNorm(x) * w
__device__ __forceinline__ void cpc_norm(const float* xs, const __nv_bfloat16* w, float eps, float* inv,
                                         __nv_bfloat16* ahi, __nv_bfloat16* alo) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (warp < kCpcTok) {
        float ss = 0.f;
        for (int c = lane; c < kCpcH; c += 32) {
            const float v = xs[warp * kCpcH + c];
            ss += v * v;
        }
        ss = warp_sum(ss);
        if (lane == 0) inv[warp] = rsqrtf(ss / (float)kCpcH + eps);
    }
    __syncthreads();
    for (int e = threadIdx.x; e < kCpcTok * kCpcH / 2; e += kCpcThreads) {
        const int t = e / (kCpcH / 2), c = 2 * (e % (kCpcH / 2));
        const float v0 = xs[t * kCpcH + c] * inv[t] * __bfloat162float(w[c]);
        const float v1 = xs[t * kCpcH + c + 1] * inv[t] * __bfloat162float(w[c + 1]);
        const __nv_bfloat162 hi = __floats2bfloat162_rn(v0, v1);
        const float2 hf = __bfloat1622float2(hi);
        *reinterpret_cast<__nv_bfloat162*>(ahi + t * kCpcActLd + c) = hi;
        *reinterpret_cast<__nv_bfloat162*>(alo + t * kCpcActLd + c) = __floats2bfloat162_rn(v0 - hf.x, v1 - hf.y);
    }
    __syncthreads();
}

// the 64 columns [64 rank, +64) of x for all tokens, from this CTA to every CTA of the cluster
__device__ __forceinline__ void cpc_broadcast_xslice(float* xs, int rank) {
    const uint32_t base = smem_u32(xs);
    for (int e = threadIdx.x; e < kCpcCtas * kCpcTok * 16; e += kCpcThreads) {
        const int peer = e / (kCpcTok * 16), r = e % (kCpcTok * 16);
        const int t = r / 16, c4 = r % 16;
        const int col = 64 * rank + 4 * c4;
        const float4 v = *reinterpret_cast<const float4*>(xs + t * kCpcH + col);
        st_dsmem_f32x4(map_to_rank(base + (uint32_t)(t * kCpcH + col) * 4u, (uint32_t)peer), v.x, v.y, v.z, v.w);
    }
}

__device__ __forceinline__ void st_dsmem_b32(uint32_t addr, uint32_t v) {
    asm volatile("st.shared::cluster.b32 [%0], %1;" ::"r"(addr), "r"(v) : "memory");
}

__device__ __forceinline__ void st_dsmem_f32(uint32_t addr, float v) {
    asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}

__global__ void __launch_bounds__(kCpcThreads, 1) cp_cluster_stage_kernel(const CpClusterParams p) {
    extern __shared__ __align__(16) uint8_t smem[];
    float* xs = reinterpret_cast<float*>(smem + CpcSmem::XS);
    __nv_bfloat16* act_hi = reinterpret_cast<__nv_bfloat16*>(smem + CpcSmem::ACT_HI);
    __nv_bfloat16* act_lo = reinterpret_cast<__nv_bfloat16*>(smem + CpcSmem::ACT_LO);
    __nv_bfloat16* feat_hi = reinterpret_cast<__nv_bfloat16*>(smem + CpcSmem::FEAT_HI);
    __nv_bfloat16* feat_lo = reinterpret_cast<__nv_bfloat16*>(smem + CpcSmem::FEAT_LO);
    float* outb = reinterpret_cast<float*>(smem + CpcSmem::OUT);
    float* part = reinterpret_cast<float*>(smem + CpcSmem::PART);
    float* recv = reinterpret_cast<float*>(smem + CpcSmem::RECV);
    float* qs = reinterpret_cast<float*>(smem + CpcSmem::QS);
    float* inv = reinterpret_cast<float*>(smem + CpcSmem::INV);

    const int rank = (int)cluster_ctarank();
    const int b0 = (blockIdx.x / kCpcCtas) * kCpcTok;  // first stream of this cluster
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int pos = p.stage + 1, ctx = p.stage + 2;     // the new token's position, keys visible
    const float scale = rsqrtf((float)kCpcD);

    griddep_wait();  // x_in comes from the previous stage's sampling kernel
    for (int e = threadIdx.x; e < kCpcTok * kCpcH; e += kCpcThreads) {
        const int t = e / kCpcH, c = e % kCpcH;
        xs[e] = b0 + t < p.nr ? p.x_in[(size_t)(b0 + t) * kCpcH + c] : 0.f;
    }
    __syncthreads();
    CPC_STAMP(0);

    for (int l = 0; l < kCpcL; ++l) {
        // ---- input norm, QKV rows [128 rank, +128)
        cpc_norm(xs, p.in_norm + (size_t)l * kCpcH, p.eps, inv, act_hi, act_lo);
        cpc_gemm_rows(p.w_qkv[l], 8 * rank, 8, kCpcH / 16, 2, act_hi, act_lo, kCpcActLd, part, outb, 128);
        CPC_STAMP(1 + 7 * l);
        // ---- epilogue per (token, head of this CTA): q/k RMSNorm + RoPE; q kept, k/v to the cache
        {
            const int t = warp >> 1, hh = warp & 1;  // 16 warps = 8 tokens x 2 heads
            const int region = rank < 8 ? 0 : (rank < 12 ? 1 : 2);  // q / k / v rows
            float v0 = outb[t * 128 + 64 * hh + 2 * lane], v1 = outb[t * 128 + 64 * hh + 2 * lane + 1];
            if (region < 2) {
                const __nv_bfloat16* nw = (region == 0 ? p.q_norm : p.k_norm) + (size_t)l * kCpcD;
                const float r = rsqrtf(warp_sum(v0 * v0 + v1 * v1) / (float)kCpcD + p.eps);
                v0 *= r * __bfloat162float(nw[2 * lane]);
                v1 *= r * __bfloat162float(nw[2 * lane + 1]);
                // rotate-half RoPE: dims d < 32 pair with d + 32 (lane l <-> l ^ 16)
                const float w0 = __shfl_xor_sync(0xffffffffu, v0, 16), w1 = __shfl_xor_sync(0xffffffffu, v1, 16);
                const int dd = (2 * lane) & 31;
                const float c0 = p.rope_cos[pos * 32 + dd], s0 = p.rope_sin[pos * 32 + dd];
                const float c1 = p.rope_cos[pos * 32 + dd + 1], s1 = p.rope_sin[pos * 32 + dd + 1];
                if (lane < 16) {
                    v0 = v0 * c0 - w0 * s0;
                    v1 = v1 * c1 - w1 * s1;
                } else {
                    v0 = v0 * c0 + w0 * s0;
                    v1 = v1 * c1 + w1 * s1;
                }
            }
            if (region == 0) {
                qs[t * 128 + 64 * hh + 2 * lane] = v0;
                qs[t * 128 + 64 * hh + 2 * lane + 1] = v1;
            } else if (b0 + t < p.nr && b0 + t < p.bmax) {
                const int head = 2 * (rank - (region == 1 ? 8 : 12)) + hh;
                kv_t* dst = p.kv + (((((size_t)(b0 + t) * kCpcL + l) * 2 + (region - 1)) * kCpcHkv + head) * 16 + pos) *
                                       kCpcD + 2 * lane;
                *reinterpret_cast<__half2*>(dst) = __halves2half2(to_kv(v0), to_kv(v1));
            }
        }
        cluster_sync();  // A: the new K/V rows are in the cache; every CTA is done reading act
        CPC_STAMP(2 + 7 * l);
        // ---- attention: CTA r < 8 owns q heads 2r, 2r+1 (kv head r); one warp per (token, head)
        if (rank < 8) {
            const int t = warp >> 1, hh = warp & 1, head = 2 * rank + hh;
            const bool ok = b0 + t < p.nr && b0 + t < p.bmax;
            float o0 = 0.f, o1 = 0.f;
            if (ok) {
                const kv_t* kb = p.kv + ((((size_t)(b0 + t) * kCpcL + l) * 2 + 0) * kCpcHkv + rank) * 16 * kCpcD;
                const kv_t* vb = kb + (size_t)kCpcHkv * 16 * kCpcD;
                float sc = -INFINITY;
                if (lane < ctx) {
                    const float* q = qs + t * 128 + 64 * hh;
                    float acc = 0.f;
#pragma unroll
                    for (int d8 = 0; d8 < kCpcD / 8; ++d8) {
                        const uint4 raw = *reinterpret_cast<const uint4*>(kb + lane * kCpcD + 8 * d8);
                        const __half2* hp = reinterpret_cast<const __half2*>(&raw);
#pragma unroll
                        for (int j = 0; j < 4; ++j) {
                            const float2 kf = __half22float2(hp[j]);
                            acc += q[8 * d8 + 2 * j] * kf.x + q[8 * d8 + 2 * j + 1] * kf.y;
                        }
                    }
                    sc = acc * scale;
                }
                const float mx = warp_max(sc);
                const float pk = lane < ctx ? __expf(sc - mx) : 0.f;
                const float inv_l = 1.f / warp_sum(pk);
                for (int k = 0; k < ctx; ++k) {
                    const float pkk = __shfl_sync(0xffffffffu, pk, k);
                    const float2 vf = __half22float2(*reinterpret_cast<const __half2*>(vb + k * kCpcD + 2 * lane));
                    o0 += pkk * vf.x;
                    o1 += pkk * vf.y;
                }
                o0 *= inv_l;
                o1 *= inv_l;
            }
            // the head's output, as the O projection's hi/lo operand, into every CTA of the cluster
            const __nv_bfloat162 hi = __floats2bfloat162_rn(o0, o1);
            const float2 hf = __bfloat1622float2(hi);
            const __nv_bfloat162 lo = __floats2bfloat162_rn(o0 - hf.x, o1 - hf.y);
            const int col = 64 * head + 2 * lane;
            const uint32_t ah = smem_u32(act_hi + t * kCpcActLd + col), al = smem_u32(act_lo + t * kCpcActLd + col);
            for (int peer = 0; peer < kCpcCtas; ++peer) {
                st_dsmem_b32(map_to_rank(ah, (uint32_t)peer), *reinterpret_cast<const uint32_t*>(&hi));
                st_dsmem_b32(map_to_rank(al, (uint32_t)peer), *reinterpret_cast<const uint32_t*>(&lo));
            }
        }
        cluster_sync();  // B: every CTA holds the whole attention output
        CPC_STAMP(3 + 7 * l);
        // ---- O rows [64 rank, +64) + residual, slice to every CTA
        cpc_gemm_rows(p.w_o[l], 4 * rank, 4, kCpcH / 16, 4, act_hi, act_lo, kCpcActLd, part, outb, 64);
        for (int e = threadIdx.x; e < kCpcTok * 64; e += kCpcThreads) {
            const int t = e / 64, c = e % 64;
            xs[t * kCpcH + 64 * rank + c] += outb[t * 64 + c];
        }
        __syncthreads();
        cpc_broadcast_xslice(xs, rank);
        cluster_sync();  // C: x complete in every CTA
        CPC_STAMP(4 + 7 * l);
        // ---- post-attention norm, gate/up rows [384 rank, +384) -> SwiGLU features [192 rank, +192)
        cpc_norm(xs, p.post_norm + (size_t)l * kCpcH, p.eps, inv, act_hi, act_lo);
        cpc_gemm_rows(p.w_gu[l], 24 * rank, 24, kCpcH / 16, 2, act_hi, act_lo, kCpcActLd, part, outb, 384);
        for (int e = threadIdx.x; e < kCpcTok * kCpcFeat; e += kCpcThreads) {
            const int t = e / kCpcFeat, f = e % kCpcFeat;
            const int tile = f / 64, j = f % 64;
            const float g = outb[t * 384 + 128 * tile + j], u = outb[t * 384 + 128 * tile + 64 + j];
            const float a = __fdividef(g, 1.0f + __expf(-g)) * u;
            const __nv_bfloat16 hi = __float2bfloat16(a);
            feat_hi[t * kCpcFeatLd + f] = hi;
            feat_lo[t * kCpcFeatLd + f] = __float2bfloat16(a - __bfloat162float(hi));
        }
        __syncthreads();
        CPC_STAMP(5 + 7 * l);
        // ---- down: all 1024 output rows over this CTA's 192 features; partial columns
        // [64 j, +64) go to CTA j (reduce-scatter)
        {
            const uint4* w = p.w_down[l] + (size_t)rank * 64 * (kCpcFeat / 16) * 32;
            const uint32_t rbase = smem_u32(recv);
            for (int m = warp; m < 64; m += kCpcWarps) {
                float acc[4] = {0.f, 0.f, 0.f, 0.f};
                cpc_mma_unit(w + (size_t)m * (kCpcFeat / 16) * 32, kCpcFeat / 16, feat_hi, feat_lo, kCpcFeatLd, 0,
                             lane, acc);
                const int dst = m >> 2, gq = lane >> 2, qq = lane & 3;
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int i = gq + (e >= 2 ? 8 : 0), t = 2 * qq + (e & 1);
                    const int c = (m & 3) * 16 + i;
                    st_dsmem_f32(map_to_rank(rbase + (uint32_t)((rank * kCpcTok + t) * 64 + c) * 4u, (uint32_t)dst),
                                 acc[e]);
                }
            }
        }
        cluster_sync();  // D: every CTA's partials for its columns have arrived
        CPC_STAMP(6 + 7 * l);
        for (int e = threadIdx.x; e < kCpcTok * 64; e += kCpcThreads) {
            const int t = e / 64, c = e % 64;
            float s = 0.f;
            for (int src = 0; src < kCpcCtas; ++src) s += recv[(src * kCpcTok + t) * 64 + c];  // fixed order
            xs[t * kCpcH + 64 * rank + c] += s;
        }
        __syncthreads();
        cpc_broadcast_xslice(xs, rank);
        cluster_sync();  // E: x complete in every CTA
        CPC_STAMP(7 + 7 * l);
    }
    // ---- final norm, lm_head rows [128 rank, +128) -> logits
    cpc_norm(xs, p.final_norm, p.eps, inv, act_hi, act_lo);
    cpc_gemm_rows(p.w_head, 8 * rank, 8, kCpcH / 16, 2, act_hi, act_lo, kCpcActLd, part, outb, 128);
    CPC_STAMP(36);
    griddep_launch();
    for (int e = threadIdx.x; e < kCpcTok * 128; e += kCpcThreads) {
        const int t = e / 128, c = e % 128;
        if (b0 + t < p.nr) p.logits[(size_t)(b0 + t) * kCpcV + 128 * rank + c] = outb[t * 128 + c];
    }
    cluster_sync();  // no CTA leaves while a peer may still write into its shared memory
}

// Pack rows of W [N][ld] (bf16, columns [c0, c0 + Kp)) into mma.sync m16n8k16 A fragments:
// out[(mt * Kp / 16 + ks) * 32 + lane] = the lane's four bf16 pairs of tile (mt, ks).
__global__ void pack_a_frag_kernel(const __nv_bfloat16* W, int ld, int c0, int N, int Kp, uint4* out) {
    const int KS = Kp / 16;
    const size_t total = (size_t)(N / 16) * KS * 32;
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= total) return;
    const int lane = (int)(i % 32), ks = (int)((i / 32) % KS), mt = (int)(i / (32 * (size_t)KS));
    const int gq = lane >> 2, qq = lane & 3;
    const int r0 = 16 * mt + gq, r1 = r0 + 8, k = c0 + 16 * ks + 2 * qq;
    const uint32_t* w32 = reinterpret_cast<const uint32_t*>(W);
    auto pair = [&](int r, int kk) { return w32[((size_t)r * ld + kk) / 2]; };  // kk even: an aligned bf16 pair
    out[i] = make_uint4(pair(r0, k), pair(r1, k), pair(r0, k + 8), pair(r1, k + 8));
}

inline int pack_a_frag(const __nv_bfloat16* W, int ld, int c0, int N, int Kp, uint4* out, cudaStream_t st) {
    const size_t total = (size_t)(N / 16) * (Kp / 16) * 32;
    pack_a_frag_kernel<<<(unsigned)((total + 255) / 256), 256, 0, st>>>(W, ld, c0, N, Kp, out);
    QTTS_LAUNCH_CHECK();
    return QTTS_OK;
}

inline int launch_cp_cluster_stage(const CpClusterParams& p, cudaStream_t st) {
    QTTS_CHECK_CUDA((func_attr_once<cp_cluster_stage_kernel>(CpcSmem::BYTES, /*nonportable_cluster=*/true)));
    const int clusters = (p.nr + kCpcTok - 1) / kCpcTok;
    const cudaError_t e = launch_pdl(cp_cluster_stage_kernel, dim3(clusters * kCpcCtas), dim3(kCpcThreads),
                                     CpcSmem::BYTES, st, dim3(kCpcCtas, 1, 1), p);
    if (e != cudaSuccess) {
        set_error("launch of cp_cluster_stage_kernel failed: %s", cudaGetErrorString(e));
        return QTTS_ERR_CUDA;
    }
    return QTTS_OK;
}

}  // namespace qtts
