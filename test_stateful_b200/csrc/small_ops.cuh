// Bandwidth-bound helper kernels on the decode path: RMSNorm, embedding
// gathers, the codec embedding sum, KV block copy / scatter / gather, and the
// row bookkeeping of the code predictor.
#pragma once

#include "common.cuh"

namespace qtts {

// ---------------------------------------------------------------------------
// RMSNorm (Qwen3RMSNorm): y = w * x * rsqrt(mean(x^2) + eps), fp32 in, bf16 out.
// With y_lo, the bf16 residual y - bf16(y) is stored too (the hi/lo operand of
// the tcgen05 GEMM).
// ---------------------------------------------------------------------------
__device__ __forceinline__ void store_hilo4(__nv_bfloat16* hi, __nv_bfloat16* lo, float a, float b, float c, float d) {
    __nv_bfloat162 h01 = __floats2bfloat162_rn(a, b);
    __nv_bfloat162 h23 = __floats2bfloat162_rn(c, d);
    uint2 pack;
    pack.x = *reinterpret_cast<uint32_t*>(&h01);
    pack.y = *reinterpret_cast<uint32_t*>(&h23);
    *reinterpret_cast<uint2*>(hi) = pack;
    if (lo) {
        __nv_bfloat162 l01 = __floats2bfloat162_rn(a - __low2float(h01), b - __high2float(h01));
        __nv_bfloat162 l23 = __floats2bfloat162_rn(c - __low2float(h23), d - __high2float(h23));
        pack.x = *reinterpret_cast<uint32_t*>(&l01);
        pack.y = *reinterpret_cast<uint32_t*>(&l23);
        *reinterpret_cast<uint2*>(lo) = pack;
    }
}

__global__ void __launch_bounds__(256) rmsnorm_kernel(const float* __restrict__ x, int H, int ld,
                                                      const __nv_bfloat16* __restrict__ w, float eps,
                                                      __nv_bfloat16* __restrict__ y, __nv_bfloat16* __restrict__ y_lo) {
    __shared__ float red[8];
    const int r = blockIdx.x;
    griddep_wait();
    griddep_launch();
    const float* xr = x + (size_t)r * ld;
    float ss = 0.f;
    for (int i = threadIdx.x * 4; i < H; i += 1024) {
        const float4 v = *reinterpret_cast<const float4*>(xr + i);
        ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
    }
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) tot += red[i];
    const float inv = rsqrtf(tot / (float)H + eps);
    __nv_bfloat16* yr = y + (size_t)r * H;
    __nv_bfloat16* yl = y_lo ? y_lo + (size_t)r * H : nullptr;
    for (int i = threadIdx.x * 4; i < H; i += 1024) {
        const float4 v = *reinterpret_cast<const float4*>(xr + i);
        const __nv_bfloat162 w01 = *reinterpret_cast<const __nv_bfloat162*>(w + i);
        const __nv_bfloat162 w23 = *reinterpret_cast<const __nv_bfloat162*>(w + i + 2);
        store_hilo4(yr + i, yl ? yl + i : nullptr, v.x * inv * __low2float(w01), v.y * inv * __high2float(w01),
                    v.z * inv * __low2float(w23), v.w * inv * __high2float(w23));
    }
}

inline int launch_rmsnorm(const float* x, int M, int H, int ld, const void* w, float eps, void* y, cudaStream_t st,
                          void* y_lo = nullptr) {
    if (M <= 0) return QTTS_OK;
    if (H % 4 != 0 || ld % 4 != 0) {
        set_error("rmsnorm: H and ld must be multiples of 4");
        return QTTS_ERR_UNSUPPORTED;
    }
    QTTS_LAUNCH(rmsnorm_kernel, dim3(M), dim3(256), 0, st, x, H, ld, reinterpret_cast<const __nv_bfloat16*>(w), eps,
                reinterpret_cast<__nv_bfloat16*>(y), reinterpret_cast<__nv_bfloat16*>(y_lo));
    return QTTS_OK;
}

// ---------------------------------------------------------------------------
// row gathers
// ---------------------------------------------------------------------------
// Input of code-predictor stages 1..14: the stage's codec embedding row already projected to the
// code predictor's width (table = emb_s · W_proj^T + b_proj, computed once at load: the projection
// is linear and its inputs are a fixed table), written as the residual stream x, plus what the
// first layer's folded input norm needs: the bf16 pair of x∘γ and per-128-column sums of x².
// Run by the whole CTA of row r (the code predictor's sampling kernel, right after it picks the
// code); warp w of an iteration covers the 128 columns of tile (w + iteration·warps).
__device__ __forceinline__ void embed_projected_row(const float* __restrict__ table, int V, int H, int64_t id,
                                                    const __nv_bfloat16* __restrict__ gamma, float* __restrict__ x,
                                                    __nv_bfloat16* __restrict__ xn, __nv_bfloat16* __restrict__ xn_lo,
                                                    float* __restrict__ ss, int r) {
    if (id < 0 || id >= V) id = 0;  // stay in bounds; callers pass sampled (valid) ids
    const float4* src = reinterpret_cast<const float4*>(table + (size_t)id * H);
    for (int c4 = threadIdx.x; c4 < H / 4; c4 += blockDim.x) {
        const float4 v = src[c4];
        reinterpret_cast<float4*>(x + (size_t)r * H)[c4] = v;
        const float a[4] = {v.x, v.y, v.z, v.w};
        float sq = 0.f;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const int c = c4 * 4 + k;
            const float xg = a[k] * __bfloat162float(gamma[c]);
            const __nv_bfloat16 hi = __float2bfloat16(xg);
            xn[(size_t)r * H + c] = hi;
            xn_lo[(size_t)r * H + c] = __float2bfloat16(xg - __bfloat162float(hi));
            sq += a[k] * a[k];
        }
        sq = warp_sum(sq);
        if ((threadIdx.x & 31) == 0) ss[(size_t)r * (H / 128) + c4 / 32] = sq;
    }
}


// Stage-0 input of the code predictor: rows [2b] = hidden[b], [2b+1] = codec_emb[tok0[b]]
// (CodePredictorUnrolled.forward, utils.py:1019-1020), as a hi/lo operand pair
// (the embedding is exact in bf16, its lo row is zero).
__global__ void cp_stage0_rows_kernel(const __nv_bfloat16* __restrict__ hidden, const __nv_bfloat16* __restrict__ hidden_lo,
                                      const __nv_bfloat16* __restrict__ emb, int V, int H,
                                      const int64_t* __restrict__ tok, int tok_ld, __nv_bfloat16* __restrict__ out,
                                      __nv_bfloat16* __restrict__ out_lo) {
    const int b = blockIdx.x;
    griddep_wait();
    griddep_launch();
    int64_t id = tok[(size_t)b * tok_ld];
    if (id < 0 || id >= V) id = 0;
    const uint4* h = reinterpret_cast<const uint4*>(hidden + (size_t)b * H);
    const uint4* hl = reinterpret_cast<const uint4*>(hidden_lo + (size_t)b * H);
    const uint4* e = reinterpret_cast<const uint4*>(emb + (size_t)id * H);
    uint4* o0 = reinterpret_cast<uint4*>(out + (size_t)(2 * b) * H);
    uint4* o1 = reinterpret_cast<uint4*>(out + (size_t)(2 * b + 1) * H);
    uint4* l0 = reinterpret_cast<uint4*>(out_lo + (size_t)(2 * b) * H);
    uint4* l1 = reinterpret_cast<uint4*>(out_lo + (size_t)(2 * b + 1) * H);
    const uint4 z = make_uint4(0, 0, 0, 0);
    for (int i = threadIdx.x; i < H / 8; i += blockDim.x) {
        o0[i] = h[i];
        o1[i] = e[i];
        l0[i] = hl[i];
        l1[i] = z;
    }
}

// ---------------------------------------------------------------------------
// codec embedding sum + next input embedding
// ---------------------------------------------------------------------------
__global__ void codec_sum_kernel(const int64_t* __restrict__ codes, int G, const __nv_bfloat16* __restrict__ t0,
                                 int V0, const __nv_bfloat16* __restrict__ tc, int Vc, int H,
                                 const float* __restrict__ text_add, float* __restrict__ csum,
                                 float* __restrict__ next_x, const int32_t* __restrict__ row_map,
                                 int32_t* __restrict__ noise_step) {
    const int r = blockIdx.x;
    griddep_wait();
    griddep_launch();
    const size_t orow = row_map ? (size_t)row_map[r] : (size_t)r;  // output / text row
    if (noise_step && threadIdx.x == 0) noise_step[orow] += 1;     // this stream sampled one more frame
    extern __shared__ int64_t ids[];
    for (int g = threadIdx.x; g < G; g += blockDim.x) {
        int64_t c = codes[(size_t)r * G + g];
        const int64_t lim = g == 0 ? V0 : Vc;
        ids[g] = (c < 0 || c >= lim) ? -1 : c;  // CP tables are zero beyond Vc (codec_embedding_sum.py:46-49)
    }
    __syncthreads();
    for (int h = threadIdx.x * 2; h < H; h += blockDim.x * 2) {
        float a = 0.f, b = 0.f;
        for (int g = 0; g < G; ++g) {
            const int64_t id = ids[g];
            if (id < 0) continue;
            const __nv_bfloat16* row = g == 0 ? t0 + (size_t)id * H : tc + ((size_t)(g - 1) * Vc + id) * H;
            const __nv_bfloat162 v = *reinterpret_cast<const __nv_bfloat162*>(row + h);
            a += __low2float(v);
            b += __high2float(v);
        }
        if (csum) {
            csum[orow * H + h] = a;
            csum[orow * H + h + 1] = b;
        }
        if (text_add) {
            a += text_add[orow * H + h];
            b += text_add[orow * H + h + 1];
        }
        next_x[orow * H + h] = a;
        next_x[orow * H + h + 1] = b;
    }
}

// x[r] = x_in[row_map ? row_map[r] : r]  (the residual stream starts in fp32)
__global__ void load_x_kernel(const float* __restrict__ x_in, float* __restrict__ x, int rows, int H,
                              const int32_t* __restrict__ row_map) {
    griddep_wait();
    griddep_launch();
    const size_t n = (size_t)rows * H;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const size_t r = i / H, c = i % H;
        const size_t src = row_map ? (size_t)row_map[r] : r;
        x[i] = x_in[src * H + c];
    }
}

// ---------------------------------------------------------------------------
// KV pool: block copy (copy-on-write), row scatter / gather
// ---------------------------------------------------------------------------
__global__ void kv_copy_blocks_kernel(uint4* __restrict__ pool, size_t block_vec, const int32_t* __restrict__ src,
                                      const int32_t* __restrict__ dst, int num_blocks) {
    const int i = blockIdx.y;
    griddep_wait();
    griddep_launch();
    const int s = src[i], d = dst[i];
    if (s < 0 || d < 0 || s >= num_blocks || d >= num_blocks) return;
    const uint4* a = pool + (size_t)s * block_vec;
    uint4* b = pool + (size_t)d * block_vec;
    for (size_t k = (size_t)blockIdx.x * blockDim.x + threadIdx.x; k < block_vec; k += (size_t)gridDim.x * blockDim.x)
        b[k] = a[k];
}

// rows [n][L2][Hkv][D] -> pool[(blk, l2, g, off, d)]   (KV element type kv_t)
__global__ void kv_scatter_kernel(kv_t* __restrict__ pool, int L2, int Hkv, int D, int bs, int num_blocks,
                                  const kv_t* __restrict__ rows, const int32_t* __restrict__ mapping) {
    const int i = blockIdx.x;
    const int m = mapping[i];
    if (m < 0) return;
    const int blk = m / bs, off = m % bs;
    if (blk >= num_blocks) return;
    const int per = L2 * Hkv * D;
    for (int e = threadIdx.x; e < per; e += blockDim.x) {
        const int d = e % D, g = (e / D) % Hkv, l2 = e / (D * Hkv);
        pool[((((size_t)blk * L2 + l2) * Hkv + g) * bs + off) * D + d] = rows[(size_t)i * per + e];
    }
}

// out [L2][Hkv][n][D] from the slot's block table
__global__ void kv_gather_kernel(const kv_t* __restrict__ pool, int L2, int Hkv, int D, int bs,
                                 int num_blocks, const int32_t* __restrict__ table_row, int n,
                                 kv_t* __restrict__ out) {
    const int t = blockIdx.x;
    int blk = table_row[t / bs];
    const int off = t % bs;
    const bool ok = blk >= 0 && blk < num_blocks;
    const int per = L2 * Hkv * D;
    for (int e = threadIdx.x; e < per; e += blockDim.x) {
        const int d = e % D, g = (e / D) % Hkv, l2 = e / (D * Hkv);
        const kv_t v = ok ? pool[((((size_t)blk * L2 + l2) * Hkv + g) * bs + off) * D + d] : __float2half(0.f);
        out[(((size_t)l2 * Hkv + g) * n + t) * D + d] = v;
    }
}

// row -> slot map for n_rows x n_new rows: row i*n_new+j belongs to slots[i]
__global__ void expand_rows_kernel(const int32_t* __restrict__ slots, int n_rows, int n_new, int32_t* __restrict__ out) {
    griddep_wait();
    griddep_launch();
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n_rows * n_new; i += gridDim.x * blockDim.x)
        out[i] = slots[i / n_new];
}

}  // namespace qtts
