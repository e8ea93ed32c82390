// Streaming code2wav decoder: one frame per stream per step
// (Code2WavStreamingWrapper.forward, scripts/export/code2wav_streaming.py:708-810,
// as export_09_talker_code2wav_fused.py:145-160 drives it at T = 1).
//
// Layout.  Every activation that a causal convolution reads is kept in a
// slot-indexed history buffer [slot][ctx + T][C]: rows [0, ctx) hold the
// left context carried from the previous step (the reference's conv states,
// code2wav_streaming.py:159-193), rows [ctx, ctx + T) this step's frames.  A
// producer (a GEMM epilogue) writes the ACTIVATED values there (SnakeBeta is
// applied before the convolution in the reference, and the carried state is
// of activated values too: code2wav_streaming.py:73-93, 845-853), the
// convolution reads taps t + j*d, and one roll kernel at the end of the step
// moves the last ctx rows to the front — 21 buffers, the reference's 17 conv
// + 4 transposed-conv states.  A transposed conv (kernel 2s, stride s) reads
// [x(i-1) | x(i)] from a ctx = 1 buffer: the previous input frame replaces the
// reference's bias-free overlap tail, which equals W[:, :, s:] x(i-1).
//
// Convolutions run as tcgen05 GEMMs (gemm_tc.cuh).  Where a stream's step has
// a multiple of 128 rows (the residual convolutions of blocks 2-3 and block 3's
// transposed conv), the GEMM reads its operand tiles by TMA straight from the
// history buffer (implicit convolution: tap j is a row offset of j*dilation;
// those buffers pad channels to a multiple of 64); the short ones go through an
// im2col gather.  The fused epilogue adds bias, scales/residual-adds, applies
// the NEXT activation and scatters into the next history buffer.
// Decoder transformer: RMSNorm kernel + QKV GEMM whose epilogue does q/k norm,
// RoPE at the stream's frame index and stores K/V into a per-slot ring of
// `window` frames (the sliding-window cache, code2wav_streaming.py:29-66 with
// the executor's crop to window-1 past frames, executor.py:68-79, 1374-1441);
// the ring is read in any order because softmax attention over keys that
// already carry their RoPE phase is order-free.
#pragma once

#include <vector>

#include <algorithm>

#include "engine.cuh"

namespace qtts {

inline int pad64(int x) { return (x + 63) / 64 * 64; }
inline int pad128(int x) { return (x + 127) / 128 * 128; }

// ---------------------------------------------------------------------------
// RVQ decode (code2wav_streaming.py:681-706): q = sum_g table_g[clamp(code_g)]
// with the output projections folded into the tables by the host.  Writes the
// pre_conv input row, and the per-row frame bookkeeping of this step.
// ---------------------------------------------------------------------------
// One CTA per (stream s, frame t of the chunk): row rr = s * F + t.
__global__ void __launch_bounds__(256) c2w_rvq_kernel(const float* __restrict__ tables, int G, int V, int CD,
                                                      const int64_t* __restrict__ codes, int codes_ld, int F,
                                                      const int32_t* __restrict__ slots, int max_slots,
                                                      const int32_t* __restrict__ frame, int window, int max_frames,
                                                      int32_t* __restrict__ row_slot, int32_t* __restrict__ row_pos,
                                                      int32_t* __restrict__ row_kv, int32_t* __restrict__ row_nkeys,
                                                      int32_t* __restrict__ row_lo, ActView dst) {
    const int rr = blockIdx.x, r = rr / F, t = rr - r * F;
    griddep_wait();
    griddep_launch();
    // every later kernel of the step indexes state through row_slot: a slot
    // outside [0, max_slots) is redirected to the spare slot max_slots
    int slot = slots[r];
    if (slot < 0 || slot >= max_slots) {
        if (threadIdx.x == 0) record_error(DEV_ERR_BAD_SLOT);
        slot = max_slots;
    }
    __shared__ int idx[32];
    if (threadIdx.x < G) {
        long long c = codes[(size_t)rr * codes_ld + threadIdx.x];
        c = c < 0 ? 0 : (c >= V ? V - 1 : c);  // export_09_talker_code2wav_fused.py:146
        idx[threadIdx.x] = (int)c;
    }
    __syncthreads();
    for (int c = threadIdx.x; c < CD; c += blockDim.x) {
        float acc = 0.f;
        for (int g = 0; g < G; ++g) acc += tables[((size_t)g * V + idx[g]) * CD + c];
        reinterpret_cast<__nv_bfloat16*>(dst.ptr)[view_index(dst, r, slot, t, c)] = __float2bfloat16(acc);
    }
    if (threadIdx.x == 0) {
        // frame t of the chunk sees min(f0, window - F) past frames and the chunk's frames up to t
        // (the executor's max_past = window - chunk, executor.py:1374-1380); the ring holds frame
        // f at position f % window, and the chunk's writes never land on a frame it still reads
        const int f0 = frame[slot], f = f0 + t;
        const int nk = min(f0, window - F) + t + 1;
        if (t == 0) row_slot[r] = slot;
        row_pos[rr] = f < max_frames ? f : max_frames - 1;
        row_kv[rr] = slot * window + f % window;
        row_nkeys[rr] = nk;
        row_lo[rr] = (f + 1 - nk) % window;
    }
}

// ---------------------------------------------------------------------------
// im2col over a history buffer: X[r*T + t][j*C + c] = H[slot][t + j*d][c] for
// j < taps, zero up to K (tile padding).  8 bf16 per thread-iteration.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) c2w_im2col_kernel(const __nv_bfloat16* __restrict__ H, int seq_rows, int C,
                                                         int taps, int dil, int T, const int32_t* __restrict__ slots,
                                                         int n, __nv_bfloat16* __restrict__ X, int K) {
    griddep_wait();
    griddep_launch();
    const int kv = K >> 3;
    const size_t total = (size_t)n * T * kv;
    for (size_t v = (size_t)blockIdx.x * blockDim.x + threadIdx.x; v < total; v += (size_t)gridDim.x * blockDim.x) {
        const int row = (int)(v / kv), k = (int)(v % kv) * 8;
        const int r = row / T, t = row - r * T;
        const int j = k / C, c = k - j * C;
        uint4 val = make_uint4(0, 0, 0, 0);
        if (j < taps)
            val = *reinterpret_cast<const uint4*>(H + ((size_t)slots[r] * seq_rows + t + j * dil) * C + c);
        *reinterpret_cast<uint4*>(X + (size_t)row * K + k) = val;
    }
}

// ---------------------------------------------------------------------------
// window attention of the decoder transformer (one query frame per stream):
// keys are ring positions [0, nkeys) of the stream's slot.  One warp per head.
// q fp32 [n][heads*D]; ring [slot][layers][2][heads][window][D] (fp16).
// ---------------------------------------------------------------------------
template <int D>
__global__ void __launch_bounds__(128) c2w_attn_kernel(const float* __restrict__ q, const kv_t* __restrict__ ring,
                                                       int heads, int layers, int layer, int window, int F,
                                                       const int32_t* __restrict__ slots,
                                                       const int32_t* __restrict__ nkeys,
                                                       const int32_t* __restrict__ lo, float scale,
                                                       __nv_bfloat16* __restrict__ out,
                                                       __nv_bfloat16* __restrict__ out_lo) {
    static_assert(D == 32 || D == 64, "head_dim 32 or 64");
    constexpr int PER = D / 32;  // output dims per lane
    __shared__ float qs[4][D];
    const int r = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int h = blockIdx.y * 4 + warp;
    griddep_wait();
    griddep_launch();
    if (h >= heads) return;
    const int slot = slots[r / F];  // row r = (stream, frame of the chunk)
    const int n = nkeys[r], k0 = lo[r];
    for (int d = lane; d < D; d += 32) qs[warp][d] = q[((size_t)r * heads + h) * D + d];
    __syncwarp();
    const size_t kbase = ((((size_t)slot * layers + layer) * 2 + 0) * heads + h) * window * D;
    const size_t vbase = ((((size_t)slot * layers + layer) * 2 + 1) * heads + h) * window * D;
    float s[3];
    float mx = -INFINITY;
#pragma unroll
    for (int c = 0; c < 3; ++c) {
        const int k = c * 32 + lane;
        s[c] = -INFINITY;
        if (k < n) {
            const kv_t* kr = ring + kbase + (size_t)((k0 + k) % window) * D;
            float acc = 0.f;
#pragma unroll
            for (int d = 0; d < D; d += 8) {
                const uint4 u = *reinterpret_cast<const uint4*>(kr + d);
                const __half2* hp = reinterpret_cast<const __half2*>(&u);
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float2 f = __half22float2(hp[e]);
                    acc += f.x * qs[warp][d + 2 * e] + f.y * qs[warp][d + 2 * e + 1];
                }
            }
            s[c] = acc * scale;
            mx = fmaxf(mx, s[c]);
        }
    }
    mx = warp_max(mx);
    float sum = 0.f;
#pragma unroll
    for (int c = 0; c < 3; ++c) {
        s[c] = (c * 32 + lane < n) ? __expf(s[c] - mx) : 0.f;
        sum += s[c];
    }
    sum = warp_sum(sum);
    float o[PER];
#pragma unroll
    for (int e = 0; e < PER; ++e) o[e] = 0.f;
#pragma unroll
    for (int c = 0; c < 3; ++c) {
        for (int j = 0; j < 32; ++j) {
            const int k = c * 32 + j;
            if (k >= n) break;  // uniform across the warp
            const float pk = __shfl_sync(0xffffffffu, s[c], j);
            const kv_t* vr = ring + vbase + (size_t)((k0 + k) % window) * D;
#pragma unroll
            for (int e = 0; e < PER; ++e) o[e] += pk * __half2float(vr[lane * PER + e]);
        }
    }
    const float inv = 1.0f / sum;
#pragma unroll
    for (int e = 0; e < PER; ++e) {
        const float v = o[e] * inv;
        const size_t oi = ((size_t)r * heads + h) * D + lane * PER + e;
        const __nv_bfloat16 hi = __float2bfloat16(v);
        out[oi] = hi;
        if (out_lo) out_lo[oi] = __float2bfloat16(v - __bfloat162float(hi));
    }
}

// ---------------------------------------------------------------------------
// ConvNeXt front (code2wav_streaming.py:819-827): depthwise causal conv k7 over
// the history buffer (fp32) + LayerNorm over channels -> bf16 GEMM operand.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) c2w_dwconv_ln_kernel(const float* __restrict__ H, int seq_rows, int C, int T,
                                                            const int32_t* __restrict__ slots,
                                                            const float* __restrict__ w, const float* __restrict__ b,
                                                            const float* __restrict__ g, const float* __restrict__ beta,
                                                            float eps, __nv_bfloat16* __restrict__ X) {
    __shared__ float red[2][8];
    const int row = blockIdx.x, r = row / T, t = row - r * T;
    griddep_wait();
    griddep_launch();
    const float* base = H + ((size_t)slots[r] * seq_rows + t) * C;  // tap j reads row t + j
    float acc[4];
    float s1 = 0.f;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        const int c = threadIdx.x + e * 256;
        acc[e] = 0.f;
        if (c < C) {
            float a = b[c];
#pragma unroll
            for (int j = 0; j < 7; ++j) a += w[c * 7 + j] * base[(size_t)j * C + c];
            acc[e] = a;
            s1 += a;
        }
    }
    s1 = warp_sum(s1);
    if ((threadIdx.x & 31) == 0) red[0][threadIdx.x >> 5] = s1;
    __syncthreads();
    float mean = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) mean += red[0][i];
    mean /= (float)C;
    float s2 = 0.f;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        const int c = threadIdx.x + e * 256;
        if (c < C) s2 += (acc[e] - mean) * (acc[e] - mean);
    }
    s2 = warp_sum(s2);
    if ((threadIdx.x & 31) == 0) red[1][threadIdx.x >> 5] = s2;
    __syncthreads();
    float var = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) var += red[1][i];
    const float rstd = rsqrtf(var / (float)C + eps);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        const int c = threadIdx.x + e * 256;
        if (c < C) X[(size_t)row * C + c] = __float2bfloat16((acc[e] - mean) * rstd * g[c] + beta[c]);
    }
}

// ---------------------------------------------------------------------------
// last conv (k7, C -> 1) + clamp (code2wav_streaming.py:792-799).  A chunk of
// 512 outputs and its 6 context rows are staged channel-major in shared memory.
// ---------------------------------------------------------------------------
constexpr int kFinalThreads = 128;
constexpr int kFinalPer = 4;                             // consecutive outputs per thread
constexpr int kFinalChunk = kFinalThreads * kFinalPer;  // outputs per CTA
constexpr int kFinalRows = kFinalChunk + 8;             // staged rows (chunk + 6 context, even stride)
constexpr int kFinalMaxC = 128;

inline size_t final_conv_smem(int C) { return (size_t)C * kFinalRows * 2 + (size_t)7 * C * 4; }

// Staged channel-major, s[c][q]: thread t reads rows 4t .. 4t+9 of a channel as five bf16 pairs
// and accumulates its four outputs from them (28 multiply-adds per 5 loads).
__global__ void __launch_bounds__(kFinalThreads) c2w_final_conv_kernel(const __nv_bfloat16* __restrict__ H,
                                                                       int seq_rows, int C, int T,
                                                                       const int32_t* __restrict__ slots,
                                                                       const float* __restrict__ w, float bias,
                                                                       float* __restrict__ wav) {
    extern __shared__ __align__(16) uint8_t fsm[];
    __nv_bfloat16* s = reinterpret_cast<__nv_bfloat16*>(fsm);  // [C][kFinalRows]
    float* ws = reinterpret_cast<float*>(fsm + (size_t)C * kFinalRows * 2);
    const int r = blockIdx.y, t0 = blockIdx.x * kFinalChunk;
    griddep_wait();
    griddep_launch();
    const __nv_bfloat16* base = H + ((size_t)slots[r] * seq_rows + t0) * C;
    const int rows = min(kFinalChunk + 6, T + 6 - t0);
    const int c8n = C / 8;
    for (int i = threadIdx.x; i < rows * c8n; i += kFinalThreads) {
        const int c8 = i / rows, q = i - c8 * rows;  // consecutive threads: consecutive rows
        const uint4 u = *reinterpret_cast<const uint4*>(base + (size_t)q * C + c8 * 8);
        const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(&u);
#pragma unroll
        for (int k = 0; k < 8; ++k) s[(size_t)(c8 * 8 + k) * kFinalRows + q] = h[k];
    }
    for (int i = threadIdx.x; i < 7 * C; i += kFinalThreads) ws[i] = w[i];
    __syncthreads();
    const int tl = threadIdx.x * kFinalPer;  // first output of this thread within the chunk
    if (t0 + tl >= T) return;
    float acc[kFinalPer];
#pragma unroll
    for (int k = 0; k < kFinalPer; ++k) acc[k] = bias;
    for (int c = 0; c < C; ++c) {
        const __nv_bfloat162* row = reinterpret_cast<const __nv_bfloat162*>(s + (size_t)c * kFinalRows + tl);
        float x[kFinalPer + 6];
#pragma unroll
        for (int i = 0; i < (kFinalPer + 6) / 2; ++i) {
            const float2 f = __bfloat1622float2(row[i]);
            x[2 * i] = f.x;
            x[2 * i + 1] = f.y;
        }
#pragma unroll
        for (int j = 0; j < 7; ++j) {
            const float wj = ws[j * C + c];
#pragma unroll
            for (int k = 0; k < kFinalPer; ++k) acc[k] += wj * x[k + j];
        }
    }
    float* out = wav + (size_t)r * T + t0 + tl;  // T % 4 == 0: all four outputs exist
    float4 o;
    o.x = fminf(fmaxf(acc[0], -1.0f), 1.0f);
    o.y = fminf(fmaxf(acc[1], -1.0f), 1.0f);
    o.z = fminf(fmaxf(acc[2], -1.0f), 1.0f);
    o.w = fminf(fmaxf(acc[3], -1.0f), 1.0f);
    if ((reinterpret_cast<uintptr_t>(out) & 15) == 0) {
        *reinterpret_cast<float4*>(out) = o;
    } else {  // caller buffer not 16-byte aligned
        out[0] = o.x;
        out[1] = o.y;
        out[2] = o.z;
        out[3] = o.w;
    }
}

// ---------------------------------------------------------------------------
// state roll / reset over the history buffers
// ---------------------------------------------------------------------------
struct RollJob {
    uint8_t* ptr;
    int seq_rows, ctx, T, row_bytes;  // T: rows per frame (a call of F frames uses F * T)
};
constexpr int kMaxRollJobs = 24;
constexpr int kRollChunk = 512;  // bytes of a row per CTA
constexpr int kRollChunks = 8;   // grid.z: rows up to 4 KB
constexpr int kRollMaxCtx = 54;

struct RollTable {
    RollJob job[kMaxRollJobs];
    int n;
};

// rows [T, T + ctx) -> [0, ctx) of each active slot (T = F * rows per frame); the
// CTA stages its column chunk of all ctx rows before writing, so T < ctx
// (overlapping ranges) is safe.  Also advances each slot's frame counter by F.
__global__ void __launch_bounds__(128) c2w_roll_kernel(const __grid_constant__ RollTable tab,
                                                       const int32_t* __restrict__ slots, int F,
                                                       int32_t* __restrict__ frame) {
    __shared__ uint4 buf[kRollMaxCtx * (kRollChunk / 16)];
    griddep_wait();
    griddep_launch();
    if (blockIdx.y == 0 && blockIdx.z == 0 && threadIdx.x == 0) frame[slots[blockIdx.x]] += F;
    if ((int)blockIdx.y >= tab.n) return;
    const RollJob& j = tab.job[blockIdx.y];
    const int T = j.T * F;
    const int off = blockIdx.z * kRollChunk;
    if (off >= j.row_bytes || j.ctx <= 0 || j.ctx > kRollMaxCtx) return;
    const int vec = min(kRollChunk, j.row_bytes - off) / 16;
    uint8_t* seg = j.ptr + (size_t)slots[blockIdx.x] * j.seq_rows * j.row_bytes + off;
    for (int i = threadIdx.x; i < j.ctx * vec; i += blockDim.x) {
        const int q = i / vec, e = i - q * vec;
        buf[q * (kRollChunk / 16) + e] = *reinterpret_cast<const uint4*>(seg + (size_t)(T + q) * j.row_bytes + e * 16);
    }
    __syncthreads();
    for (int i = threadIdx.x; i < j.ctx * vec; i += blockDim.x) {
        const int q = i / vec, e = i - q * vec;
        *reinterpret_cast<uint4*>(seg + (size_t)q * j.row_bytes + e * 16) = buf[q * (kRollChunk / 16) + e];
    }
}

__global__ void __launch_bounds__(128) c2w_reset_kernel(const __grid_constant__ RollTable tab,
                                                        const int32_t* __restrict__ slots, int max_slots,
                                                        int32_t* __restrict__ frame) {
    griddep_wait();
    griddep_launch();
    const int slot = slots[blockIdx.x];
    if (slot < 0 || slot >= max_slots) {
        if (blockIdx.y == 0 && threadIdx.x == 0) record_error(DEV_ERR_BAD_SLOT);
        return;
    }
    if (blockIdx.y == 0 && threadIdx.x == 0) frame[slot] = 0;
    if ((int)blockIdx.y >= tab.n) return;
    const RollJob& j = tab.job[blockIdx.y];
    uint8_t* seg = j.ptr + (size_t)slot * j.seq_rows * j.row_bytes;
    const int vec = j.row_bytes / 16;
    for (int i = threadIdx.x; i < j.ctx * vec; i += blockDim.x)
        reinterpret_cast<uint4*>(seg)[i] = make_uint4(0, 0, 0, 0);
}

}  // namespace qtts

// ---------------------------------------------------------------------------
// the decoder object: buffers, GEMM plans and the launch sequence
// ---------------------------------------------------------------------------
struct qtts_c2w {
    qtts_c2w_desc d;
    bool background = false;   // launches without programmatic dependent launch (qtts_c2w_set_background)
    int S;                     // max streams per step (= max slots)
    int Fm;                    // max frames per stream per call (chunk)
    int T_up[2], T_in[4], T_blk[4], cin[4], cout[4];  // rows per stream per FRAME
    int K_pc, K_c0, K_tc[4], K_c1[4], N_c[4], N_tc[4];
    // implicit convolution (the GEMM reads the history buffer directly, no im2col) where the
    // rows per stream are a multiple of 128; those history buffers pad channels to 64
    bool impl_tc[4], impl_c1[4];
    int cinpad[4], cpad[4];
    int32_t *frame = nullptr, *row_slot = nullptr, *row_pos = nullptr, *row_kv = nullptr, *row_nkeys = nullptr,
            *row_lo = nullptr;
    qtts::kv_t* ring = nullptr;
    __nv_bfloat16 *H_pc = nullptr, *Xa = nullptr, *Xb = nullptr;
    float *x = nullptr, *qbuf = nullptr;
    __nv_bfloat16 *xn = nullptr, *xn_lo = nullptr, *attn = nullptr, *attn_lo = nullptr, *act = nullptr,
                  *act_lo = nullptr;
    __nv_bfloat16 *U0 = nullptr, *U1 = nullptr, *Xln = nullptr, *Xg = nullptr, *H_c0 = nullptr, *H_fin = nullptr;
    float* H_dw[2] = {nullptr, nullptr};
    __nv_bfloat16* H_tc[4] = {};
    float* h[4] = {};
    __nv_bfloat16* H_res[4][3] = {};
    __nv_bfloat16* X2[4] = {};
    qtts::RollTable roll;
    std::vector<void*> allocs;
    std::vector<std::pair<const void*, size_t>> alloc_bytes;  // usable bytes of each allocation
    qtts::GemmPlan pre_conv, in_proj, out_proj, conv0;
    std::vector<qtts::LayerGemms> layer;
    qtts::GemmPlan up_t[2], pw1[2], pw2[2], blk_t[4], c1[4][3], c2[4][3];
    int launches = 0;
};

namespace qtts {

template <class T>
inline int c2w_alloc(qtts_c2w* c, T** p, size_t count) {
    void* ptr = nullptr;
    QTTS_CHECK_CUDA(cudaMalloc(&ptr, count * sizeof(T) + 256));
    QTTS_CHECK_CUDA(cudaMemset(ptr, 0, count * sizeof(T) + 256));
    c->allocs.push_back(ptr);
    c->alloc_bytes.emplace_back(ptr, count * sizeof(T));
    *p = reinterpret_cast<T*>(ptr);
    return QTTS_OK;
}

// bytes of the decoder allocation `p` starts (0 when p is not one of them: not checked)
inline unsigned long long c2w_bytes(const qtts_c2w* c, const void* p) {
    for (const auto& a : c->alloc_bytes)
        if (a.first == p) return a.second;
    return 0;
}

inline ActView view_slot(const qtts_c2w* c, void* p, int ctx, int T, int ld) {
    return ActView{p, 1, ctx + T, ctx, ld, c2w_bytes(c, p)};
}
inline ActView view_rows(const qtts_c2w* c, void* p, int T, int ld) {
    return ActView{p, 0, T, 0, ld, c2w_bytes(c, p)};
}

// Whether a convolution whose input has T rows per frame reads its operand straight from the
// history buffer (implicit convolution).  A GEMM row tile must not span two streams, so a
// stream's rows are padded to a multiple of 128: used when no padding is needed, or when the
// largest call (max_chunk frames) has at least 512 rows and pads them by at most 1/8.
inline bool c2w_implicit_rows(int T, int max_chunk) {
    if (T % 128 == 0) return true;
    const int R = max_chunk * T, pad = (R + 127) / 128 * 128 - R;
    return R >= 512 && pad * 8 <= R;
}

inline ConvEpi conv_epi(const qtts_c2w* c, int T_rows, int phases, int C_o, int n_valid) {
    ConvEpi e;
    memset(&e, 0, sizeof(e));
    e.T_rows = T_rows;
    e.phases = phases;
    e.C_o = C_o;
    e.n_valid = n_valid;
    e.act = ACT_NONE;
    (void)c;
    return e;
}

inline int conv_plan(GemmPlan* g, const void* X, int rows, int K, const void* W, int N, const void* bias,
                     const ConvEpi& e, const void* X_lo = nullptr) {
    int rc = gemm_plan(g, X, rows, K, W, N, kEpiConv, nullptr, bias, nullptr, X_lo);
    if (rc) return rc;
    g->p.conv = e;
    return QTTS_OK;
}

// history buffer segment: ctx rows + Fm frames of T rows; a call of F frames rolls rows [F*T, F*T + ctx)
inline void add_roll(qtts_c2w* c, void* p, int ctx, int T, int Fm, int row_bytes) {
    RollJob& j = c->roll.job[c->roll.n++];
    j.ptr = reinterpret_cast<uint8_t*>(p);
    j.seq_rows = ctx + Fm * T;
    j.ctx = ctx;
    j.T = T;
    j.row_bytes = row_bytes;
}

inline int c2w_build(qtts_c2w* c) {
    const qtts_c2w_desc& d = c->d;
    const int S = d.max_slots, LAT = d.latent, HID = d.hidden, NH = d.heads, HD = d.head_dim, I = d.inter;
    const int L = d.layers, W = d.window, CD = d.codebook_dim, CN = d.convnext_dim, D0 = d.decoder_dim;
    if (S <= 0 || L <= 0 || (HD != 32 && HD != 64) || W < 1 || W > 96 || d.max_frames < 1 ||
        d.num_codebooks > 32 || d.num_codebooks < 1 || CD % 8 != 0 || LAT % 128 != 0 || HID % 128 != 0 ||
        (3 * NH * HD) % 128 != 0 || I % 64 != 0 || CN % 128 != 0 || LAT > 1024 || NH * HD != HID) {
        set_error("c2w: unsupported configuration");
        return QTTS_ERR_UNSUPPORTED;
    }
    if (d.up_ratio[0] != 2 || d.up_ratio[1] != 2) {
        set_error("c2w: upsampling ratios must be (2, 2)");
        return QTTS_ERR_UNSUPPORTED;
    }
    for (int j = 0; j < 3; ++j)
        if (d.dilations[j] < 1 || 6 * d.dilations[j] > kRollMaxCtx) {
            set_error("c2w: dilation %d outside [1, %d]", d.dilations[j], kRollMaxCtx / 6);
            return QTTS_ERR_UNSUPPORTED;
        }
    const int Fm = d.max_chunk > 0 ? d.max_chunk : 1;
    if (Fm > W) {
        set_error("c2w: max_chunk %d above the window %d", Fm, W);
        return QTTS_ERR_UNSUPPORTED;
    }
    c->S = S;
    c->Fm = Fm;
    const int S1 = S + 1;  // slot-indexed state has a spare slot for rejected slot ids
    const int SF = S * Fm;  // rows of a call at one row per frame
    c->T_up[0] = 2;
    c->T_up[1] = 4;
    int T = 4;
    for (int b = 0; b < 4; ++b) {
        c->T_in[b] = T;
        c->cin[b] = D0 >> b;
        c->cout[b] = D0 >> (b + 1);
        T *= d.rates[b];
        c->T_blk[b] = T;
        if (c->cout[b] % 8 != 0 || d.rates[b] < 1) {
            set_error("c2w: decoder channels must stay multiples of 8");
            return QTTS_ERR_UNSUPPORTED;
        }
        c->impl_tc[b] = c2w_implicit_rows(c->T_in[b], Fm);
        c->impl_c1[b] = c2w_implicit_rows(c->T_blk[b], Fm);
        c->cinpad[b] = c->impl_tc[b] ? pad64(c->cin[b]) : c->cin[b];
        c->cpad[b] = c->impl_c1[b] ? pad64(c->cout[b]) : c->cout[b];
        c->K_tc[b] = c->impl_tc[b] ? 2 * c->cinpad[b] : pad64(2 * c->cin[b]);
        c->N_tc[b] = pad128(d.rates[b] * c->cout[b]);
        c->K_c1[b] = c->impl_c1[b] ? 7 * c->cpad[b] : pad64(7 * c->cout[b]);
        c->N_c[b] = pad128(c->cout[b]);
    }
    if (c->cout[3] > kFinalMaxC || (c->T_blk[3] % 4) != 0) {
        set_error("c2w: last decoder width above %d or samples per frame not a multiple of 4", kFinalMaxC);
        return QTTS_ERR_UNSUPPORTED;
    }
    QTTS_CHECK_CUDA(cudaFuncSetAttribute(c2w_final_conv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)final_conv_smem(kFinalMaxC)));
    c->K_pc = pad64(3 * CD);
    c->K_c0 = pad64(7 * LAT);

    QTTS_TRY(c2w_alloc(c, &c->frame, S1));
    QTTS_TRY(c2w_alloc(c, &c->row_slot, S));
    QTTS_TRY(c2w_alloc(c, &c->row_pos, SF));
    QTTS_TRY(c2w_alloc(c, &c->row_kv, SF));
    QTTS_TRY(c2w_alloc(c, &c->row_nkeys, SF));
    QTTS_TRY(c2w_alloc(c, &c->row_lo, SF));
    QTTS_TRY(c2w_alloc(c, &c->ring, (size_t)S1 * L * 2 * NH * W * HD));
    QTTS_TRY(c2w_alloc(c, &c->H_pc, (size_t)S1 * (2 + Fm) * CD));
    size_t xa = (size_t)SF * c->K_pc;
    xa = std::max(xa, (size_t)SF * 4 * c->K_c0);
    for (int b = 0; b < 4; ++b) {
        if (!c->impl_tc[b]) xa = std::max(xa, (size_t)SF * c->T_in[b] * c->K_tc[b]);
        if (!c->impl_c1[b]) xa = std::max(xa, (size_t)SF * c->T_blk[b] * c->K_c1[b]);
    }
    QTTS_TRY(c2w_alloc(c, &c->Xa, xa));
    QTTS_TRY(c2w_alloc(c, &c->Xb, (size_t)SF * LAT));
    QTTS_TRY(c2w_alloc(c, &c->x, (size_t)SF * HID));
    QTTS_TRY(c2w_alloc(c, &c->xn, (size_t)SF * HID));
    QTTS_TRY(c2w_alloc(c, &c->xn_lo, (size_t)SF * HID));
    QTTS_TRY(c2w_alloc(c, &c->qbuf, (size_t)SF * NH * HD));
    QTTS_TRY(c2w_alloc(c, &c->attn, (size_t)SF * NH * HD));
    QTTS_TRY(c2w_alloc(c, &c->attn_lo, (size_t)SF * NH * HD));
    QTTS_TRY(c2w_alloc(c, &c->act, (size_t)SF * I));
    QTTS_TRY(c2w_alloc(c, &c->act_lo, (size_t)SF * I));
    QTTS_TRY(c2w_alloc(c, &c->U0, (size_t)SF * LAT));
    QTTS_TRY(c2w_alloc(c, &c->U1, (size_t)SF * 2 * LAT));
    QTTS_TRY(c2w_alloc(c, &c->Xln, (size_t)SF * 4 * LAT));
    QTTS_TRY(c2w_alloc(c, &c->Xg, (size_t)SF * 4 * CN));
    for (int i = 0; i < 2; ++i) QTTS_TRY(c2w_alloc(c, &c->H_dw[i], (size_t)S1 * (6 + Fm * c->T_up[i]) * LAT));
    QTTS_TRY(c2w_alloc(c, &c->H_c0, (size_t)S1 * (6 + Fm * 4) * LAT));
    for (int b = 0; b < 4; ++b) {
        const int Tb = c->T_blk[b], co = c->cout[b];
        QTTS_TRY(c2w_alloc(c, &c->H_tc[b], (size_t)S1 * (1 + Fm * c->T_in[b]) * c->cinpad[b]));
        QTTS_TRY(c2w_alloc(c, &c->h[b], (size_t)SF * Tb * co));
        for (int j = 0; j < 3; ++j)
            QTTS_TRY(c2w_alloc(c, &c->H_res[b][j], (size_t)S1 * (6 * d.dilations[j] + Fm * Tb) * c->cpad[b]));
        QTTS_TRY(c2w_alloc(c, &c->X2[b], (size_t)SF * Tb * c->N_c[b]));
    }
    QTTS_TRY(c2w_alloc(c, &c->H_fin, (size_t)S1 * (6 + Fm * c->T_blk[3]) * c->cout[3]));

    // the 21 streaming states, in the reference's order (conv 0..16, transconv 0..3);
    // segments hold ctx + Fm * (rows per frame) rows
    c->roll.n = 0;
    add_roll(c, c->H_pc, 2, 1, Fm, CD * 2);
    add_roll(c, c->H_dw[0], 6, c->T_up[0], Fm, LAT * 4);
    add_roll(c, c->H_dw[1], 6, c->T_up[1], Fm, LAT * 4);
    add_roll(c, c->H_c0, 6, 4, Fm, LAT * 2);
    for (int b = 0; b < 4; ++b)
        for (int j = 0; j < 3; ++j)
            add_roll(c, c->H_res[b][j], 6 * d.dilations[j], c->T_blk[b], Fm, c->cpad[b] * 2);
    add_roll(c, c->H_fin, 6, c->T_blk[3], Fm, c->cout[3] * 2);
    for (int b = 0; b < 4; ++b) add_roll(c, c->H_tc[b], 1, c->T_in[b], Fm, c->cinpad[b] * 2);
    for (int i = 0; i < c->roll.n; ++i)
        if (c->roll.job[i].row_bytes % 16 != 0 || c->roll.job[i].row_bytes > kRollChunks * kRollChunk) {
            set_error("c2w: state rows must be multiples of 16 bytes, at most %d", kRollChunks * kRollChunk);
            return QTTS_ERR_UNSUPPORTED;
        }

    // ---- front + transformer (one row per frame; plans sized for Fm frames per stream)
    QTTS_TRY(gemm_plan(&c->pre_conv, c->Xa, SF, c->K_pc, d.w_pre_conv, LAT, QTTS_EPI_BF16, c->Xb, d.b_pre_conv,
                       nullptr));
    QTTS_TRY(gemm_plan(&c->in_proj, c->Xb, SF, LAT, d.w_in_proj, HID, QTTS_EPI_F32, c->x, d.b_in_proj, nullptr));
    c->layer.resize(L);
    for (int l = 0; l < L; ++l) {
        LayerGemms& g = c->layer[l];
        qtts_qkv_epilogue q = {};
        q.num_heads = NH;
        q.kv_heads = NH;
        q.head_dim = HD;
        q.q_norm_w = bf(d.w_q_norm, (size_t)l * HD);
        q.k_norm_w = bf(d.w_k_norm, (size_t)l * HD);
        q.rms_eps = d.rms_eps;
        q.rope_cos = d.rope_cos;
        q.rope_sin = d.rope_sin;
        q.max_pos = d.max_frames;
        q.row_pos = c->row_pos;
        q.slot_mapping = c->row_kv;  // slot * window + frame % window
        q.kv_pool = c->ring;         // "blocks" of `window` positions, one per slot
        q.layer = l;
        q.num_layers = L;
        q.block_size = W;
        QTTS_TRY(gemm_plan(&g.qkv, c->xn, SF, HID, bf(d.w_qkv, (size_t)l * 3 * HID * HID), 3 * HID,
                           QTTS_EPI_QKV_ROPE, c->qbuf, nullptr, &q, c->xn_lo));
        ConvEpi eo = conv_epi(c, 1, 1, HID, HID);
        eo.scale = bf(d.attn_scale, (size_t)l * HID);
        eo.res = view_rows(c, c->x, 1, HID);
        eo.out32 = eo.res;
        QTTS_TRY(conv_plan(&g.o, c->attn, SF, HID, bf(d.w_o, (size_t)l * HID * HID), HID, nullptr, eo, c->attn_lo));
        QTTS_TRY(gemm_plan(&g.gu, c->xn, SF, HID, bf(d.w_gate_up, (size_t)l * 2 * I * HID), 2 * I, QTTS_EPI_SWIGLU,
                           c->act, nullptr, nullptr, c->xn_lo, c->act_lo));
        ConvEpi ed = eo;
        ed.scale = bf(d.mlp_scale, (size_t)l * HID);
        QTTS_TRY(conv_plan(&g.down, c->act, SF, I, bf(d.w_down, (size_t)l * HID * I), HID, nullptr, ed, c->act_lo));
    }
    QTTS_TRY(gemm_plan(&c->out_proj, c->xn, SF, HID, d.w_out_proj, LAT, QTTS_EPI_BF16, c->U0, d.b_out_proj, nullptr,
                       c->xn_lo));
    // ---- upsampling: transposed conv (k = s = 2) + ConvNeXt
    for (int i = 0; i < 2; ++i) {
        const int Tin = i == 0 ? 1 : 2, To = c->T_up[i];
        ConvEpi et = conv_epi(c, Tin, 2, LAT, 2 * LAT);
        et.out32 = view_slot(c, c->H_dw[i], 6, Fm * To, LAT);
        QTTS_TRY(conv_plan(&c->up_t[i], i == 0 ? c->U0 : c->U1, SF * Tin, LAT, d.up_w[i], 2 * LAT, d.up_b[i], et));
        ConvEpi e1 = conv_epi(c, 1, 1, CN, CN);
        e1.act = ACT_GELU;
        e1.out16 = view_rows(c, c->Xg, 1, CN);
        QTTS_TRY(conv_plan(&c->pw1[i], c->Xln, SF * To, LAT, d.pw1_w[i], CN, d.pw1_b[i], e1));
        ConvEpi e2 = conv_epi(c, To, 1, LAT, LAT);
        e2.scale = reinterpret_cast<const __nv_bfloat16*>(d.gamma[i]);
        e2.res = view_slot(c, c->H_dw[i], 6, Fm * To, LAT);
        e2.out16 = i == 0 ? view_rows(c, c->U1, 2, LAT) : view_slot(c, c->H_c0, 6, Fm * 4, LAT);
        QTTS_TRY(conv_plan(&c->pw2[i], c->Xg, SF * To, CN, d.pw2_w[i], LAT, d.pw2_b[i], e2));
    }
    // ---- decoder conv k7 (latent -> decoder_dim), then SnakeBeta of block 0 into its transconv input
    {
        ConvEpi e = conv_epi(c, 4, 1, D0, D0);
        e.act = ACT_SNAKE;
        e.act_p = d.blk_snake[0];
        e.out16 = view_slot(c, c->H_tc[0], 1, Fm * 4, c->cinpad[0]);
        QTTS_TRY(conv_plan(&c->conv0, c->Xa, SF * 4, c->K_c0, d.w_conv0, pad128(D0), d.b_conv0, e));
    }
    for (int b = 0; b < 4; ++b) {
        const int Tb = c->T_blk[b], co = c->cout[b], s = d.rates[b];
        ConvEpi et = conv_epi(c, c->T_in[b], s, co, s * co);
        et.out32 = view_rows(c, c->h[b], Tb, co);
        et.act = ACT_SNAKE;
        et.act_p = d.res_act1[b][0];
        et.out16 = view_slot(c, c->H_res[b][0], 6 * d.dilations[0], Fm * Tb, c->cpad[b]);
        if (c->impl_tc[b])
            QTTS_TRY(gemm_plan_implicit(&c->blk_t[b], c->H_tc[b], S1 * (1 + Fm * c->T_in[b]), c->cinpad[b], 2, 1,
                                        c->T_in[b], 1 + Fm * c->T_in[b], SF * c->T_in[b], d.blk_tw[b], c->N_tc[b],
                                        d.blk_tb[b], et));
        else
            QTTS_TRY(conv_plan(&c->blk_t[b], c->Xa, SF * c->T_in[b], c->K_tc[b], d.blk_tw[b], c->N_tc[b],
                               d.blk_tb[b], et));
        for (int j = 0; j < 3; ++j) {
            ConvEpi e1 = conv_epi(c, Tb, 1, co, co);
            e1.act = ACT_SNAKE;
            e1.act_p = d.res_act2[b][j];
            e1.out16 = view_rows(c, c->X2[b], Tb, c->N_c[b]);
            const int dil = d.dilations[j];
            if (c->impl_c1[b])
                QTTS_TRY(gemm_plan_implicit(&c->c1[b][j], c->H_res[b][j], S1 * (6 * dil + Fm * Tb), c->cpad[b], 7,
                                            dil, Tb, 6 * dil + Fm * Tb, SF * Tb, d.res_w1[b][j], c->N_c[b],
                                            d.res_b1[b][j], e1));
            else
                QTTS_TRY(conv_plan(&c->c1[b][j], c->Xa, SF * Tb, c->K_c1[b], d.res_w1[b][j], c->N_c[b],
                                   d.res_b1[b][j], e1));
            ConvEpi e2 = conv_epi(c, Tb, 1, co, co);
            e2.res = view_rows(c, c->h[b], Tb, co);
            e2.out32 = e2.res;
            e2.act = ACT_SNAKE;
            if (j < 2) {
                e2.act_p = d.res_act1[b][j + 1];
                e2.out16 = view_slot(c, c->H_res[b][j + 1], 6 * d.dilations[j + 1], Fm * Tb, c->cpad[b]);
            } else if (b < 3) {
                e2.act_p = d.blk_snake[b + 1];
                e2.out16 = view_slot(c, c->H_tc[b + 1], 1, Fm * Tb, c->cinpad[b + 1]);
            } else {
                e2.act_p = d.final_snake;
                e2.out16 = view_slot(c, c->H_fin, 6, Fm * Tb, co);
            }
            QTTS_TRY(conv_plan(&c->c2[b][j], c->X2[b], SF * Tb, c->N_c[b], d.res_w2[b][j], c->N_c[b],
                               d.res_b2[b][j], e2));
        }
    }
    return QTTS_OK;
}

inline int c2w_im2col(const qtts_c2w* c, const __nv_bfloat16* H, int ctx, int seq_rows, int T, int C, int taps,
                      int dil, int K, const int32_t* slots, int n, cudaStream_t st) {
    const size_t total = (size_t)n * T * (K / 8);
    const int blocks = (int)std::min<size_t>((total + 255) / 256, (size_t)num_sms() * 8);
    QTTS_LAUNCH(c2w_im2col_kernel, dim3(blocks), dim3(256), 0, st, H, seq_rows, C, taps, dil, T, slots, n, c->Xa, K);
    return QTTS_OK;
}

// A plan built for one frame's rows per stream, run on F frames: rows per stream and the
// stride of the per-call (not slot-indexed) buffers scale by F; history buffers keep their
// segment size (ctx + Fm * rows per frame).
// An implicit convolution pads each stream's rows to whole 128-row tiles (the epilogue skips the
// padding rows).
inline int run_conv(GemmPlan g, int M, const int32_t* slots, cudaStream_t st, int F) {
    const int T = g.p.conv.T_rows * F;  // rows per stream of this call
    g.p.conv.row_slot = slots;
    g.p.conv.T_rows = T;
    for (ActView* v : {&g.p.conv.res, &g.p.conv.out32, &g.p.conv.out16})
        if (!v->by_slot) v->seq_rows *= F;
    g.p.ix.row_slot = slots;  // implicit convolutions read the history rows of each row's slot
    if (g.p.ix.on) {
        const int Tpad = (T + 127) / 128 * 128;
        g.p.ix.T = Tpad;
        g.p.conv.T_rows = Tpad;
        g.p.conv.T_valid = T;
        M = M / T * Tpad;
    }
    return gemm_run(g, M, st);
}

inline int c2w_step_impl(qtts_c2w* c, const int64_t* codes, int codes_ld, int F, const int32_t* slots_in, int n,
                         float* wav, cudaStream_t st) {
    const qtts_c2w_desc& d = c->d;
    if (n <= 0 || n > c->S || !codes || !slots_in || !wav || codes_ld < d.num_codebooks) {
        set_error("c2w_step: n=%d outside (0, %d] or missing pointers", n, c->S);
        return QTTS_ERR_INVALID;
    }
    if (F < 1 || F > c->Fm) {
        set_error("c2w_step: %d frames outside [1, %d] (max_chunk)", F, c->Fm);
        return QTTS_ERR_INVALID;
    }
    const int Fm = c->Fm, nF = n * F;
    const int LAT = d.latent, HID = d.hidden, NH = d.heads, HD = d.head_dim, CD = d.codebook_dim, L = d.layers;
    QTTS_LAUNCH(c2w_rvq_kernel, dim3(nF), dim3(256), 0, st, d.rvq_tables, d.num_codebooks, d.codebook_size, CD, codes,
                codes_ld, F, slots_in, c->S, (const int32_t*)c->frame, d.window, d.max_frames, c->row_slot,
                c->row_pos, c->row_kv, c->row_nkeys, c->row_lo, view_slot(c, c->H_pc, 2, Fm, CD));
    const int32_t* slots = c->row_slot;  // validated slot of each stream
    QTTS_TRY(c2w_im2col(c, c->H_pc, 2, 2 + Fm, F, CD, 3, 1, c->K_pc, slots, n, st));
    QTTS_TRY(gemm_run(c->pre_conv, nF, st));
    QTTS_TRY(gemm_run(c->in_proj, nF, st));
    for (int l = 0; l < L; ++l) {
        const LayerGemms& g = c->layer[l];
        QTTS_TRY(launch_rmsnorm(c->x, nF, HID, HID, bf(d.w_in_norm, (size_t)l * HID), d.rms_eps, c->xn, st,
                                c->xn_lo));
        QTTS_TRY(gemm_run(g.qkv, nF, st));
        const float scale = 1.0f / sqrtf((float)HD);
        if (HD == 64)
            QTTS_LAUNCH(c2w_attn_kernel<64>, dim3(nF, ceil_div(NH, 4)), dim3(128), 0, st, (const float*)c->qbuf,
                        (const kv_t*)c->ring, NH, L, l, d.window, F, slots, (const int32_t*)c->row_nkeys,
                        (const int32_t*)c->row_lo, scale, c->attn, c->attn_lo);
        else
            QTTS_LAUNCH(c2w_attn_kernel<32>, dim3(nF, ceil_div(NH, 4)), dim3(128), 0, st, (const float*)c->qbuf,
                        (const kv_t*)c->ring, NH, L, l, d.window, F, slots, (const int32_t*)c->row_nkeys,
                        (const int32_t*)c->row_lo, scale, c->attn, c->attn_lo);
        QTTS_TRY(run_conv(g.o, nF, slots, st, F));
        QTTS_TRY(launch_rmsnorm(c->x, nF, HID, HID, bf(d.w_post_norm, (size_t)l * HID), d.rms_eps, c->xn, st,
                                c->xn_lo));
        QTTS_TRY(gemm_run(g.gu, nF, st));
        QTTS_TRY(run_conv(g.down, nF, slots, st, F));
    }
    QTTS_TRY(launch_rmsnorm(c->x, nF, HID, HID, d.w_final_norm, d.rms_eps, c->xn, st, c->xn_lo));
    QTTS_TRY(gemm_run(c->out_proj, nF, st));
    for (int i = 0; i < 2; ++i) {
        const int Tin = i == 0 ? 1 : 2, To = c->T_up[i];
        QTTS_TRY(run_conv(c->up_t[i], nF * Tin, slots, st, F));
        QTTS_LAUNCH(c2w_dwconv_ln_kernel, dim3(nF * To), dim3(256), 0, st, (const float*)c->H_dw[i], 6 + Fm * To,
                    LAT, F * To, slots, d.dw_w[i], d.dw_b[i], d.ln_w[i], d.ln_b[i], d.ln_eps, c->Xln);
        QTTS_TRY(run_conv(c->pw1[i], nF * To, slots, st, F));
        QTTS_TRY(run_conv(c->pw2[i], nF * To, slots, st, F));
    }
    QTTS_TRY(c2w_im2col(c, c->H_c0, 6, 6 + Fm * 4, F * 4, LAT, 7, 1, c->K_c0, slots, n, st));
    QTTS_TRY(run_conv(c->conv0, nF * 4, slots, st, F));
    for (int b = 0; b < 4; ++b) {
        const int Tb = c->T_blk[b], co = c->cout[b];
        if (!c->impl_tc[b])
            QTTS_TRY(c2w_im2col(c, c->H_tc[b], 1, 1 + Fm * c->T_in[b], F * c->T_in[b], c->cin[b], 2, 1, c->K_tc[b],
                                slots, n, st));
        QTTS_TRY(run_conv(c->blk_t[b], nF * c->T_in[b], slots, st, F));
        for (int j = 0; j < 3; ++j) {
            const int dil = d.dilations[j];
            if (!c->impl_c1[b])
                QTTS_TRY(c2w_im2col(c, c->H_res[b][j], 6 * dil, 6 * dil + Fm * Tb, F * Tb, co, 7, dil, c->K_c1[b],
                                    slots, n, st));
            QTTS_TRY(run_conv(c->c1[b][j], nF * Tb, slots, st, F));
            QTTS_TRY(run_conv(c->c2[b][j], nF * Tb, slots, st, F));
        }
    }
    const int T3 = F * c->T_blk[3];
    QTTS_LAUNCH(c2w_final_conv_kernel, dim3(ceil_div(T3, kFinalChunk), n), dim3(kFinalThreads),
                final_conv_smem(c->cout[3]), st, (const __nv_bfloat16*)c->H_fin, 6 + Fm * c->T_blk[3], c->cout[3], T3,
                slots, d.final_w, d.final_b, wav);
    QTTS_LAUNCH(c2w_roll_kernel, dim3(n, c->roll.n, kRollChunks), dim3(128), 0, st, c->roll, slots, F, c->frame);
    return QTTS_OK;
}

inline int c2w_step(qtts_c2w* c, const int64_t* codes, int codes_ld, int F, const int32_t* slots, int n, float* wav,
                    cudaStream_t st) {
    const int before = g_launch_count;
    if (c->background) ++g_pdl_suppress;
    const int rc = c2w_step_impl(c, codes, codes_ld, F, slots, n, wav, st);
    if (c->background) --g_pdl_suppress;
    c->launches = g_launch_count - before;
    return rc;
}

inline int c2w_reset(qtts_c2w* c, const int32_t* slots, int n, cudaStream_t st) {
    if (n <= 0) return QTTS_OK;
    QTTS_LAUNCH(c2w_reset_kernel, dim3(n, c->roll.n), dim3(128), 0, st, c->roll, slots, c->S, c->frame);
    return QTTS_OK;
}

// ---------------------------------------------------------------------------
// warm state: the per-slot state in this decoder's layout (qtts_c2w_state_part)
// ---------------------------------------------------------------------------
constexpr int kC2wStateParts = 22;

// valid channels of roll job j (the reference's state order: conv 0..16, transconv 0..3)
inline int c2w_state_channels(const qtts_c2w* c, int j) {
    const qtts_c2w_desc& d = c->d;
    if (j == 0) return d.codebook_dim;
    if (j <= 3) return d.latent;
    if (j <= 15) return c->cout[(j - 4) / 3];
    if (j == 16) return c->cout[3];
    return c->cin[j - 17];
}

inline int c2w_state_layout(const qtts_c2w* c, qtts_c2w_state_part* parts, int max_parts) {
    if (!parts || max_parts < kC2wStateParts || c->roll.n != kC2wStateParts - 1) {
        set_error("c2w_state_layout: need room for %d parts", kC2wStateParts);
        return QTTS_ERR_INVALID;
    }
    const qtts_c2w_desc& d = c->d;
    parts[0].rows = d.layers * 2 * d.heads * d.window;
    parts[0].row_elems = d.head_dim;
    parts[0].valid_elems = d.head_dim;
    parts[0].dtype = 2;
    for (int j = 0; j < c->roll.n; ++j) {
        const RollJob& r = c->roll.job[j];
        const int esz = (j == 1 || j == 2) ? 4 : 2;  // the ConvNeXt inputs are kept in fp32
        parts[1 + j].rows = r.ctx;
        parts[1 + j].row_elems = r.row_bytes / esz;
        parts[1 + j].valid_elems = c2w_state_channels(c, j);
        parts[1 + j].dtype = esz == 4 ? 1 : 0;
    }
    return QTTS_OK;
}

__global__ void c2w_set_frame_kernel(int32_t* frame, int slot, int value) {
    griddep_wait();
    griddep_launch();
    if (threadIdx.x == 0) frame[slot] = value;
}

inline int c2w_write_state(qtts_c2w* c, int slot, int part, const void* src, size_t bytes, cudaStream_t st) {
    if (slot < 0 || slot >= c->S || part < 0 || part >= kC2wStateParts || !src) {
        set_error("c2w_write_state: slot %d / part %d outside [0, %d) / [0, %d)", slot, part, c->S, kC2wStateParts);
        return QTTS_ERR_INVALID;
    }
    const qtts_c2w_desc& d = c->d;
    void* dst;
    size_t want;
    if (part == 0) {
        want = (size_t)d.layers * 2 * d.heads * d.window * d.head_dim * sizeof(kv_t);
        dst = c->ring + (size_t)slot * d.layers * 2 * d.heads * d.window * d.head_dim;
    } else {
        const RollJob& r = c->roll.job[part - 1];
        want = (size_t)r.ctx * r.row_bytes;  // rows [0, ctx) of the slot's segment
        dst = r.ptr + (size_t)slot * r.seq_rows * r.row_bytes;
    }
    if (bytes != want) {
        set_error("c2w_write_state: part %d holds %zu bytes, got %zu", part, want, bytes);
        return QTTS_ERR_INVALID;
    }
    QTTS_CHECK_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToDevice, st));
    return QTTS_OK;
}

inline int c2w_set_frame(qtts_c2w* c, int slot, int frame, cudaStream_t st) {
    if (slot < 0 || slot >= c->S || frame < 0 || frame >= c->d.max_frames) {
        set_error("c2w_set_frame: slot %d / frame %d outside [0, %d) / [0, %d)", slot, frame, c->S,
                  c->d.max_frames);
        return QTTS_ERR_INVALID;
    }
    QTTS_LAUNCH(c2w_set_frame_kernel, dim3(1), dim3(32), 0, st, c->frame, slot, frame);
    return QTTS_OK;
}

}  // namespace qtts
