// Shared device helpers for the sm_100a kernels: status handling, bounded
// mbarrier waits, TMA / bulk-copy issue, tcgen05 (TMEM + UMMA) wrappers,
// cluster / distributed-shared-memory access, bf16 conversions.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <cstdio>
#include <cstring>
#include <string>

#include "../../include/qtts_b200.h"

namespace qtts {

// ----------------------------------------------------------------------------
// host-side error text (per thread) and helpers
// ----------------------------------------------------------------------------
void set_error(const char* fmt, ...);

#define QTTS_CHECK_CUDA(expr)                                                         \
    do {                                                                              \
        cudaError_t _e = (expr);                                                      \
        if (_e != cudaSuccess) {                                                      \
            ::qtts::set_error("%s failed: %s (%s:%d)", #expr, cudaGetErrorString(_e), \
                              __FILE__, __LINE__);                                    \
            return QTTS_ERR_CUDA;                                                     \
        }                                                                             \
    } while (0)

#define QTTS_REQUIRE(cond, ...)            \
    do {                                   \
        if (!(cond)) {                     \
            ::qtts::set_error(__VA_ARGS__); \
            return QTTS_ERR_INVALID;       \
        }                                  \
    } while (0)

// One-time kernel attribute set-up, per kernel and device.  cudaFuncSetAttribute
// applies to the current device only, so a process that drives several GPUs
// needs it once on each; the kernel is a template argument so every kernel has
// its own record.  The bit of a device is set after its calls succeed (two
// threads racing on the first call both set the same values, which is
// harmless).  Devices past 63 set the attributes on every call.
template <auto Kernel>
inline cudaError_t func_attr_once(int smem_bytes, bool nonportable_cluster = false) {
    static std::atomic<unsigned long long> done{0};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    const unsigned long long bit = dev < 64 ? (1ull << dev) : 0ull;
    if (bit && (done.load(std::memory_order_acquire) & bit)) return cudaSuccess;
    e = cudaFuncSetAttribute(Kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes);
    if (e == cudaSuccess && nonportable_cluster)
        e = cudaFuncSetAttribute(Kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    if (e == cudaSuccess && bit) done.fetch_or(bit, std::memory_order_acq_rel);
    return e;
}

#define QTTS_LAUNCH_CHECK()                                                                   \
    do {                                                                                      \
        cudaError_t _e = cudaGetLastError();                                                  \
        if (_e != cudaSuccess) {                                                              \
            ::qtts::set_error("kernel launch failed: %s (%s:%d)", cudaGetErrorString(_e),     \
                              __FILE__, __LINE__);                                            \
            return QTTS_ERR_CUDA;                                                             \
        }                                                                                     \
    } while (0)

// ----------------------------------------------------------------------------
// device error word: bounded waits record where they gave up
// ----------------------------------------------------------------------------
__device__ int g_device_error;

enum DeviceErr : int {
    DEV_ERR_GEMM_PRODUCER = 1,
    DEV_ERR_GEMM_MMA = 2,
    DEV_ERR_GEMM_EPILOGUE = 3,
    DEV_ERR_ATTN_WAIT = 4,
    DEV_ERR_DRAIN = 5,
    DEV_ERR_BAD_SLOT = 6,  // a code2wav row named a slot outside the decoder's range
    DEV_ERR_SELFTEST_WAIT = 7,  // qtts_selftest_bounded_wait: the wait ran out, as the test intends
    DEV_ERR_ATTN_BOUNDS = 8,    // an attention kernel met a row / slot / index outside its buffers
    DEV_ERR_GRID_BARRIER = 9,   // a persistent kernel's grid barrier ran out of time
    DEV_ERR_GEMM_BOUNDS = 10,   // a GEMM epilogue access would have left its buffer (skipped)
};

// Wall-clock limit of every device-side wait (ns).  A correct kernel waits
// micro-seconds; two seconds means something is wrong, and the kernel then
// records the error and leaves instead of hanging the GPU.
constexpr unsigned long long kWaitLimitNs = 2000000000ull;

__device__ __forceinline__ unsigned long long globaltimer() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void record_error(int code) { atomicCAS(&g_device_error, 0, code); }

// ----------------------------------------------------------------------------
// shared-memory addresses, mbarriers
// ----------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait on an mbarrier phase.  Returns false (and records `err`) when
// the phase did not complete within `limit_ns` of %globaltimer.
__device__ __forceinline__ bool mbar_wait_for(uint64_t* bar, uint32_t parity, int err,
                                              unsigned long long limit_ns) {
    if (mbar_try_wait(bar, parity)) return true;
    const unsigned long long t0 = globaltimer();
    while (true) {
        if (mbar_try_wait(bar, parity)) return true;
        if (globaltimer() - t0 > limit_ns) {
            record_error(err);
            return false;
        }
    }
}

// The wait every kernel uses: kWaitLimitNs.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int err) {
    return mbar_wait_for(bar, parity, err, kWaitLimitNs);
}

__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ----------------------------------------------------------------------------
// TMA (tensor) and bulk (linear) copies global -> shared, completing on an mbarrier
// ----------------------------------------------------------------------------
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// 2-D tiled load: c0 = innermost coordinate (elements), c1 = row.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
        : "memory");
}

// Linear bulk copy of `bytes` (multiple of 16, both addresses 16-byte aligned).
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// ----------------------------------------------------------------------------
// tcgen05: TMEM allocation, UMMA issue, commit, TMEM -> register loads
// ----------------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
                 "r"(ncols)
                 : "memory");
}

__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc]^T, kind::f16 (bf16 inputs, fp32 accumulate).
__device__ __forceinline__ void umma_bf16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                          uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Arrive on `bar` once every UMMA issued so far by this thread has completed.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     smem_u32(bar))
                 : "memory");
}

// 32 lanes x 32 bits, 16 consecutive columns: thread i of the warp gets lane (32*(warp%4)+i).
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// 32 lanes x 32 bits, 16 consecutive columns: the inverse of tmem_ld16.
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const float (&v)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
            taddr),
        "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
        "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
        "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
        "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
        "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
        "r"(__float_as_uint(v[15]))
        : "memory");
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// Instruction descriptor: kind::f16, A/B fp16 K-major, D fp32, M x N.
__host__ __device__ constexpr uint32_t make_idesc_f16(int M, int N) {
    return (1u << 4)                       // D format fp32
           | ((uint32_t)(N >> 3) << 17)    // N (A, B format fp16 = 0)
           | ((uint32_t)(M >> 4) << 24);   // M
}

// Shared-memory matrix descriptor for a K-major tile written by TMA with
// 128-byte swizzle: rows of 128 B, 8-row atoms of 1024 B (SBO), version 1 (sm100).
__device__ __forceinline__ uint64_t make_sw128_desc(uint32_t smem_addr) {
    uint64_t d = 0;
    d |= (uint64_t)((smem_addr >> 4) & 0x3FFF);        // start address
    d |= (uint64_t)1 << 16;                            // leading byte offset (unused for swizzled K-major)
    d |= (uint64_t)(1024 >> 4) << 32;                  // stride byte offset: 8 rows x 128 B
    d |= (uint64_t)1 << 46;                            // descriptor version (Blackwell)
    d |= (uint64_t)2 << 61;                            // SWIZZLE_128B
    return d;
}

// Instruction descriptor: kind::f16, A/B bf16 K-major, D fp32, M x N.
__host__ __device__ constexpr uint32_t make_idesc_bf16(int M, int N) {
    return (1u << 4)                       // D format fp32
           | (1u << 7)                     // A format bf16
           | (1u << 10)                    // B format bf16
           | ((uint32_t)(N >> 3) << 17)    // N
           | ((uint32_t)(M >> 4) << 24);   // M
}

// ----------------------------------------------------------------------------
// clusters / distributed shared memory
// ----------------------------------------------------------------------------
__device__ __forceinline__ uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_arrive() {
    asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() {
    asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__device__ __forceinline__ uint32_t map_to_rank(uint32_t local_smem_addr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local_smem_addr), "r"(rank));
    return r;
}

__device__ __forceinline__ float ld_dsmem_f32(uint32_t addr) {
    float v;
    asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
    return v;
}

// No memory clobber: callers read data published by a cluster barrier, and the
// compiler may keep several of these loads in flight before their first use.
__device__ __forceinline__ float4 ld_dsmem_f32x4(uint32_t addr) {
    float4 v;
    asm volatile("ld.shared::cluster.v4.f32 {%0,%1,%2,%3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "r"(addr));
    return v;
}

// Store to (possibly another CTA's) shared memory in the cluster.
__device__ __forceinline__ void st_dsmem_f32x4(uint32_t addr, float a, float b, float c, float d) {
    asm volatile("st.shared::cluster.v4.f32 [%0], {%1,%2,%3,%4};" ::"r"(addr), "f"(a), "f"(b), "f"(c), "f"(d)
                 : "memory");
}

// ----------------------------------------------------------------------------
// numerics
// ----------------------------------------------------------------------------
__device__ __forceinline__ float bf16_round(float x) { return __bfloat162float(__float2bfloat16(x)); }

// KV cache element: fp16.  Same two bytes as the reference's bf16 cache, three
// more mantissa bits; K is RMS-normalised per head and V is a bounded linear
// map of a normalised input, so values sit far inside fp16 range (stores
// saturate at +-65504 all the same).
using kv_t = __half;
__device__ __forceinline__ kv_t to_kv(float x) { return __float2half_rn(fminf(fmaxf(x, -65504.f), 65504.f)); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

inline int ceil_div(int a, int b) { return (a + b - 1) / b; }

// kernels enqueued by this host thread (the engine reports it per step)
inline thread_local int g_launch_count = 0;

// ----------------------------------------------------------------------------
// programmatic dependent launch: a kernel launched with the attribute may
// start while its predecessor drains; it must call griddep_wait() before it
// touches anything the predecessor writes, and calls griddep_launch() to let
// its own successor start early.  Without a programmatic predecessor both are
// no-ops.  QTTS_PDL=0 in the environment turns the attribute off.
// ----------------------------------------------------------------------------
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

inline bool pdl_enabled() {
    static const bool on = [] {
        const char* v = getenv("QTTS_PDL");
        return !(v && v[0] == '0');
    }();
    return on;
}

// Launches made while this is non-zero go without programmatic dependent launch (a code2wav
// decoder marked as background: its CTAs would otherwise sit resident, holding shared memory,
// while they wait for their predecessor, keeping a concurrent stream's CTAs off those SMs).
// Host-side state of the one engine thread (as the reference's executor).
inline int g_pdl_suppress = 0;

// Launch with the programmatic-serialization attribute (and an optional cluster shape).
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                              dim3 cluster, Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    int n = 0;
    if (pdl_enabled() && !g_pdl_suppress) {
        attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[n].val.programmaticStreamSerializationAllowed = 1;
        ++n;
    }
    if (cluster.x * cluster.y * cluster.z > 1) {
        attr[n].id = cudaLaunchAttributeClusterDimension;
        attr[n].val.clusterDim.x = cluster.x;
        attr[n].val.clusterDim.y = cluster.y;
        attr[n].val.clusterDim.z = cluster.z;
        ++n;
    }
    cfg.attrs = attr;
    cfg.numAttrs = n;
    ++g_launch_count;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

#define QTTS_LAUNCH(kernel, grid, block, smem, st, ...)                                                 \
    do {                                                                                                \
        cudaError_t _e = ::qtts::launch_pdl(kernel, grid, block, smem, st, dim3(1, 1, 1), __VA_ARGS__); \
        if (_e != cudaSuccess) {                                                                        \
            ::qtts::set_error("launch of %s failed: %s (%s:%d)", #kernel, cudaGetErrorString(_e),       \
                              __FILE__, __LINE__);                                                      \
            return QTTS_ERR_CUDA;                                                                       \
        }                                                                                               \
    } while (0)

// cuTensorMapEncodeTiled through the runtime's driver entry point (no -lcuda).
typedef CUresult (*PFN_encodeTiled)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                    const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                    CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline PFN_encodeTiled get_encode_fn() {
    static PFN_encodeTiled fn = nullptr;
    if (!fn) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_encodeTiled>(p);
    }
    return fn;
}

inline int num_sms() {
    static int n = 0;
    if (n == 0) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        if (n <= 0) n = 148;
    }
    return n;
}

}  // namespace qtts
