// Code-predictor stage as one persistent launch.
//
// A code-predictor stage s >= 1 (utils.py:1003-1042, KV-cached: one new token per
// stream) is 5 transformer layers and the stage's lm_head.  As separate launches
// it is a chain of ~26 dependent kernels, and at 64 streams each one is a few
// microseconds of launch, ramp and drain around well under a microsecond of
// weight streaming (about 124 MB of bf16 weights per stage, L2-resident).  Here
// one launch walks the stage's GEMMs as a PROGRAM of phases:
//
//   per layer: QKV (paired tiles, q/k norm + RoPE + KV store + the decode
//   attention in the epilogue) | O (+ residual, folded post-norm) |
//   gate/up (+ SwiGLU) | down (+ residual, folded next norm)
//   then the lm_head (folded final norm, fp32 logits)
//
// with a grid-wide barrier between phases.  Each phase is exactly the
// per-launch GEMM's work: 128-row weight tiles on the UMMA M side, the tokens
// as a bf16 hi/lo pair on N (TMEM accumulator of 2 x 64 columns), split-K over
// the 8 CTAs of a thread-block cluster with the partial sums reduced through
// distributed shared memory, and the same fused epilogues (gemm_epilogue,
// pair_attention).  What the persistent form adds:
//
//  * the CTAs stay resident (cooperative launch, one CTA per SM, clusters of 8):
//    no launch, ramp or drain between phases, only a ~1 us grid barrier;
//  * the weights do not depend on the previous phase, so the producer thread
//    issues the TMA loads of its NEXT job's weight tiles into the free ring
//    stages before this job's epilogue and the barrier; after the barrier only
//    the activation tiles (written by the previous phase) are on the critical
//    path;
//  * a cluster with several jobs in one phase (gate/up: 48 tiles over 18
//    clusters) issues the next job's loads, activations included, under the
//    current job's epilogue.
//
// Every wait is bounded (mbarrier waits and the grid barrier give up after
// kWaitLimitNs, record a device error and carry on without issuing work), and
// every CTA of a cluster runs the same sequence of cluster barriers, so a
// failure ends the launch instead of hanging the GPU.
#pragma once

#include "gemm_tc.cuh"

namespace qtts {

constexpr int kCppCluster = 8;  // CTAs per cluster: split-K 8, or 2 paired tiles x split-K 4
constexpr int kCppStages = 4;   // ring stages (weight tile + hi/lo activation tiles)
constexpr int kCppBN = 64;      // tokens per tile
constexpr int kCppThreads = 128;
constexpr int kCppMaxPhases = 32;

// optional timestamps (a profiling build defines CPP_STAMP(i))
#ifndef CPP_STAMP
#define CPP_STAMP(i) \
    do {             \
    } while (0)
#endif
#ifndef CPP_STAMP_JOB
#define CPP_STAMP_JOB(ph, j, i) \
    do {                        \
    } while (0)
#endif

// One phase of the program: a GEMM plan's tensor maps and parameters.  M (the
// streams of the launch) and splits are set by the kernel.
struct alignas(64) CpPhase {
    CUtensorMap mw;    // weights [N][K] bf16, box 64 x 128
    CUtensorMap mx;    // activation hi [rows][K], box 64 x kCppBN
    CUtensorMap mxlo;  // activation lo
    GemmParams p;
    int tiles_n;       // 128-row weight tiles
    int members;       // weight tiles per cluster (paired QKV: 2); split-K = 8 / members
    int pair;          // paired QKV tiles (decode attention after the epilogue)
};

// What the kernel keeps of a phase in shared memory (loaded once per launch).
struct alignas(16) CppInfo {
    GemmParams p;
    int tiles_n, members, pair, pad;
};

struct CppLayout {
    static constexpr int A_BYTES = 128 * 64 * 2;
    static constexpr int B_BYTES = kCppBN * 64 * 2;
    static constexpr int STAGE_BYTES = A_BYTES + 2 * B_BYTES;
    static constexpr int RING = kCppStages * STAGE_BYTES;
    static constexpr int PART_BYTES = kCppBN * 128 * 4;  // fp32 partial [token][128 rows]
    static constexpr int SCRATCH_BYTES = 7 * 128 * 4;    // as the per-launch kernel's scratch
    static constexpr int INFO_BYTES = kCppMaxPhases * (int)sizeof(CppInfo);
    static constexpr int BAR_BYTES = 256;
    static constexpr int PART = RING;
    static constexpr int SCRATCH = PART + PART_BYTES;
    static constexpr int INFO = SCRATCH + SCRATCH_BYTES;
    static constexpr int BAR = (INFO + INFO_BYTES + 15) / 16 * 16;
    static constexpr int SMEM = 1024 + BAR + BAR_BYTES;
    static_assert(STAGE_BYTES % 1024 == 0, "stages keep the 1024-B alignment of the swizzled tiles");
    static_assert(sizeof(CppInfo) % 16 == 0 && SMEM <= 227 * 1024, "shared memory layout");
};

__device__ __forceinline__ int cpp_jobs(const CppInfo& ph, int tiles_m) {
    return ph.tiles_n / ph.members * tiles_m;
}

// Grid barrier: every CTA adds one to a counter (release) and waits until it reaches
// `target` (acquire).  The counter only grows during a launch; the launch's last CTA to
// leave resets it.  Bounded: gives up after kWaitLimitNs and records the error.
__device__ __forceinline__ bool cpp_grid_barrier(unsigned* counter, unsigned target) {
    asm volatile("fence.acq_rel.gpu;\n\tred.relaxed.gpu.global.add.u32 [%0], 1;" ::"l"(counter) : "memory");
    const unsigned long long t0 = globaltimer();
    while (true) {
        unsigned v;
        asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(counter) : "memory");
        if (v >= target) return true;
        if (globaltimer() - t0 > kWaitLimitNs) {
            record_error(DEV_ERR_GRID_BARRIER);
            return false;
        }
    }
}

__device__ __forceinline__ void fence_proxy_async_global() {
    asm volatile("fence.proxy.async.global;" ::: "memory");
}

// Job j of a phase for the cluster: weight tile, token tile, this CTA's K range.  The
// cluster holds `members` weight tiles x (8 / members) splits; rank = member + members * split.
struct CppJob {
    int tile_n, tile_m, split, pm, splits, kb0, nkb;
};

__device__ __forceinline__ CppJob cpp_job(const CppInfo& ph, int j, int tiles_m, int crank) {
    CppJob J;
    const int unit = j / tiles_m;
    J.tile_m = j - unit * tiles_m;
    J.splits = kCppCluster / ph.members;
    J.split = crank / ph.members;
    J.pm = crank - J.split * ph.members;
    J.tile_n = ph.members * unit + J.pm;
    const int kblocks = ph.p.kblocks;
    const int per_split = kblocks / J.splits, rem = kblocks % J.splits;
    J.kb0 = J.split * per_split + min(J.split, rem);
    J.nkb = per_split + (J.split < rem ? 1 : 0);
    return J;
}

// gbar[0]: barrier counter, gbar[1]: CTAs that have left (both zero between launches).
__global__ void __launch_bounds__(kCppThreads, 1)
    cp_persist_kernel(const CpPhase* __restrict__ prog, int n_phases, int nr, unsigned* gbar) {
    using L = CppLayout;
    constexpr int BN = kCppBN, S = kCppStages, NT = kCppThreads;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    float* P = reinterpret_cast<float*>(smem + L::PART);
    float* scratch = reinterpret_cast<float*>(smem + L::SCRATCH);
    CppInfo* info = reinterpret_cast<CppInfo*>(smem + L::INFO);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::BAR);
    uint64_t* empty = full + S;
    uint64_t* accum = empty + S;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accum + 1);
    volatile int* dead = reinterpret_cast<volatile int*>(tmem_slot + 1);  // a wait of this CTA gave up
    int* counts = reinterpret_cast<int*>(tmem_slot + 2);  // [0] stages loaded (producer), [1] consumed (MMA)

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int crank = (int)cluster_ctarank();
    const int cid = (int)blockIdx.x / kCppCluster, n_clusters = (int)gridDim.x / kCppCluster;
    const int tiles_m = (nr + BN - 1) / BN;
    CPP_STAMP(0);
    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(accum, 1);
        *dead = 0;
        counts[0] = counts[1] = 0;
        fence_mbar_init();
        tma_prefetch_desc(&prog[0].mw);
        tma_prefetch_desc(&prog[0].mx);
        tma_prefetch_desc(&prog[0].mxlo);
    }
    // the program's parameters (written before the launch) into shared memory: every
    // thread copies 32-bit words of all phases, loads in flight together
    {
        static_assert(sizeof(GemmParams) % 4 == 0, "copied as 32-bit words");
        constexpr int W = (int)(sizeof(GemmParams) / 4);
        const int n = (n_phases < kCppMaxPhases ? n_phases : kCppMaxPhases) * W;
        for (int e = threadIdx.x; e < n; e += NT) {
            const int ph = e / W, w = e - ph * W;
            reinterpret_cast<uint32_t*>(&info[ph].p)[w] = reinterpret_cast<const uint32_t*>(&prog[ph].p)[w];
        }
        for (int ph = threadIdx.x; ph < n_phases && ph < kCppMaxPhases; ph += NT) {
            info[ph].tiles_n = prog[ph].tiles_n;
            info[ph].members = prog[ph].members;
            info[ph].pair = prog[ph].pair;
        }
    }
    if (warp == 2) {
        tmem_alloc(tmem_slot, 2 * BN);
        tmem_relinquish();
    }
    __syncthreads();
    for (int ph = threadIdx.x; ph < n_phases && ph < kCppMaxPhases; ph += NT) {
        info[ph].p.M = nr;
        info[ph].p.splits = kCppCluster / info[ph].members;
    }
    griddep_wait();  // the stage input, the KV cache and gbar belong to earlier kernels
    CPP_STAMP(1);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    int it = 0;       // ring k-blocks of all earlier jobs (uniform across the CTA)
    int jc = 0;       // jobs done (accumulator barrier parity)
    int pre_w = 0;    // producer only: k-blocks of the current job whose weight / activation
    int pre_x = 0;    // loads were issued ahead of it
    for (int ph = 0; ph < n_phases; ++ph) {
        const CppInfo& PI = info[ph];
        const GemmParams& gp = PI.p;
        const CpPhase& PH = prog[ph];
        if (threadIdx.x == 0 && ph + 1 < n_phases) {  // the next phase's descriptors
            tma_prefetch_desc(&prog[ph + 1].mw);
            tma_prefetch_desc(&prog[ph + 1].mx);
            tma_prefetch_desc(&prog[ph + 1].mxlo);
        }
        if (ph + 1 == n_phases) griddep_launch();  // the sampling kernel may start its prologue
        CPP_STAMP(2 + 2 * ph);
        const int jobs = cpp_jobs(PI, tiles_m);
        for (int j = cid; j < jobs; j += n_clusters) {
            const CppJob J = cpp_job(PI, j, tiles_m, crank);
            CPP_STAMP_JOB(ph, j, 0);
            if (threadIdx.x == 0) {
                // ---------------- producer: this job's remaining loads ----------------
                for (int i = 0; i < J.nkb && !*dead; ++i) {
                    const int g = it + i, s = g % S;
                    uint8_t* a = smem + s * L::STAGE_BYTES;
                    if (i >= pre_w) {
                        if (g >= S && !mbar_wait(&empty[s], ((uint32_t)(g / S) & 1u) ^ 1u, DEV_ERR_GEMM_PRODUCER)) {
                            *dead = 1;
                            break;
                        }
                        mbar_arrive_expect_tx(&full[s], L::STAGE_BYTES);
                        tma_load_2d(a, &PH.mw, &full[s], (J.kb0 + i) * 64, J.tile_n * 128);
                        ++counts[0];
                    }
                    if (i >= pre_x) {
                        tma_load_2d(a + L::A_BYTES, &PH.mx, &full[s], (J.kb0 + i) * 64, J.tile_m * BN);
                        tma_load_2d(a + L::A_BYTES + L::B_BYTES, &PH.mxlo, &full[s], (J.kb0 + i) * 64, J.tile_m * BN);
                    }
                }
                // ---------------- prefetch: the next job's weights (and, in the same
                // phase, its activations) into the stages this job's MMAs free ----------------
                int ph2 = ph, j2 = j + n_clusters;
                while (ph2 < n_phases && j2 >= cpp_jobs(info[ph2], tiles_m)) {
                    ++ph2;
                    j2 = cid;
                }
                pre_w = pre_x = 0;
                if (ph2 < n_phases && !*dead) {
                    const CpPhase& NX = prog[ph2];
                    const CppJob J2 = cpp_job(info[ph2], j2, tiles_m, crank);
                    const int n = J2.nkb < S ? J2.nkb : S;
                    for (int i = 0; i < n; ++i) {
                        const int g = it + J.nkb + i, s = g % S;
                        uint8_t* a = smem + s * L::STAGE_BYTES;
                        if (g >= S && !mbar_wait(&empty[s], ((uint32_t)(g / S) & 1u) ^ 1u, DEV_ERR_GEMM_PRODUCER)) {
                            *dead = 1;
                            break;
                        }
                        mbar_arrive_expect_tx(&full[s], L::STAGE_BYTES);
                        tma_load_2d(a, &NX.mw, &full[s], (J2.kb0 + i) * 64, J2.tile_n * 128);
                        ++counts[0];
                        ++pre_w;
                        if (ph2 == ph) {
                            tma_load_2d(a + L::A_BYTES, &NX.mx, &full[s], (J2.kb0 + i) * 64, J2.tile_m * BN);
                            tma_load_2d(a + L::A_BYTES + L::B_BYTES, &NX.mxlo, &full[s], (J2.kb0 + i) * 64,
                                        J2.tile_m * BN);
                            ++pre_x;
                        }
                    }
                }
            } else if (threadIdx.x == 32) {
                // ---------------- UMMA issuer ----------------
                const uint32_t idesc = make_idesc_bf16(128, 2 * BN);
                for (int i = 0; i < J.nkb && !*dead; ++i) {
                    const int g = it + i, s = g % S;
                    if (!mbar_wait(&full[s], (uint32_t)(g / S) & 1u, DEV_ERR_GEMM_MMA)) {
                        *dead = 1;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a = smem_u32(smem + s * L::STAGE_BYTES);
                    const uint64_t da = make_sw128_desc(a);
                    const uint64_t db = make_sw128_desc(a + L::A_BYTES);
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk)
                        umma_bf16(tmem, da + 2 * kk, db + 2 * kk, idesc, (i > 0 || kk > 0) ? 1u : 0u);
                    umma_commit(&empty[s]);
                    ++counts[1];
                }
                umma_commit(accum);  // fires when this job's UMMAs have completed (at once if none)
            }
            __syncwarp();
            CPP_STAMP_JOB(ph, j, 1);
            it += J.nkb;
            const int m0 = J.split * BN / J.splits;
            const int per = (J.split + 1) * BN / J.splits - m0;
            // the epilogue's own loads (norm sums, token metadata, old residual values) while
            // the tiles land and the UMMAs run
            epilogue_meta<BN, NT>(gp, scratch, m0, per, J.tile_m);
            float pre_old[8];
            const bool prefetch = gp.epilogue == QTTS_EPI_RESIDUAL && per <= 8;
            if (prefetch) residual_prefetch<BN, NT>(gp, m0, per, J.tile_n, J.tile_m, pre_old);

            // ---------------- TMEM -> partial ----------------
            const bool ok = mbar_wait(accum, (uint32_t)jc & 1u, DEV_ERR_GEMM_EPILOGUE);
            ++jc;
            tc_fence_after();
            __syncthreads();
            const bool good = ok && !*dead;
            CPP_STAMP_JOB(ph, j, 2);
            {
                const int row = warp * 32 + lane;
#pragma unroll 1
                for (int c = 0; c < BN; c += 16) {
                    float v[16], vl[16];
                    tmem_ld16(tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)c, v);
                    tmem_ld16(tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)(c + BN), vl);
#pragma unroll
                    for (int k = 0; k < 16; ++k) P[(c + k) * 128 + row] = good ? v[k] + vl[k] : 0.0f;
                }
            }
            tc_fence_before();
            __syncthreads();
            CPP_STAMP_JOB(ph, j, 3);

            // ---------------- split-K reduction across the cluster, epilogue ----------------
            cluster_arrive();  // this CTA's partial is in its shared memory
            CPP_STAMP_JOB(ph, j, 4);
            cluster_wait();
            CPP_STAMP_JOB(ph, j, 5);
            cluster_reduce_slice<NT>(P, m0, per, J.splits, PI.members, J.pm);
            if (!PI.pair) cluster_arrive();  // done reading the peers' partials
            __syncthreads();
            CPP_STAMP_JOB(ph, j, 6);
            gemm_epilogue<BN, NT>(gp, P, m0, per, J.tile_n, J.tile_m, scratch, prefetch ? pre_old : nullptr);
            CPP_STAMP_JOB(ph, j, 7);
            if (PI.pair) {
                // both tiles' stores (q, cache K/V) reach the cluster before either reads them;
                // this barrier also ends the reads of the peers' partials
                __syncthreads();
                cluster_arrive();
                cluster_wait();
                pair_attention<BN>(gp, m0, per, J.tile_n, J.tile_m, J.pm, scratch);
            } else {
                cluster_wait();  // no peer still reads this CTA's partial
            }
            CPP_STAMP_JOB(ph, j, 8);
            // the next phase reads this job's stores through TMA (the async proxy)
            fence_proxy_async_global();
            // the next job's early loads rewrite the scratch this job's epilogue reads
            __syncthreads();
            CPP_STAMP_JOB(ph, j, 9);
        }
        CPP_STAMP(3 + 2 * ph);
        if (ph + 1 < n_phases) {
            __syncthreads();
            if (threadIdx.x == 0) {
                if (!cpp_grid_barrier(&gbar[0], (unsigned)(ph + 1) * gridDim.x)) *dead = 1;
                fence_proxy_async_global();
            }
            __syncthreads();
        }
    }
    // ---------------- drain (after a failure), release TMEM, reset the barrier ----------------
    __syncthreads();
    if (threadIdx.x == 0 && *dead) {
        for (int i = counts[1]; i < counts[0]; ++i) mbar_wait(&full[i % S], (uint32_t)(i / S) & 1u, DEV_ERR_DRAIN);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 2) tmem_dealloc(tmem, 2 * BN);
    if (threadIdx.x == 0) {
        __threadfence();
        if (atomicAdd(&gbar[1], 1u) == gridDim.x - 1) {
            gbar[0] = 0;
            gbar[1] = 0;
            __threadfence();
        }
    }
    CPP_STAMP(63);
}

// Clusters of 8 that fit the GPU at one CTA per SM (at most 18: 144 CTAs).
inline int cp_persist_clusters() {
    static int n = -1;
    if (n < 0) {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(kCppCluster * 32);
        cfg.blockDim = dim3(kCppThreads);
        cfg.dynamicSmemBytes = CppLayout::SMEM;
        cudaLaunchAttribute at[1];
        at[0].id = cudaLaunchAttributeClusterDimension;
        at[0].val.clusterDim.x = kCppCluster;
        at[0].val.clusterDim.y = 1;
        at[0].val.clusterDim.z = 1;
        cfg.attrs = at;
        cfg.numAttrs = 1;
        int c = 0;
        if (cudaFuncSetAttribute(cp_persist_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, CppLayout::SMEM) !=
                cudaSuccess ||
            cudaOccupancyMaxActiveClusters(&c, cp_persist_kernel, &cfg) != cudaSuccess)
            c = 0;
        n = c < 18 ? c : 18;
    }
    return n;
}

// One stage: the program prog[0 .. n_phases) for nr streams.  Cooperative launch (all CTAs
// resident, which the grid barrier needs) with clusters of 8 and programmatic dependent launch.
inline int launch_cp_persist(const CpPhase* prog, int n_phases, int nr, unsigned* gbar, cudaStream_t st) {
    const int clusters = cp_persist_clusters();
    if (clusters <= 0) {
        set_error("cp_persist: no cluster of %d CTAs fits (%d B shared memory each)", kCppCluster, CppLayout::SMEM);
        return QTTS_ERR_CUDA;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(kCppCluster * clusters);
    cfg.blockDim = dim3(kCppThreads);
    cfg.dynamicSmemBytes = CppLayout::SMEM;
    cfg.stream = st;
    cudaLaunchAttribute at[3];
    int n = 0;
    at[n].id = cudaLaunchAttributeClusterDimension;
    at[n].val.clusterDim.x = kCppCluster;
    at[n].val.clusterDim.y = 1;
    at[n].val.clusterDim.z = 1;
    ++n;
    at[n].id = cudaLaunchAttributeCooperative;
    at[n].val.cooperative = 1;
    ++n;
    if (pdl_enabled() && !g_pdl_suppress) {
        at[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        at[n].val.programmaticStreamSerializationAllowed = 1;
        ++n;
    }
    cfg.attrs = at;
    cfg.numAttrs = n;
    ++g_launch_count;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, cp_persist_kernel, prog, n_phases, nr, gbar);
    if (e != cudaSuccess) {
        set_error("launch of cp_persist_kernel failed: %s", cudaGetErrorString(e));
        return QTTS_ERR_CUDA;
    }
    return QTTS_OK;
}

// Program entry from a GEMM plan (BN = 64 maps): `members` weight tiles per cluster
// (split-K 8 / members; paired QKV tiles: 2).
inline int cp_phase_from_plan(CpPhase* ph, const GemmPlan& g, bool pair, int members) {
    memset(ph, 0, sizeof(*ph));
    ph->mw = g.mw;
    ph->mx = g.mx64;
    ph->mxlo = g.split ? g.mlo64 : g.mx64;
    ph->p = g.p;
    ph->tiles_n = g.p.N / 128;
    ph->members = pair ? 2 : members;
    ph->pair = pair ? 1 : 0;
    if (kCppCluster % ph->members != 0 || ph->tiles_n % ph->members != 0 ||
        g.p.kblocks < kCppCluster / ph->members) {
        set_error("cp_persist: %d tiles, %d k-blocks do not fit %d tiles per cluster", ph->tiles_n, g.p.kblocks,
                  ph->members);
        return QTTS_ERR_UNSUPPORTED;
    }
    return QTTS_OK;
}

}  // namespace qtts
