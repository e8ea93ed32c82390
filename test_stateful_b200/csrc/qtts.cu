// libqtts_b200.so — one translation unit holding every sm_100a kernel of the
// decode backend and the extern "C" entry points declared in
// include/qtts_b200.h.  Each entry point validates its arguments, launches on
// the caller's stream and returns a status code; nothing here allocates per
// call except qtts_engine_create and qtts_c2w_create.
#include <cstdarg>
#include <mutex>
#include <new>

#include "common.cuh"
#include "code2wav.cuh"
#include "engine.cuh"

namespace qtts {

static thread_local char g_err[1024] = {0};

void set_error(const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof(g_err), fmt, ap);
    va_end(ap);
}

static bool state_ok(const qtts_paged_state* s) {
    return s && s->free_stack && s->free_top && s->refcount && s->block_table && s->seq_len && s->position_offset &&
           s->num_blocks > 0 && s->block_size == 16 && s->max_slots > 0 && s->max_blocks_per_seq > 0;
}

}  // namespace qtts

using namespace qtts;

extern "C" {

int qtts_version(void) { return 1; }

int qtts_last_error(char* buf, size_t size) {
    if (!buf || size == 0) return QTTS_ERR_INVALID;
    snprintf(buf, size, "%s", g_err);
    return QTTS_OK;
}

int qtts_device_error(int* out) {
    if (!out) return QTTS_ERR_INVALID;
    int v = 0, zero = 0;
    QTTS_CHECK_CUDA(cudaMemcpyFromSymbol(&v, g_device_error, sizeof(int)));
    QTTS_CHECK_CUDA(cudaMemcpyToSymbol(g_device_error, &zero, sizeof(int)));
    *out = v;
    return QTTS_OK;
}

// ---------------------------------------------------------------- paged state
int qtts_sched_init(const qtts_paged_state* st, qtts_stream_t stream) {
    QTTS_REQUIRE(state_ok(st), "sched_init: incomplete paged state (block_size must be 16)");
    sched_init_kernel<<<64, 256, 0, (cudaStream_t)stream>>>(view_of(st));
    QTTS_LAUNCH_CHECK();
    return QTTS_OK;
}

int qtts_sched_append(const qtts_paged_state* st, const int32_t* slots, int n_rows, int n_new, int32_t* slot_mapping,
                      int32_t* row_ctx, int32_t* row_pos, int32_t* cow_src, int32_t* cow_dst, int32_t* status,
                      qtts_stream_t stream) {
    QTTS_REQUIRE(state_ok(st), "sched_append: incomplete paged state");
    QTTS_REQUIRE(slots && slot_mapping && row_ctx && row_pos && cow_src && cow_dst && status,
                 "sched_append: null output");
    QTTS_REQUIRE(n_rows > 0 && n_rows <= kSchedThreads && n_new > 0, "sched_append: n_rows in [1, %d], n_new > 0",
                 kSchedThreads);
    sched_append_kernel<<<1, kSchedThreads, 0, (cudaStream_t)stream>>>(view_of(st), slots, n_rows, n_new,
                                                                       slot_mapping, row_ctx, row_pos, cow_src,
                                                                       cow_dst, status);
    QTTS_LAUNCH_CHECK();
    return QTTS_OK;
}

int qtts_kv_copy_blocks(void* kv_pool, size_t block_elems, int num_blocks, const int32_t* cow_src,
                        const int32_t* cow_dst, int n, qtts_stream_t stream) {
    QTTS_REQUIRE(kv_pool && cow_src && cow_dst && n >= 0, "kv_copy_blocks: bad arguments");
    QTTS_REQUIRE(block_elems % 8 == 0, "kv_copy_blocks: block size must be a multiple of 8 elements");
    if (n == 0) return QTTS_OK;
    kv_copy_blocks_kernel<<<dim3(64, n), 256, 0, (cudaStream_t)stream>>>(reinterpret_cast<uint4*>(kv_pool),
                                                                        block_elems / 8, cow_src, cow_dst, num_blocks);
    QTTS_LAUNCH_CHECK();
    return QTTS_OK;
}

int qtts_sched_share_prefix(const qtts_paged_state* st, int slot, const int32_t* blocks, int prefix_len,
                            int32_t* status, qtts_stream_t stream) {
    QTTS_REQUIRE(state_ok(st) && blocks, "sched_share_prefix: bad arguments");
    sched_share_prefix_kernel<<<1, 1, 0, (cudaStream_t)stream>>>(view_of(st), slot, blocks, prefix_len, status);
    QTTS_LAUNCH_CHECK();
    return QTTS_OK;
}

int qtts_sched_make_entry(const qtts_paged_state* st, int slot, int prefix_len, int32_t* blocks_out,
                          qtts_stream_t stream) {
    QTTS_REQUIRE(state_ok(st) && blocks_out, "sched_make_entry: bad arguments");
    QTTS_REQUIRE(slot >= 0 && slot < st->max_slots && prefix_len >= 0 &&
                     prefix_len <= st->max_blocks_per_seq * st->block_size,
                 "sched_make_entry: slot/prefix_len out of range");
    sched_make_entry_kernel<<<1, 1, 0, (cudaStream_t)stream>>>(view_of(st), slot, prefix_len, blocks_out);
    QTTS_LAUNCH_CHECK();
    return QTTS_OK;
}

int qtts_sched_drop_blocks(const qtts_paged_state* st, const int32_t* blocks, int n, qtts_stream_t stream) {
    QTTS_REQUIRE(state_ok(st) && blocks && n >= 0, "sched_drop_blocks: bad arguments");
    if (n == 0) return QTTS_OK;
    sched_drop_blocks_kernel<<<1, 1, 0, (cudaStream_t)stream>>>(view_of(st), blocks, n);
    QTTS_LAUNCH_CHECK();
    return QTTS_OK;
}

int qtts_sched_release(const qtts_paged_state* st, int slot, qtts_stream_t stream) {
    QTTS_REQUIRE(state_ok(st) && slot >= 0 && slot < st->max_slots, "sched_release: bad slot");
    sched_release_kernel<<<1, 1, 0, (cudaStream_t)stream>>>(view_of(st), slot);
    QTTS_LAUNCH_CHECK();
    return QTTS_OK;
}

int qtts_kv_scatter(void* kv_pool, const qtts_paged_state* st, int layers, int kv_heads, int head_dim,
                    const void* kv_rows, const int32_t* slot_mapping, int n, qtts_stream_t stream) {
    QTTS_REQUIRE(kv_pool && state_ok(st) && kv_rows && slot_mapping && n >= 0, "kv_scatter: bad arguments");
    if (n == 0) return QTTS_OK;
    kv_scatter_kernel<<<n, 256, 0, (cudaStream_t)stream>>>(
        reinterpret_cast<kv_t*>(kv_pool), 2 * layers, kv_heads, head_dim, st->block_size, st->num_blocks,
        reinterpret_cast<const kv_t*>(kv_rows), slot_mapping);
    QTTS_LAUNCH_CHECK();
    return QTTS_OK;
}

int qtts_kv_gather(const void* kv_pool, const qtts_paged_state* st, int layers, int kv_heads, int head_dim, int slot,
                   int n_tokens, void* out, qtts_stream_t stream) {
    QTTS_REQUIRE(kv_pool && state_ok(st) && out && slot >= 0 && slot < st->max_slots && n_tokens >= 0 &&
                     n_tokens <= st->max_blocks_per_seq * st->block_size,
                 "kv_gather: bad arguments");
    if (n_tokens == 0) return QTTS_OK;
    kv_gather_kernel<<<n_tokens, 256, 0, (cudaStream_t)stream>>>(
        reinterpret_cast<const kv_t*>(kv_pool), 2 * layers, kv_heads, head_dim, st->block_size,
        st->num_blocks, st->block_table + (size_t)slot * st->max_blocks_per_seq, n_tokens,
        reinterpret_cast<kv_t*>(out));
    QTTS_LAUNCH_CHECK();
    return QTTS_OK;
}

// ---------------------------------------------------------------- kernels
int qtts_gemm(const void* X, const void* X_lo, int M, int K, const void* W, int N, int epilogue, void* out,
              void* out_lo, const void* bias, const qtts_qkv_epilogue* qkv, qtts_stream_t stream) {
    QTTS_REQUIRE(X && W && out && M > 0, "gemm: null pointer or M <= 0");
    QTTS_REQUIRE(epilogue >= QTTS_EPI_BF16 && epilogue <= QTTS_EPI_QKV_ROPE, "gemm: unknown epilogue %d", epilogue);
    QTTS_REQUIRE(epilogue != QTTS_EPI_SWIGLU || N % 256 == 0 || N == 128, "gemm: SwiGLU needs N %% 128 == 0");
    GemmPlan g;
    int rc = gemm_plan(&g, X, M, K, W, N, epilogue, out, bias, qkv, X_lo, out_lo);
    if (rc) return rc;
    return gemm_run(g, M, (cudaStream_t)stream);
}

int qtts_rmsnorm(const float* x, int M, int H, int ld, const void* w, float eps, void* y, void* y_lo,
                 qtts_stream_t stream) {
    QTTS_REQUIRE(x && w && y && M >= 0 && H > 0 && ld >= H, "rmsnorm: bad arguments");
    return launch_rmsnorm(x, M, H, ld, w, eps, y, (cudaStream_t)stream, y_lo);
}

int qtts_paged_attention(const void* q, int R, int num_heads, int kv_heads, int head_dim, const void* kv_pool,
                         int layer, int num_layers, int block_size, int num_blocks, const int32_t* block_table,
                         int max_blocks_per_seq, const int32_t* row_slot, const int32_t* row_ctx, int max_ctx,
                         int split_blocks, float* ws_o, float* ws_ml, void* out, void* out_lo,
                         qtts_stream_t stream) {
    QTTS_REQUIRE(q && kv_pool && block_table && row_slot && row_ctx && ws_o && ws_ml && out && R >= 0,
                 "paged_attention: null pointer");
    QTTS_REQUIRE(block_size == 16, "paged_attention: block_size must be 16");
    QTTS_REQUIRE(kv_heads > 0 && num_heads == 2 * kv_heads, "paged_attention: needs 2 query heads per kv head");
    QTTS_REQUIRE(layer >= 0 && layer < num_layers && max_ctx > 0 && max_ctx <= max_blocks_per_seq * block_size,
                 "paged_attention: layer / max_ctx out of range");
    AttnParams p = {};
    p.q = reinterpret_cast<const float*>(q);
    p.kv = reinterpret_cast<const kv_t*>(kv_pool);
    p.num_heads = num_heads;
    p.kv_heads = kv_heads;
    p.layer = layer;
    p.num_layers = num_layers;
    p.block_size = block_size;
    p.num_blocks = num_blocks;
    p.block_table = block_table;
    p.mbps = max_blocks_per_seq;
    p.row_slot = row_slot;
    p.row_ctx = row_ctx;
    QTTS_REQUIRE(split_blocks >= 0 && split_blocks <= 1024, "paged_attention: split_blocks out of range");
    p.split_blocks = split_blocks > 0 ? split_blocks : QTTS_ATTN_SPLIT_BLOCKS;
    p.max_splits = attn_max_splits(max_ctx, p.split_blocks);
    p.scale_log2 = 1.4426950408889634f / sqrtf((float)head_dim);
    p.ws_o = ws_o;
    p.ws_ml = ws_ml;
    p.out = reinterpret_cast<__nv_bfloat16*>(out);
    p.out_lo = reinterpret_cast<__nv_bfloat16*>(out_lo);
    p.R = R;
    return launch_attention(p, head_dim, (cudaStream_t)stream);
}

int qtts_paged_attention_prefill(const void* q, int R, int rows_per_stream, int num_heads, int kv_heads,
                                 int head_dim, const void* kv_pool, int layer, int num_layers, int block_size,
                                 int num_blocks, const int32_t* block_table, int max_blocks_per_seq,
                                 const int32_t* row_slot, const int32_t* row_ctx, int max_ctx, int split_blocks,
                                 float* ws_o, float* ws_ml, void* out, void* out_lo, qtts_stream_t stream) {
    QTTS_REQUIRE(q && kv_pool && block_table && row_slot && row_ctx && ws_o && ws_ml && out && R >= 0,
                 "paged_attention_prefill: null pointer");
    QTTS_REQUIRE(head_dim == 128, "paged_attention_prefill: head_dim %d (the tile kernel takes 128)", head_dim);
    QTTS_REQUIRE(rows_per_stream >= 1 && R % rows_per_stream == 0,
                 "paged_attention_prefill: %d rows are not streams of %d tokens", R, rows_per_stream);
    QTTS_REQUIRE(block_size == 16, "paged_attention_prefill: block_size must be 16");
    QTTS_REQUIRE(kv_heads > 0 && num_heads == 2 * kv_heads,
                 "paged_attention_prefill: needs 2 query heads per kv head");
    QTTS_REQUIRE(layer >= 0 && layer < num_layers && max_ctx > 0 && max_ctx <= max_blocks_per_seq * block_size,
                 "paged_attention_prefill: layer / max_ctx out of range");
    QTTS_REQUIRE(split_blocks >= 0 && split_blocks <= 1024, "paged_attention_prefill: split_blocks out of range");
    AttnParams p = {};
    p.q = reinterpret_cast<const float*>(q);
    p.kv = reinterpret_cast<const kv_t*>(kv_pool);
    p.num_heads = num_heads;
    p.kv_heads = kv_heads;
    p.layer = layer;
    p.num_layers = num_layers;
    p.block_size = block_size;
    p.num_blocks = num_blocks;
    p.block_table = block_table;
    p.mbps = max_blocks_per_seq;
    p.row_slot = row_slot;
    p.row_ctx = row_ctx;
    p.split_blocks = split_blocks > 0 ? split_blocks : QTTS_ATTN_SPLIT_BLOCKS;
    p.max_splits = attn_max_splits(max_ctx, p.split_blocks);
    p.scale_log2 = 1.4426950408889634f / sqrtf((float)head_dim);
    p.ws_o = ws_o;
    p.ws_ml = ws_ml;
    p.out = reinterpret_cast<__nv_bfloat16*>(out);
    p.out_lo = reinterpret_cast<__nv_bfloat16*>(out_lo);
    p.R = R;
    p.rows_per_stream = rows_per_stream;
    return launch_prefill_attention(p, (cudaStream_t)stream);
}

int qtts_sample(const float* logits, int R, int V, int ld, int topk, const float* gumbel, int gumbel_ld, uint64_t seed,
                const int64_t* noise_key, int step, const float* temperature, const float* penalty, int64_t* counts,
                int eos_id, int64_t* tok_out, int tok_ld, qtts_stream_t stream) {
    QTTS_REQUIRE(logits && tok_out && R >= 0 && V > 0 && ld >= V, "sample: bad arguments");
    SampleParams p = {logits, R, V, ld, topk, gumbel, gumbel_ld, seed, noise_key, nullptr, step, temperature,
                      penalty, counts, nullptr, eos_id, tok_out, tok_ld};
    return launch_sample(p, (cudaStream_t)stream);
}

int qtts_philox_gumbel(uint64_t seed, const int64_t* keys, const int32_t* frames, int stage, int R, int cols,
                       float* out, qtts_stream_t stream) {
    QTTS_REQUIRE(keys && frames && out && R >= 0 && cols > 0 && cols <= 4096, "philox_gumbel: bad arguments");
    QTTS_REQUIRE(stage >= 0 && stage < 16, "philox_gumbel: stage %d outside [0, 16)", stage);
    if (R == 0) return QTTS_OK;
    philox_gumbel_kernel<<<R, 64, 0, (cudaStream_t)stream>>>(seed, keys, frames, stage, cols, out);
    QTTS_LAUNCH_CHECK();
    return QTTS_OK;
}

int qtts_codec_sum(const int64_t* codes, int R, int G, const void* talker_table, int V0, const void* cp_tables, int Vc,
                   int H, const float* text_add, float* codec_sum_out, float* next_x, qtts_stream_t stream) {
    QTTS_REQUIRE(codes && talker_table && next_x && R >= 0 && G >= 1 && H % 2 == 0, "codec_sum: bad arguments");
    QTTS_REQUIRE(G == 1 || cp_tables, "codec_sum: cp_tables needed for G > 1");
    if (R == 0) return QTTS_OK;
    codec_sum_kernel<<<R, 256, G * sizeof(int64_t), (cudaStream_t)stream>>>(
        codes, G, reinterpret_cast<const __nv_bfloat16*>(talker_table), V0,
        reinterpret_cast<const __nv_bfloat16*>(cp_tables), Vc, H, text_add, codec_sum_out, next_x, nullptr, nullptr);
    QTTS_LAUNCH_CHECK();
    return QTTS_OK;
}

// ---------------------------------------------------------------- engine
int qtts_engine_create(const qtts_model_desc* desc, qtts_engine** out) {
    QTTS_REQUIRE(desc && out, "engine_create: null argument");
    QTTS_REQUIRE(state_ok(&desc->pool) && desc->kv_pool, "engine_create: paged pool incomplete");
    QTTS_REQUIRE(desc->heads == 2 * desc->kv_heads && desc->cp_heads == 2 * desc->cp_kv_heads,
                 "engine_create: attention kernels need 2 query heads per kv head");
    QTTS_REQUIRE(desc->max_batch > 0 && desc->max_batch <= kSchedThreads && desc->max_prefill_rows >= 0,
                 "engine_create: max_batch in [1, %d]", kSchedThreads);
    QTTS_REQUIRE(desc->cp_stages + 1 <= 16, "engine_create: code predictor sequence must fit one 16-token block");
    qtts_engine* e = new (std::nothrow) qtts_engine();
    if (!e) {
        set_error("engine_create: out of host memory");
        return QTTS_ERR_INVALID;
    }
    e->d = *desc;
    const int rc = engine_build(e);
    if (rc != QTTS_OK) {
        for (void* p : e->allocs) cudaFree(p);
        delete e;
        return rc;
    }
    *out = e;
    return QTTS_OK;
}

int qtts_engine_destroy(qtts_engine* e) {
    if (!e) return QTTS_OK;
    for (void* p : e->allocs) cudaFree(p);
    delete e;
    return QTTS_OK;
}

int qtts_engine_step(qtts_engine* e, qtts_step_io* io, qtts_stream_t stream) {
    QTTS_REQUIRE(e && io, "engine_step: null argument");
    return engine_step(e, *io, (cudaStream_t)stream);
}

// ---------------------------------------------------------------- code2wav
int qtts_c2w_create(const qtts_c2w_desc* desc, qtts_c2w** out) {
    QTTS_REQUIRE(desc && out, "c2w_create: null argument");
    QTTS_REQUIRE(desc->rvq_tables && desc->w_pre_conv && desc->w_qkv && desc->w_conv0 && desc->final_w &&
                     desc->rope_cos && desc->rope_sin,
                 "c2w_create: weights incomplete");
    qtts_c2w* c = new (std::nothrow) qtts_c2w();
    if (!c) {
        set_error("c2w_create: out of host memory");
        return QTTS_ERR_INVALID;
    }
    c->d = *desc;
    const int rc = c2w_build(c);
    if (rc != QTTS_OK) {
        for (void* p : c->allocs) cudaFree(p);
        delete c;
        return rc;
    }
    *out = c;
    return QTTS_OK;
}

int qtts_c2w_destroy(qtts_c2w* c) {
    if (!c) return QTTS_OK;
    for (void* p : c->allocs) cudaFree(p);
    delete c;
    return QTTS_OK;
}

int qtts_c2w_reset(qtts_c2w* c, const int32_t* slots, int n, qtts_stream_t stream) {
    QTTS_REQUIRE(c && (n == 0 || slots), "c2w_reset: null argument");
    QTTS_REQUIRE(n >= 0 && n <= c->S, "c2w_reset: n=%d outside [0, %d]", n, c->S);
    return c2w_reset(c, slots, n, (cudaStream_t)stream);
}

int qtts_c2w_step(qtts_c2w* c, const int64_t* codes, int codes_ld, int frames, const int32_t* slots, int n, float* wav,
                  qtts_stream_t stream) {
    QTTS_REQUIRE(c, "c2w_step: null decoder");
    return c2w_step(c, codes, codes_ld, frames, slots, n, wav, (cudaStream_t)stream);
}

int qtts_c2w_launches(const qtts_c2w* c) { return c ? c->launches : 0; }

int qtts_c2w_state_layout(const qtts_c2w* c, qtts_c2w_state_part* parts, int max_parts) {
    QTTS_REQUIRE(c, "c2w_state_layout: null decoder");
    return c2w_state_layout(c, parts, max_parts);
}

int qtts_c2w_write_state(qtts_c2w* c, int slot, int part, const void* src, size_t bytes, qtts_stream_t stream) {
    QTTS_REQUIRE(c, "c2w_write_state: null decoder");
    return c2w_write_state(c, slot, part, src, bytes, (cudaStream_t)stream);
}

int qtts_c2w_set_frame(qtts_c2w* c, int slot, int frame, qtts_stream_t stream) {
    QTTS_REQUIRE(c, "c2w_set_frame: null decoder");
    return c2w_set_frame(c, slot, frame, (cudaStream_t)stream);
}

int qtts_c2w_set_background(qtts_c2w* c, int background) {
    QTTS_REQUIRE(c, "c2w_set_background: null decoder");
    c->background = background != 0;
    return QTTS_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Self-test of the bounded device wait (the failure path of every mbarrier
// wait in the library): one thread waits on an mbarrier phase with the
// caller's limit.  With arrive = 0 nothing completes the phase, so the wait
// runs out, records DEV_ERR_SELFTEST_WAIT in the device error word and the
// kernel writes QTTS_ERR_TIMEOUT to *status and returns; with arrive = 1 the
// thread arrives first and the wait succeeds (QTTS_OK).  The context stays
// usable either way.
// ---------------------------------------------------------------------------
namespace qtts {
__global__ void selftest_wait_kernel(unsigned long long limit_ns, int arrive, int32_t* status) {
    __shared__ __align__(8) uint64_t bar;
    mbar_init(&bar, 1);
    fence_mbar_init();
    if (arrive) mbar_arrive(&bar);
    const bool ok = mbar_wait_for(&bar, 0, DEV_ERR_SELFTEST_WAIT, limit_ns);
    status[0] = ok ? QTTS_OK : QTTS_ERR_TIMEOUT;
}
}  // namespace qtts

extern "C" int qtts_selftest_bounded_wait(unsigned long long limit_ns, int arrive, int32_t* status,
                                          qtts_stream_t stream) {
    QTTS_REQUIRE(status, "selftest_bounded_wait: null status");
    QTTS_REQUIRE(limit_ns > 0 && limit_ns <= kWaitLimitNs, "selftest_bounded_wait: limit %llu ns outside (0, %llu]",
                 limit_ns, kWaitLimitNs);
    selftest_wait_kernel<<<1, 1, 0, (cudaStream_t)stream>>>(limit_ns, arrive, status);
    QTTS_LAUNCH_CHECK();
    return QTTS_OK;
}

// ---------------------------------------------------------------------------
// Paged attention without caller scratch.
//
// qtts_paged_attention needs two scratch buffers for its split-KV partial
// results, which the caller allocates.  Some callers cannot allocate device
// memory at the point where they run attention: a host that owns every device
// allocation itself and hands plugins only the tensors of the call (a
// TensorRT-style plugin or a fixed-arena serving runtime), or a latency-bound
// thread that must not call cudaMalloc because it can synchronise the device.
// For them this variant keeps the partials in the static device array below,
// which every GPU that loads the library holds until the process exits.
//
// Limit: R * num_heads * max_splits * head_dim <= kNoAllocMaxPartials
// (4 MiB of fp32, e.g. 64 rows x 16 heads x 8 splits (2048 keys) x 128),
// with max_splits = ceil(ceil(max_ctx / 16) / QTTS_ATTN_SPLIT_BLOCKS).  The
// (max, sum) area is sized for the smallest head_dim the kernels take (32),
// so every shape within that limit fits.
// The device address of the array is looked up once per device and kept for
// the life of the process; a cudaDeviceReset followed by new work on that
// device is not supported by this entry point.
// Nothing in the array needs to start at zero: each call writes every partial
// it later reads.  All calls share the one array, so two calls that overlap
// on the GPU (different streams, no ordering between them) race on it.
// ---------------------------------------------------------------------------
namespace {

constexpr size_t kNoAllocMaxPartials = size_t(1) << 20;               // o partials, floats
constexpr int kNoAllocMinHeadDim = 32;                                 // smallest head_dim the kernels take
constexpr size_t kNoAllocMaxStats = kNoAllocMaxPartials / kNoAllocMinHeadDim * 2;  // (max, sum) pairs, floats
static __device__ __align__(256) float g_noalloc_attn_scratch[kNoAllocMaxPartials + kNoAllocMaxStats];

constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mu;
float* g_noalloc_ptr[kMaxDevices] = {nullptr};

// Device address of the static array on the current device, looked up once per device.
int noalloc_scratch(float** out) {
    int dev = 0;
    QTTS_CHECK_CUDA(cudaGetDevice(&dev));
    if (dev < 0 || dev >= kMaxDevices) {
        set_error("paged_attention_noalloc: device index %d out of range", dev);
        return QTTS_ERR_INVALID;
    }
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (!g_noalloc_ptr[dev]) {
        void* p = nullptr;
        const cudaError_t rc = cudaGetSymbolAddress(&p, g_noalloc_attn_scratch);
        if (rc != cudaSuccess || !p) {
            set_error("paged_attention_noalloc: cudaGetSymbolAddress failed: %s", cudaGetErrorString(rc));
            return QTTS_ERR_CUDA;
        }
        g_noalloc_ptr[dev] = static_cast<float*>(p);
    }
    *out = g_noalloc_ptr[dev];
    return QTTS_OK;
}

}  // namespace

extern "C" int qtts_paged_attention_noalloc(const void* q, int R, int num_heads, int kv_heads, int head_dim,
                                            const void* kv_pool, int layer, int num_layers, int block_size,
                                            int num_blocks, const int32_t* block_table, int max_blocks_per_seq,
                                            const int32_t* row_slot, const int32_t* row_ctx, int max_ctx, void* out,
                                            void* out_lo, qtts_stream_t stream) {
    QTTS_REQUIRE(R >= 0 && num_heads > 0 && head_dim >= kNoAllocMinHeadDim && max_ctx > 0,
                 "paged_attention_noalloc: bad shape (head_dim %d; the static scratch serves head_dim >= %d)",
                 head_dim, kNoAllocMinHeadDim);
    const size_t splits = (size_t)attn_max_splits(max_ctx);
    const size_t need_o = (size_t)R * num_heads * splits * head_dim;
    const size_t need_ml = (size_t)R * num_heads * splits * 2;
    if (need_o > kNoAllocMaxPartials) {
        set_error("paged_attention_noalloc: %zu rows x heads x splits x head_dim partials exceed the static scratch "
                  "of %zu floats; use fewer rows or qtts_paged_attention with caller scratch",
                  need_o, kNoAllocMaxPartials);
        return QTTS_ERR_INVALID;
    }
    if (need_ml > kNoAllocMaxStats) {  // cannot happen for head_dim >= 32 once need_o fits
        set_error("paged_attention_noalloc: %zu (max, sum) floats exceed the static scratch of %zu floats",
                  need_ml, kNoAllocMaxStats);
        return QTTS_ERR_INVALID;
    }
    float* scratch = nullptr;
    const int rc = noalloc_scratch(&scratch);
    if (rc != QTTS_OK) return rc;
    return qtts_paged_attention(q, R, num_heads, kv_heads, head_dim, kv_pool, layer, num_layers, block_size,
                                num_blocks, block_table, max_blocks_per_seq, row_slot, row_ctx, max_ctx, 0, scratch,
                                scratch + kNoAllocMaxPartials, out, out_lo, stream);
}
