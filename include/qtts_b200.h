/*
 * qtts_b200.h — C ABI of the B200 (sm_100a) decode backend for the Qwen3-TTS
 * standalone engine.
 *
 * The reference engine reaches its GPU work through one call,
 * Executor.launch_decode_step -> TRTEngine.infer -> execute_async_v3
 * (engine/backend/executor.py:1087-1183, 220-336), whose tensor contract is
 * the fused talker+code-predictor+code2wav graph
 * (scripts/export/export_09_talker_code2wav_fused.py:1-33, 106-166;
 * dtypes scripts/python/trt_fused_io_formats.py:63-118).  This library is the
 * new device side of that boundary: plain device pointers, sizes and a
 * cudaStream_t, int status codes, no C++ or torch types.  Every function
 * returns QTTS_OK (0) or a negative status; qtts_last_error() gives the text.
 *
 * Threading: one engine thread owns all GPU state (engine/backend/engine_loop.py:53-56);
 * the functions are not re-entrant for the same handle.
 */
#ifndef QTTS_B200_H
#define QTTS_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes (mapped to ValueError / RuntimeError by the Python host,
 *      as executor.py:253-302, 394, 632-638 raise them) ---------------------- */
#define QTTS_OK                  0
#define QTTS_ERR_INVALID        -1   /* bad argument (ValueError)                  */
#define QTTS_ERR_CUDA           -2   /* a CUDA runtime call failed                  */
#define QTTS_ERR_CAPACITY       -3   /* a sequence would pass max_seq_len           */
#define QTTS_ERR_POOL_EXHAUSTED -4   /* no free KV blocks                           */
#define QTTS_ERR_TIMEOUT        -5   /* a bounded device wait gave up               */
#define QTTS_ERR_UNSUPPORTED    -6   /* shape/config outside what the kernels take  */

typedef void* qtts_stream_t; /* a cudaStream_t */

/* Library version and the last error message of this thread. */
int qtts_version(void);
int qtts_last_error(char* buf, size_t size);
/* Read and clear the device-side error word set by bounded waits (0 = none). */
int qtts_device_error(int* out);
/* Self-test of the bounded device wait that every mbarrier wait of the library uses (no
 * counterpart in the reference, whose waits are TensorRT's): one thread waits up to
 * limit_ns (<= 2 s) on an mbarrier phase.  arrive = 0: nothing completes the phase, the wait
 * runs out, the device error word records it and status[0] (device int32) = QTTS_ERR_TIMEOUT;
 * arrive = 1: the phase completes and status[0] = QTTS_OK.  No trap, no hang: the kernel
 * returns and the context stays usable. */
int qtts_selftest_bounded_wait(unsigned long long limit_ns, int arrive, int32_t* status, qtts_stream_t stream);

/* ========================================================================
 * Paged KV pool state (on device)
 *
 * Replaces KVCachePool.allocate/release/scatter_*_kv* and the prefix-cache
 * copy (engine/backend/kv_cache_pool.py:269-341, 383-395, 410-420, 480-498;
 * engine/backend/prefix_cache.py:101-148; engine/backend/engine_loop.py:823-835)
 * with a block allocator: LIFO free stack, per-block refcounts, per-slot block
 * tables and sequence lengths, all int32 in device memory.
 *   free_stack [num_blocks], free_top [1], refcount [num_blocks],
 *   block_table [max_slots * max_blocks_per_seq] (-1 = unassigned),
 *   seq_len [max_slots]
 * ======================================================================== */
typedef struct qtts_paged_state {
    int32_t* free_stack;
    int32_t* free_top;
    int32_t* refcount;
    int32_t* block_table;
    int32_t* seq_len;
    int32_t* position_offset;   /* per slot RoPE offset (kv_cache_pool.py:85-88) */
    int32_t  num_blocks;
    int32_t  block_size;        /* tokens per block (16) */
    int32_t  max_slots;
    int32_t  max_blocks_per_seq;
} qtts_paged_state;

/* Reset: stack = [num_blocks-1 .. 0] (first pop gives block 0), refcounts 0,
 * tables -1, seq_len 0, position_offset 0. */
int qtts_sched_init(const qtts_paged_state* st, qtts_stream_t stream);

/* Reserve n_new KV positions for each of n_rows slots, in batch order.
 * Outputs: slot_mapping[n_rows*n_new] (block*block_size + offset, int32),
 * row_ctx[n_rows*n_new] (keys visible to each new token = its position + 1),
 * row_pos[n_rows*n_new] (RoPE position = position_offset + position),
 * cow_src/cow_dst[n_rows] (-1 = no copy), status[1].
 * All-or-nothing: on QTTS_ERR_CAPACITY / QTTS_ERR_POOL_EXHAUSTED (written to
 * *status on the device) the state is unchanged and slot_mapping is -1.
 * Replaces the per-step gather + delta scatter of kv_cache_pool.py:410-420, 480-498. */
int qtts_sched_append(const qtts_paged_state* st, const int32_t* slots, int n_rows, int n_new,
                      int32_t* slot_mapping, int32_t* row_ctx, int32_t* row_pos,
                      int32_t* cow_src, int32_t* cow_dst, int32_t* status, qtts_stream_t stream);

/* Copy whole KV blocks for the (cow_src[i], cow_dst[i]) pairs with src >= 0.
 * kv_pool layout: [num_blocks][layers][2][kv_heads][block_size][head_dim] fp16 (same bytes as the
 * reference's bf16 cache, 3 more mantissa bits; K is RMS-normalised, V bounded). */
int qtts_kv_copy_blocks(void* kv_pool, size_t block_elems, int num_blocks, const int32_t* cow_src,
                        const int32_t* cow_dst, int n, qtts_stream_t stream);

/* Point an empty slot at n_blocks cached blocks (refcount+1 each), seq_len = prefix_len.
 * (PrefixKVCache.get + engine_loop._restore_prefix_cache, without the copy.) */
int qtts_sched_share_prefix(const qtts_paged_state* st, int slot, const int32_t* blocks,
                            int prefix_len, int32_t* status, qtts_stream_t stream);
/* Take a reference on a slot's first ceil(prefix_len/bs) blocks and write their ids
 * to blocks_out (PrefixKVCache.put without the clone, prefix_cache.py:101-148). */
int qtts_sched_make_entry(const qtts_paged_state* st, int slot, int prefix_len,
                          int32_t* blocks_out, qtts_stream_t stream);
/* Drop one reference on each listed block; blocks reaching 0 are pushed in order. */
int qtts_sched_drop_blocks(const qtts_paged_state* st, const int32_t* blocks, int n,
                           qtts_stream_t stream);
/* KVCachePool.release (kv_cache_pool.py:308-341): drop the slot's blocks, seq_len = 0. */
int qtts_sched_release(const qtts_paged_state* st, int slot, qtts_stream_t stream);

/* Write per-token K/V rows into the pool through slot_mapping (-1 skipped).
 * kv_rows: [n][layers*2][kv_heads][head_dim] fp16 (KVCachePool.scatter_prefill_kv layout). */
int qtts_kv_scatter(void* kv_pool, const qtts_paged_state* st, int layers, int kv_heads, int head_dim,
                    const void* kv_rows, const int32_t* slot_mapping, int n, qtts_stream_t stream);
/* Logical KV of one slot: out [layers*2][kv_heads][n_tokens][head_dim] fp16
 * (KVCachePool.gather_talker_kv, kv_cache_pool.py:410-420). */
int qtts_kv_gather(const void* kv_pool, const qtts_paged_state* st, int layers, int kv_heads,
                   int head_dim, int slot, int n_tokens, void* out, qtts_stream_t stream);

/* ========================================================================
 * Kernels (each replaces a piece of the fused TensorRT graph)
 * ======================================================================== */

/* Epilogues of the tcgen05 GEMM  Y[M,N] = X[M,K] · W[N,K]^T  (bf16 in, fp32 accumulate). */
#define QTTS_EPI_BF16      0  /* out bf16 [M,N] (+ bias)                                   */
#define QTTS_EPI_F32       1  /* out fp32 [M,N] (+ bias)                                   */
#define QTTS_EPI_RESIDUAL  2  /* resid fp32 [M,N] += Y            (talker_unified_modules.py:222, 227) */
#define QTTS_EPI_SWIGLU    3  /* out bf16 [M,N/2] = silu(gate)*up, W rows tile-interleaved by 64 */
#define QTTS_EPI_QKV_ROPE  4  /* per-head RMSNorm of q/k, RoPE, q -> out, k/v -> paged pool  */

typedef struct qtts_qkv_epilogue {
    int32_t num_heads, kv_heads, head_dim;
    const void* q_norm_w;        /* bf16 [head_dim] */
    const void* k_norm_w;        /* bf16 [head_dim] */
    float rms_eps;
    const float* rope_cos;       /* [max_pos][head_dim/2] */
    const float* rope_sin;
    int32_t max_pos;
    const int32_t* row_pos;      /* [M] RoPE position of each row */
    const int32_t* slot_mapping; /* [M] block*block_size+offset, -1 = do not store */
    void* kv_pool;               /* [num_blocks][layers][2][kv_heads][block_size][head_dim] fp16 */
    int32_t layer, num_layers, block_size;
} qtts_qkv_epilogue;

/* X: [M,K] bf16 row-major, W: [N,K] bf16 row-major.  N % 128 == 0, K % 64 == 0.
 * X_lo (optional, same shape): bf16 residual of the activation, X ~ X + X_lo; the kernel
 * accumulates W·X + W·X_lo in one pass over the weights.  out/resid per epilogue
 * (QKV_ROPE: q out is fp32 [M][num_heads*head_dim]); out_lo (optional, SwiGLU) receives
 * the bf16 residual of the output.  bias may be NULL (bf16 [N]).  Split-K runs as a
 * thread-block cluster reduced through distributed shared memory (no global workspace). */
int qtts_gemm(const void* X, const void* X_lo, int M, int K, const void* W, int N, int epilogue,
              void* out, void* out_lo, const void* bias, const qtts_qkv_epilogue* qkv,
              qtts_stream_t stream);

/* RMSNorm rows of fp32 x [M,H] (row stride ld) -> bf16 y [M,H]  (Qwen3RMSNorm);
 * y_lo (optional) receives bf16(y_exact - y), the lo half of a GEMM operand. */
int qtts_rmsnorm(const float* x, int M, int H, int ld, const void* w, float eps, void* y, void* y_lo,
                 qtts_stream_t stream);

/* Paged GQA attention for R query rows (decode: one row per stream; chunked prefill:
 * one row per new token).  q: [R][num_heads][head_dim] fp32, row_slot[R] selects the
 * block table row, row_ctx[R] keys visible to the row.  out: [R][num_heads*head_dim] bf16,
 * out_lo (optional): its bf16 residual (lo half of the next GEMM's operand).
 * Scratch: partial results for the split-KV reduction, allocated by the caller:
 * ws_o [R*num_heads*max_splits*head_dim] fp32, ws_ml [R*num_heads*max_splits*2] fp32,
 * with max_splits = ceil(max_ctx / (16*split_blocks)); split_blocks = KV blocks per split
 * (0 = QTTS_ATTN_SPLIT_BLOCKS; fewer blocks per split shorten each warp's chain of copies
 * at the cost of more partials).
 * (talker_unified_modules.py:159-201 with the padded bias of batch_helper.py:48-66.) */
#define QTTS_ATTN_SPLIT_BLOCKS 16
int qtts_paged_attention(const void* q, int R, int num_heads, int kv_heads, int head_dim,
                         const void* kv_pool, int layer, int num_layers, int block_size, int num_blocks,
                         const int32_t* block_table, int max_blocks_per_seq,
                         const int32_t* row_slot, const int32_t* row_ctx, int max_ctx, int split_blocks,
                         float* ws_o, float* ws_ml, void* out, void* out_lo, qtts_stream_t stream);

/* Chunked-prefill form of qtts_paged_attention (head_dim 128): the R rows are R / rows_per_stream
 * streams of rows_per_stream consecutive query tokens (row_slot equal within a stream, row_ctx
 * each token's visible keys: its stream's earlier KV plus the chunk up to itself — the causal
 * mask of talker_unified_modules.py:282-294).  With two query heads per KV head, groups of 64
 * queries x 2 heads run as 128-row tcgen05 tiles that read every KV block once; when those tiles
 * are few, a group's keys are split over several CTAs whose partials go to ws_o / ws_ml (up to
 * the max_splits the scratch sizes allow) and are folded by a second kernel.  Other head layouts
 * use 8-query mma.sync tiles.  Same output and scratch as qtts_paged_attention (executor.py:
 * 759-877 runs this attention inside its fused prefill).  q, out and out_lo must be 16-byte
 * aligned for the tcgen05 form (otherwise the 8-query tiles run). */
int qtts_paged_attention_prefill(const void* q, int R, int rows_per_stream, int num_heads, int kv_heads,
                                 int head_dim, const void* kv_pool, int layer, int num_layers, int block_size,
                                 int num_blocks, const int32_t* block_table, int max_blocks_per_seq,
                                 const int32_t* row_slot, const int32_t* row_ctx, int max_ctx, int split_blocks,
                                 float* ws_o, float* ws_ml, void* out, void* out_lo, qtts_stream_t stream);

/* Same computation as qtts_paged_attention, for callers that cannot allocate device memory
 * when they run attention (a plugin host that owns every allocation and passes only the
 * call's tensors, or a latency-bound thread that must not call cudaMalloc).  No counterpart
 * in the reference.  The split-KV partials live in a static device array of the library
 * (4.25 MiB, held on every GPU that loads it), so nothing is allocated; shapes with
 * num_rows * num_heads * max_splits * head_dim > 1048576 are rejected with QTTS_ERR_INVALID
 * (every head_dim the kernels take, 32 to 128, fits up to that limit).
 * The first call on a device looks up the array's address; make that call before any stream
 * capture.  The address is kept for the life of the process, so cudaDeviceReset followed by
 * more calls on that device is not supported.  Calls share the array: two calls that overlap
 * on the GPU race. */
int qtts_paged_attention_noalloc(const void* q, int R, int num_heads, int kv_heads, int head_dim,
                                 const void* kv_pool, int layer, int num_layers, int block_size,
                                 int num_blocks, const int32_t* block_table, int max_blocks_per_seq,
                                 const int32_t* row_slot, const int32_t* row_ctx, int max_ctx,
                                 void* out, void* out_lo, qtts_stream_t stream);

/* Top-k / temperature / Gumbel-max sampling of fp32 logits [R][V] (row stride ld).
 * Talker head (talker_unified_modules.py:373-388) when counts != NULL: suppress
 * [V-1024,V) except eos_id, repetition penalty on counts>0, counts[tok] += 1.
 * Code predictor (utils.py:986-1001) when counts == NULL.  gumbel [R][topk] fp32;
 * when NULL, noise is Philox4x32-10 keyed by (seed, noise_key[r], step, j).
 * temperature/penalty: per row fp32 or NULL (1.0).  tok_out: int64 [R] (row stride tok_ld). */
int qtts_sample(const float* logits, int R, int V, int ld, int topk, const float* gumbel,
                int gumbel_ld, uint64_t seed, const int64_t* noise_key, int step,
                const float* temperature, const float* penalty, int64_t* counts, int eos_id,
                int64_t* tok_out, int tok_ld, qtts_stream_t stream);

/* The sampling noise the library draws in-kernel, written out: out[r][j] (fp32 [R][cols]) =
 * -log(-log(clamp(u, 1e-8, 1))) with u from Philox4x32-10 keyed by (seed, keys[r],
 * 16 * frames[r] + stage, j); stage 0 = talker head, 1 + s = code-predictor stage s.
 * keys int64 [R], frames int32 [R] (the per-slot key and frame counter of the engine step).
 * Replaces, for inspection and parity, the per-slot noise tensors the reference builds on the
 * host (engine/backend/executor.py:1229-1253). */
int qtts_philox_gumbel(uint64_t seed, const int64_t* keys, const int32_t* frames, int stage, int R, int cols,
                       float* out, qtts_stream_t stream);

/* Codec embedding sum (scripts/python/codec_embedding_sum.py:71-83):
 * out[r] = bf16round(Σ_g T_g[codes[r][g]] + text_add[r]) as fp32 [R][H];
 * T_0 = talker_table [V0][H], T_g = cp_tables[g-1] [Vc][H] (bf16), codes int64 [R][G].
 * text_add fp32 [R][H] or NULL.  codec_sum_out (fp32 [R][H]) may be NULL. */
int qtts_codec_sum(const int64_t* codes, int R, int G, const void* talker_table, int V0,
                   const void* cp_tables, int Vc, int H, const float* text_add,
                   float* codec_sum_out, float* next_x, qtts_stream_t stream);

/* ========================================================================
 * Whole decode step (talker 28 layers + sampling + 15-stage code predictor +
 * codec sum) — the unit of TalkerUnifiedFusedONNX.forward
 * (talker_unified_modules.py:357-401) behind Executor.launch_decode_step.
 * ======================================================================== */
typedef struct qtts_model_desc {
    /* talker */
    int32_t layers, hidden, heads, kv_heads, head_dim, inter, vocab, eos_id, topk;
    float rms_eps;
    const void* w_qkv;        /* [layers][(heads+2*kv_heads)*head_dim][hidden]          */
    const void* w_o;          /* [layers][hidden][heads*head_dim]                        */
    const void* w_gate_up;    /* [layers][2*inter][hidden], 64-row interleave gate/up    */
    const void* w_down;       /* [layers][hidden][inter]                                 */
    const void* w_in_norm;    /* [layers][hidden]                                        */
    const void* w_post_norm;  /* [layers][hidden]                                        */
    const void* w_q_norm;     /* [layers][head_dim]                                      */
    const void* w_k_norm;     /* [layers][head_dim]                                      */
    const void* w_final_norm; /* [hidden]                                                */
    const void* w_codec_head; /* [vocab][hidden]                                         */
    const void* w_codec_emb;  /* [vocab][hidden]                                         */
    const float* rope_cos;    /* [max_pos][head_dim/2]                                   */
    const float* rope_sin;
    int32_t max_pos;
    /* code predictor */
    int32_t cp_layers, cp_hidden, cp_heads, cp_kv_heads, cp_head_dim, cp_inter, cp_vocab, cp_stages;
    float cp_rms_eps;
    const void* cp_w_proj;      /* [cp_hidden][hidden]  */
    const void* cp_b_proj;      /* [cp_hidden]          */
    const void* cp_w_qkv;       /* [cp_layers][(cp_heads+2*cp_kv_heads)*cp_head_dim][cp_hidden] */
    const void* cp_w_o;
    const void* cp_w_gate_up;
    const void* cp_w_down;
    const void* cp_w_in_norm;
    const void* cp_w_post_norm;
    const void* cp_w_q_norm;
    const void* cp_w_k_norm;
    const void* cp_w_final_norm;
    const void* cp_w_lm_head;   /* [cp_stages][cp_vocab][cp_hidden] */
    const void* cp_w_codec_emb; /* [cp_stages][cp_vocab][hidden]    */
    const float* cp_rope_cos;   /* [cp_stages+1][cp_head_dim/2] */
    const float* cp_rope_sin;
    /* pools and limits */
    qtts_paged_state pool;
    void* kv_pool;              /* talker KV blocks */
    int32_t max_batch;          /* rows per step */
    int32_t max_prefill_rows;   /* rows per prefill call */
} qtts_model_desc;

typedef struct qtts_engine qtts_engine;

int qtts_engine_create(const qtts_model_desc* desc, qtts_engine** out);
int qtts_engine_destroy(qtts_engine* e);

/* One step over n_rows rows.  For decode n_new = 1 and rows are streams; for
 * chunked prefill of a single stream n_rows = 1 and n_new = S.
 *   slots [n_rows] int32 (device), x_in fp32 [n_rows*n_new][hidden] (input embeddings,
 *   bf16-rounded like executor.py:1096), token_counts int64 [n_rows][vocab] (updated in place),
 *   gumbel fp32 [n_rows][topk] or NULL, cp_gumbel fp32 [n_rows][cp_stages][topk] or NULL,
 *   noise_seed/noise_key/noise_step (or step) for in-kernel Philox noise when the gumbel pointers are
 *   NULL: the counter of a row is noise_step[row] when given (incremented by each sampled step, so
 *   a stream's noise sequence does not depend on batching, like the per-slot generator of
 *   executor.py:1212-1227), else step; temperature/penalty fp32 [n_rows] (NULL = 1.0);
 *   sample: 0 = skip sampling/CP (prefix-only prefill).  With slot_indexed, noise_key, noise_step,
 *   temperature and penalty are per pool slot too.
 * Outputs (device): hidden bf16 [n_rows][hidden] (last new token), logits fp32 [n_rows][vocab],
 *   full_codec int64 [n_rows][1+cp_stages], codec_sum fp32 [n_rows][hidden],
 *   next_x fp32 [n_rows][hidden] = bf16round(codec_sum + text_add) (text_add fp32 [n_rows][hidden] or NULL),
 *   status int32 [1] (device; scheduler errors).  The KV of the new tokens is written to the pool. */
typedef struct qtts_step_io {
    const int32_t* slots;
    int32_t n_rows;
    int32_t n_new;
    int32_t slot_indexed;   /* 1: token_counts, text_add, codec_sum_out, next_x_out (and x_in when
                               n_new == 1) hold one row per pool slot and row r uses slots[r] */
    const float* x_in;
    int64_t* token_counts;
    const float* gumbel;
    const float* cp_gumbel;
    uint64_t noise_seed;
    const int64_t* noise_key;
    int32_t* noise_step;
    int32_t step;
    const float* temperature;
    const float* penalty;
    int32_t sample;
    const float* text_add;
    void* hidden_out;
    float* logits_out;
    int64_t* full_codec_out;
    float* codec_sum_out;
    float* next_x_out;
    int32_t* status;
    /* parity hooks (NULL in production): force_codes int64 [n_rows][1+cp_stages] makes the code
     * predictor consume these tokens instead of the sampled ones (teacher forcing; the sampled
     * tokens are still written to full_codec_out); cp_logits_out fp32 [n_rows][cp_stages][cp_vocab]
     * receives every stage's logits.  Like the reference's debug-dump hook points
     * (engine/backend/debug_dump.py:112-175), they exist to compare intermediate tensors. */
    const int64_t* force_codes;
    float* cp_logits_out;
    int32_t launches;   /* out (host): kernels this call enqueued */
} qtts_step_io;

int qtts_engine_step(qtts_engine* e, qtts_step_io* io, qtts_stream_t stream);

/* ---------------------------------------------------------------------------
 * Streaming code2wav decoder.  Replaces Code2WavStreamingWrapper.forward
 * (scripts/export/code2wav_streaming.py:708-810) as the fused graph runs it
 * at T = 1 frame per step (export_09_talker_code2wav_fused.py:145-160): codes
 * clamped to [0, codebook_size) -> RVQ tables -> causal pre_conv (k3) -> window
 * transformer -> 2 x [transposed conv x2 + ConvNeXt] -> conv k7 -> 4 x
 * [SnakeBeta, transposed conv (2s, s), 3 residual units k7 d1/3/9] -> SnakeBeta
 * -> conv k7 -> clamp(-1, 1).  The streaming state (window KV, conv left
 * contexts, transposed-conv overlaps, frame counter) lives on the device,
 * indexed by pool slot; the transposed-conv overlap is kept as the previous
 * input frame, from which the reference's bias-free overlap tail
 * (code2wav_streaming.py:118-124) is recomputed inside the GEMM.
 *
 * Weights are packed by the host (test_stateful_b200/runtime/code2wav.py):
 * bf16 unless noted; GEMM weights [N_pad][K_pad] zero-padded to N % 128 == 0
 * and K % 64 == 0; a conv [out][in][k] becomes [out][k*in] (tap-major); a
 * transposed conv (stride s, kernel 2s) becomes rows (phase p, out channel)
 * over [x(i-1) | x(i)] with taps w[:, :, p+s] and w[:, :, p]. */
typedef struct qtts_c2w_desc {
    int32_t num_codebooks, codebook_size, codebook_dim, latent, hidden, layers, heads, head_dim, inter;
    int32_t window, decoder_dim, convnext_dim, max_slots, max_frames;
    int32_t max_chunk;            /* frames per stream per qtts_c2w_step call, at most (0 = 1) */
    int32_t up_ratio[2];
    int32_t rates[4];
    int32_t dilations[3];
    float rms_eps, ln_eps;
    const float* rvq_tables;      /* fp32 [num_codebooks][codebook_size][codebook_dim]: codebook rows
                                     through output_proj, both biases folded into tables 0 and 1 */
    const void* w_pre_conv;       /* [latent][pad64(3*codebook_dim)] */
    const void* b_pre_conv;       /* [latent] */
    const void* w_in_proj;        /* [hidden][latent] */
    const void* b_in_proj;
    const void* w_in_norm;        /* [layers][hidden] */
    const void* w_qkv;            /* [layers][3*heads*head_dim][hidden] */
    const void* w_q_norm;         /* [layers][head_dim] */
    const void* w_k_norm;
    const void* w_o;              /* [layers][hidden][heads*head_dim] */
    const void* attn_scale;       /* [layers][hidden] layer scale */
    const void* w_post_norm;
    const void* w_gate_up;        /* [layers][2*inter][hidden], 64-row interleave gate/up */
    const void* w_down;           /* [layers][hidden][inter] */
    const void* mlp_scale;        /* [layers][hidden] */
    const void* w_final_norm;     /* [hidden] */
    const void* w_out_proj;       /* [latent][hidden] */
    const void* b_out_proj;
    const float* rope_cos;        /* [max_frames][head_dim/2] (theta of the decoder) */
    const float* rope_sin;
    const void* up_w[2];          /* [2*latent][latent] (phase-major rows) */
    const void* up_b[2];          /* [2*latent] */
    const float* dw_w[2];         /* fp32 [latent][7] depthwise */
    const float* dw_b[2];
    const float* ln_w[2];         /* fp32 [latent] */
    const float* ln_b[2];
    const void* pw1_w[2];         /* [convnext_dim][latent] */
    const void* pw1_b[2];
    const void* pw2_w[2];         /* [latent][convnext_dim] */
    const void* pw2_b[2];
    const void* gamma[2];         /* [latent] */
    const void* w_conv0;          /* [decoder_dim][7*latent] */
    const void* b_conv0;
    const float* blk_snake[4];    /* fp32 [2][cin]: exp(alpha), exp(-beta) */
    const void* blk_tw[4];        /* [pad128(s*cout)][2*cinp] (K padded to 64); cinp = pad64(cin) when the
                                     block's transposed conv is implicit (below), else cin */
    const void* blk_tb[4];        /* [pad128(s*cout)] */
    const float* res_act1[4][3];  /* fp32 [2][cout] */
    const float* res_act2[4][3];
    const void* res_w1[4][3];     /* [pad128(cout)][7*coutp] (K padded to 64); coutp = pad64(cout) when the
                                     block's residual convs are implicit, else cout.  A conv with T input
                                     rows per frame is implicit when T % 128 == 0, or when
                                     R = max_chunk * T >= 512 and padding R to a multiple of 128 adds at
                                     most R / 8 rows */
    const void* res_b1[4][3];     /* [pad128(cout)] */
    const void* res_w2[4][3];     /* [pad128(cout)][pad128(cout)] */
    const void* res_b2[4][3];
    const float* final_snake;     /* fp32 [2][cout of block 3] */
    const float* final_w;         /* fp32 [7][cout of block 3] (tap-major) */
    float final_b;
} qtts_c2w_desc;

typedef struct qtts_c2w qtts_c2w;

int qtts_c2w_create(const qtts_c2w_desc* desc, qtts_c2w** out);
int qtts_c2w_destroy(qtts_c2w* c);
/* Zero the streaming state of n slots (device int32 [n]): a new stream starts at frame 0. */
int qtts_c2w_reset(qtts_c2w* c, const int32_t* slots, int n, qtts_stream_t stream);
/* `frames` consecutive frames (1 <= frames <= max_chunk) for each of n streams:
 * codes int64 (device) [n][frames][codes_ld] (first num_codebooks used), slots int32 (device) [n]
 * (distinct), wav fp32 (device) [n][frames * samples_per_frame].  A chunk of F frames sees at
 * most window - F past frames plus its own frames causally (the reference caller's crop of the
 * window cache to window - chunk, engine/backend/executor.py:1374-1380); frames = 1 is the
 * fused step's streaming decode (export_09_talker_code2wav_fused.py:145-160). */
int qtts_c2w_step(qtts_c2w* c, const int64_t* codes, int codes_ld, int frames, const int32_t* slots, int n,
                  float* wav, qtts_stream_t stream);
/* Kernels the last qtts_c2w_step enqueued (host counter). */
int qtts_c2w_launches(const qtts_c2w* c);
/* background != 0: the decoder's steps run beside a latency-critical stream (the executor runs
 * step t's code2wav while step t+1's talker runs), so its kernels launch without programmatic
 * dependent launch: a waiting kernel's CTAs would otherwise hold SMs the other stream needs.
 * Default 0.  No counterpart in the reference (its code2wav is inside the fused plan). */
int qtts_c2w_set_background(qtts_c2w* c, int background);

/* Streaming state of one slot in this decoder's own layout, for installing a warm state
 * (Executor.apply_c2w_warm_state, engine/backend/executor.py:715-757; the reference's state is
 * the wrapper's 2*layers KV + 17 conv + 4 transposed-conv tensors,
 * scripts/export/code2wav_streaming.py:159-193).  Part 0 is the attention window
 * [layers][2 (k, v)][heads][window][head_dim] fp16 (frame f at window position f % window, its
 * key RoPE-rotated at position f); parts 1..17 are the causal convolutions' left contexts in the
 * reference's order (conv_state_0..16: [ctx rows][channels], the activated conv inputs); parts
 * 18..21 the transposed convolutions' previous input row (one row of the block's activated
 * input: this decoder keeps x(i-1) where the reference keeps the bias-free overlap tail
 * W[:, :, s:] x(i-1)).  A part is `rows` rows of `row_elems` elements of `dtype` (0 bf16,
 * 1 fp32, 2 fp16), the first `valid_elems` of a row real channels, the rest zero. */
typedef struct qtts_c2w_state_part {
    int32_t rows;
    int32_t row_elems;
    int32_t valid_elems;
    int32_t dtype;
} qtts_c2w_state_part;
#define QTTS_C2W_STATE_PARTS 22
/* Fills parts[0 .. QTTS_C2W_STATE_PARTS) (max_parts must be at least that). */
int qtts_c2w_state_layout(const qtts_c2w* c, qtts_c2w_state_part* parts, int max_parts);
/* Copy `bytes` (= the part's rows * row_elems * element size) from `src` (device, the part's
 * layout, contiguous) into part `part` of `slot` (0 <= slot < max_slots); stream-ordered. */
int qtts_c2w_write_state(qtts_c2w* c, int slot, int part, const void* src, size_t bytes, qtts_stream_t stream);
/* Set the slot's frame counter (frames decoded so far: the next frame's RoPE position). */
int qtts_c2w_set_frame(qtts_c2w* c, int slot, int frame, qtts_stream_t stream);

#ifdef __cplusplus
}
#endif
#endif /* QTTS_B200_H */
