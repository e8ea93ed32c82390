// The decode-step engine: the launch sequence of one TalkerUnifiedFusedONNX
// forward (talker_unified_modules.py:357-401) over the paged pool, built once
// (tensor maps, buffers, per-stage row tables) and replayed every step.
//
// Step for n_rows streams x n_new tokens (decode: n_new = 1):
//   sched append (+ COW copies) -> 28 x [RMSNorm, QKV GEMM (+q/k norm, RoPE,
//   KV store), paged attention, O GEMM (+residual), RMSNorm, gate/up GEMM
//   (+SwiGLU), down GEMM (+residual)] -> final norm of the last token ->
//   codec head -> sampling -> code predictor: stage 0 over [h_last, emb(tok0)]
//   then 14 single-token stages with a per-step KV cache (one 16-token block
//   per stream) -> codec embedding sum + text embedding -> next input.
//
// The code predictor keeps K/V across its 15 stages instead of recomputing the
// whole sequence each stage as CodePredictorUnrolled does (utils.py:1003-1042);
// attention is causal and positions restart at 0 every frame, so each
// stage's last hidden state is the same function of the same inputs.
#pragma once

#include <vector>

#include "attention.cuh"
#include "common.cuh"
#include "cp_cluster.cuh"
#include "cp_persist.cuh"
#include "gemm_tc.cuh"
#include "sampling.cuh"
#include "sched.cuh"
#include "small_ops.cuh"

namespace qtts {

struct LayerGemms {
    GemmPlan qkv, o, gu, down;
    GemmPlan qkv_pair;  // code predictor: QKV in paired-tile order (persistent program)
};

struct DevBuf {
    void* p = nullptr;
    ~DevBuf() {
        if (p) cudaFree(p);
    }
};

}  // namespace qtts

struct qtts_engine {
    qtts_model_desc d;
    int rmax;        // token rows per call (talker)
    int bmax;        // streams per call
    int qkv_rows, cp_qkv_rows;
    int max_splits, cp_max_splits;
    int attn_split;  // KV blocks per attention split (talker)
    // talker activations
    // GEMM operands are hi/lo bf16 pairs (x_lo = bf16(x - x_hi)), see gemm_tc.cuh
    float* x = nullptr;              // [rmax][H] fp32 residual stream
    __nv_bfloat16 *xn = nullptr, *xn_lo = nullptr;      // [rmax][H] normed x (layer 0) or x∘γ (folded norms)
    float* ss = nullptr;                                // [rmax][H/128] folded-norm partial sums of x²
    float* qbuf = nullptr;                              // [rmax][Hq*D] fp32 q after norm + RoPE
    __nv_bfloat16 *attn = nullptr, *attn_lo = nullptr;  // [rmax][Hq*D]
    __nv_bfloat16 *act = nullptr, *act_lo = nullptr;    // [rmax][I] SwiGLU output
    __nv_bfloat16 *hid = nullptr, *hid_lo = nullptr;    // [bmax][H] final-normed last token
    float* ws_o = nullptr;
    float* ws_ml = nullptr;
    int32_t *mapping = nullptr, *row_ctx = nullptr, *row_pos = nullptr, *row_slot = nullptr;
    int32_t *cow_src = nullptr, *cow_dst = nullptr;
    // code predictor
    __nv_bfloat16 *cp_in = nullptr, *cp_in_lo = nullptr;  // [2*bmax][H]
    float* cx = nullptr;                                  // [2*bmax][cpH]
    __nv_bfloat16 *cxn = nullptr, *cxn_lo = nullptr;      // [2*bmax][cpH] x∘γ of the folded norms
    float* css = nullptr;                                 // [2*bmax][cpH/128]
    float* cq = nullptr;
    __nv_bfloat16 *cattn = nullptr, *cattn_lo = nullptr;
    __nv_bfloat16 *cact = nullptr, *cact_lo = nullptr;
    __nv_bfloat16 *chid = nullptr, *chid_lo = nullptr;    // [bmax][cpH]
    float* clogits = nullptr;        // [bmax][cp_vocab]
    qtts::kv_t* cp_kv = nullptr;           // [bmax][cpL][2][cpHkv][16][cpD]
    float* cws_o = nullptr;
    float* cws_ml = nullptr;
    int32_t* cp_meta = nullptr;      // per stage: mapping, pos, ctx, slot  [stages][4][2*bmax]
    int32_t* cp_table = nullptr;     // identity block table [bmax]
    std::vector<void*> allocs;
    // plans (built for rmax / 2*bmax rows; M is set per call)
    std::vector<qtts::LayerGemms> tg;
    qtts::GemmPlan head;
    std::vector<qtts::LayerGemms> cg;
    qtts::GemmPlan cp_proj_pair;
    float* cp_tab = nullptr;  // [cp_stages - 1][cp_vocab][cH]: stage embeddings through the projection
    __nv_bfloat16* cp_qkv_pair = nullptr;  // code-predictor QKV rows in paired-tile order (PairAttn)
    bool cp_pair = false;
    // code-predictor stages >= 1 as one cluster kernel each (cp_cluster.cuh): weights packed
    // in mma.sync fragment order
    bool cp_cluster = false;
    uint4 *cpc_qkv = nullptr, *cpc_o = nullptr, *cpc_gu = nullptr, *cpc_down = nullptr, *cpc_head = nullptr;
    std::vector<qtts::GemmPlan> cp_heads;
    // code-predictor stages >= 1 as one persistent launch each (cp_persist.cuh): per stage a
    // program of cpp_phases GEMM phases, and the grid barrier's two counters
    bool cp_persist = false;
    qtts::CpPhase* cpp_prog = nullptr;
    int cpp_phases = 0;
    unsigned* cpp_bar = nullptr;
};

namespace qtts {

template <class T>
inline int dev_alloc(qtts_engine* e, T** p, size_t count) {
    void* ptr = nullptr;
    QTTS_CHECK_CUDA(cudaMalloc(&ptr, count * sizeof(T) + 256));
    e->allocs.push_back(ptr);
    *p = reinterpret_cast<T*>(ptr);
    return QTTS_OK;
}

#define QTTS_TRY(x)               \
    do {                          \
        int _rc = (x);            \
        if (_rc != QTTS_OK) return _rc; \
    } while (0)

inline const __nv_bfloat16* bf(const void* p, size_t off) { return reinterpret_cast<const __nv_bfloat16*>(p) + off; }

// Fold an RMSNorm between two GEMMs: `prod` (F32 / RESIDUAL epilogue writing x) also
// emits x∘γ as the hi/lo operand and the per-tile sums of x²; `cons` reads them.
inline void fold_norm_out(GemmPlan& prod, const __nv_bfloat16* gamma, __nv_bfloat16* hi, __nv_bfloat16* lo,
                          float* ss) {
    prod.p.nout.gamma = gamma;
    prod.p.nout.hi = hi;
    prod.p.nout.lo = lo;
    prod.p.nout.ss = ss;
}
inline void fold_norm_in(GemmPlan& cons, const float* ss, int hidden, float eps) {
    cons.p.nin.ss = ss;
    cons.p.nin.parts = hidden / 128;
    cons.p.nin.K = hidden;
    cons.p.nin.eps = eps;
}

inline int engine_build(qtts_engine* e) {
    const qtts_model_desc& d = e->d;
    const int H = d.hidden, D = d.head_dim, Hq = d.heads, Hkv = d.kv_heads, I = d.inter;
    e->bmax = d.max_batch;
    e->rmax = d.max_batch > d.max_prefill_rows ? d.max_batch : d.max_prefill_rows;
    e->qkv_rows = (Hq + 2 * Hkv) * D;
    const int max_ctx = d.pool.max_blocks_per_seq * d.pool.block_size;
    e->attn_split = attn_engine_split();
    e->max_splits = attn_max_splits(max_ctx, e->attn_split);
    const int rmax = e->rmax, bmax = e->bmax;
    QTTS_TRY(dev_alloc(e, &e->x, (size_t)rmax * H));
    QTTS_TRY(dev_alloc(e, &e->xn, (size_t)rmax * H));
    QTTS_TRY(dev_alloc(e, &e->xn_lo, (size_t)rmax * H));
    QTTS_TRY(dev_alloc(e, &e->ss, (size_t)rmax * (H / 128)));
    QTTS_TRY(dev_alloc(e, &e->qbuf, (size_t)rmax * Hq * D));
    QTTS_TRY(dev_alloc(e, &e->attn, (size_t)rmax * Hq * D));
    QTTS_TRY(dev_alloc(e, &e->attn_lo, (size_t)rmax * Hq * D));
    QTTS_TRY(dev_alloc(e, &e->act, (size_t)rmax * I));
    QTTS_TRY(dev_alloc(e, &e->act_lo, (size_t)rmax * I));
    QTTS_TRY(dev_alloc(e, &e->hid, (size_t)bmax * H));
    QTTS_TRY(dev_alloc(e, &e->hid_lo, (size_t)bmax * H));
    QTTS_TRY(dev_alloc(e, &e->ws_o, (size_t)rmax * Hq * e->max_splits * D));
    QTTS_TRY(dev_alloc(e, &e->ws_ml, (size_t)rmax * Hq * e->max_splits * 2));
    QTTS_TRY(dev_alloc(e, &e->mapping, (size_t)rmax));
    QTTS_TRY(dev_alloc(e, &e->row_ctx, (size_t)rmax));
    QTTS_TRY(dev_alloc(e, &e->row_pos, (size_t)rmax));
    QTTS_TRY(dev_alloc(e, &e->row_slot, (size_t)rmax));
    QTTS_TRY(dev_alloc(e, &e->cow_src, (size_t)rmax));
    QTTS_TRY(dev_alloc(e, &e->cow_dst, (size_t)rmax));

    // ---- talker GEMM plans
    e->tg.resize(d.layers);
    for (int l = 0; l < d.layers; ++l) {
        LayerGemms& g = e->tg[l];
        qtts_qkv_epilogue q = {};
        q.num_heads = Hq;
        q.kv_heads = Hkv;
        q.head_dim = D;
        q.q_norm_w = bf(d.w_q_norm, (size_t)l * D);
        q.k_norm_w = bf(d.w_k_norm, (size_t)l * D);
        q.rms_eps = d.rms_eps;
        q.rope_cos = d.rope_cos;
        q.rope_sin = d.rope_sin;
        q.max_pos = d.max_pos;
        q.row_pos = e->row_pos;
        q.slot_mapping = e->mapping;
        q.kv_pool = d.kv_pool;
        q.layer = l;
        q.num_layers = d.layers;
        q.block_size = d.pool.block_size;
        QTTS_TRY(gemm_plan(&g.qkv, e->xn, rmax, H, bf(d.w_qkv, (size_t)l * e->qkv_rows * H), e->qkv_rows,
                           QTTS_EPI_QKV_ROPE, e->qbuf, nullptr, &q, e->xn_lo));
        QTTS_TRY(gemm_plan(&g.o, e->attn, rmax, Hq * D, bf(d.w_o, (size_t)l * H * Hq * D), H, QTTS_EPI_RESIDUAL,
                           e->x, nullptr, nullptr, e->attn_lo));
        QTTS_TRY(gemm_plan(&g.gu, e->xn, rmax, H, bf(d.w_gate_up, (size_t)l * 2 * I * H), 2 * I, QTTS_EPI_SWIGLU,
                           e->act, nullptr, nullptr, e->xn_lo, e->act_lo));
        QTTS_TRY(gemm_plan(&g.down, e->act, rmax, I, bf(d.w_down, (size_t)l * H * I), H, QTTS_EPI_RESIDUAL, e->x,
                           nullptr, nullptr, e->act_lo));
        // post-attention norm folded into o-proj -> gate/up; the next layer's input
        // norm into down -> next qkv (layer 0's input norm stays a kernel)
        fold_norm_out(g.o, bf(d.w_post_norm, (size_t)l * H), e->xn, e->xn_lo, e->ss);
        fold_norm_in(g.gu, e->ss, H, d.rms_eps);
        if (l > 0) fold_norm_in(g.qkv, e->ss, H, d.rms_eps);
        if (l + 1 < d.layers) fold_norm_out(g.down, bf(d.w_in_norm, (size_t)(l + 1) * H), e->xn, e->xn_lo, e->ss);
    }
    QTTS_TRY(dev_alloc(e, &e->cp_table, (size_t)bmax));
    // ---- code predictor
    const int cH = d.cp_hidden, cD = d.cp_head_dim, cHq = d.cp_heads, cHkv = d.cp_kv_heads, cI = d.cp_inter;
    const int S = d.cp_stages;
    e->cp_qkv_rows = (cHq + 2 * cHkv) * cD;
    e->cp_max_splits = 1;
    const int crows = 2 * bmax;
    QTTS_TRY(dev_alloc(e, &e->cp_in, (size_t)crows * H));
    QTTS_TRY(dev_alloc(e, &e->cp_in_lo, (size_t)crows * H));
    QTTS_TRY(dev_alloc(e, &e->cx, (size_t)crows * cH));
    QTTS_TRY(dev_alloc(e, &e->cxn, (size_t)crows * cH));
    QTTS_TRY(dev_alloc(e, &e->cxn_lo, (size_t)crows * cH));
    QTTS_TRY(dev_alloc(e, &e->css, (size_t)crows * (cH / 128)));
    QTTS_TRY(dev_alloc(e, &e->cq, (size_t)crows * cHq * cD));
    QTTS_TRY(dev_alloc(e, &e->cattn, (size_t)crows * cHq * cD));
    QTTS_TRY(dev_alloc(e, &e->cattn_lo, (size_t)crows * cHq * cD));
    QTTS_TRY(dev_alloc(e, &e->cact, (size_t)crows * cI));
    QTTS_TRY(dev_alloc(e, &e->cact_lo, (size_t)crows * cI));
    QTTS_TRY(dev_alloc(e, &e->chid, (size_t)bmax * cH));
    QTTS_TRY(dev_alloc(e, &e->chid_lo, (size_t)bmax * cH));
    QTTS_TRY(dev_alloc(e, &e->clogits, (size_t)bmax * d.cp_vocab));
    QTTS_TRY(dev_alloc(e, &e->cp_kv, (size_t)bmax * d.cp_layers * 2 * cHkv * 16 * cD));
    QTTS_TRY(dev_alloc(e, &e->cws_o, (size_t)crows * cHq * cD));
    QTTS_TRY(dev_alloc(e, &e->cws_ml, (size_t)crows * cHq * 2));
    QTTS_TRY(dev_alloc(e, &e->cp_meta, (size_t)S * 4 * crows));
    // every stage's rows: stage 0 has rows 2b+p (p = 0: talker hidden, 1: emb(tok0)),
    // stage s >= 1 has one row per stream at position s+1.
    {
        std::vector<int32_t> meta((size_t)S * 4 * crows, 0), table(bmax);
        for (int b = 0; b < bmax; ++b) table[b] = b;
        for (int s = 0; s < S; ++s) {
            int32_t* m = meta.data() + (size_t)s * 4 * crows;
            if (s == 0) {
                for (int b = 0; b < bmax; ++b)
                    for (int p = 0; p < 2; ++p) {
                        const int r = 2 * b + p;
                        m[r] = b * 16 + p;
                        m[crows + r] = p;
                        m[2 * crows + r] = p + 1;
                        m[3 * crows + r] = b;
                    }
            } else {
                for (int b = 0; b < bmax; ++b) {
                    m[b] = b * 16 + s + 1;
                    m[crows + b] = s + 1;
                    m[2 * crows + b] = s + 2;
                    m[3 * crows + b] = b;
                }
            }
        }
        QTTS_CHECK_CUDA(cudaMemcpy(e->cp_meta, meta.data(), meta.size() * 4, cudaMemcpyHostToDevice));
        QTTS_CHECK_CUDA(cudaMemcpy(e->cp_table, table.data(), table.size() * 4, cudaMemcpyHostToDevice));
    }
    // Opt-in (QTTS_CP_PAIR=1): paired QKV tiles with the decode attention fused into the QKV
    // GEMM (head_dim 64, two query heads per KV head).  Measured about 1 % slower on the decode
    // step than QKV GEMM + short_attn_kernel (9 998 vs 10 112 frames/s with 16-CTA clusters,
    // 9 598 with 8-CTA clusters and 4-way split-K).
    {
        const char* v = getenv("QTTS_CP_PAIR");
        e->cp_pair = cD == 64 && cHq == 2 * cHkv && v && *v == '1';
        // Opt-in (QTTS_CP_PERSIST=1): stages >= 1 as one persistent launch (paired QKV tiles).
        const char* w = getenv("QTTS_CP_PERSIST");
        e->cp_persist = cD == 64 && cHq == 2 * cHkv && S > 1 && w && *w == '1' && cp_persist_clusters() > 0;
        if (e->cp_pair || e->cp_persist)
            QTTS_TRY(dev_alloc(e, &e->cp_qkv_pair, (size_t)d.cp_layers * e->cp_qkv_rows * cH));
    }
    e->cg.resize(d.cp_layers);
    for (int l = 0; l < d.cp_layers; ++l) {
        LayerGemms& g = e->cg[l];
        qtts_qkv_epilogue q = {};
        q.num_heads = cHq;
        q.kv_heads = cHkv;
        q.head_dim = cD;
        q.q_norm_w = bf(d.cp_w_q_norm, (size_t)l * cD);
        q.k_norm_w = bf(d.cp_w_k_norm, (size_t)l * cD);
        q.rms_eps = d.cp_rms_eps;
        q.rope_cos = d.cp_rope_cos;
        q.rope_sin = d.cp_rope_sin;
        q.max_pos = S + 1;
        q.row_pos = nullptr;       // set per stage
        q.slot_mapping = nullptr;  // set per stage
        q.kv_pool = e->cp_kv;
        q.layer = l;
        q.num_layers = d.cp_layers;
        q.block_size = 16;
        const __nv_bfloat16* wqkv = bf(d.cp_w_qkv, (size_t)l * e->cp_qkv_rows * cH);
        const __nv_bfloat16* wqkv_pair = nullptr;
        if (e->cp_qkv_pair) {
            // rows per KV head g: tile 2g = q heads 2g, 2g+1; tile 2g+1 = k_g, v_g
            __nv_bfloat16* dst = e->cp_qkv_pair + (size_t)l * e->cp_qkv_rows * cH;
            const size_t row = (size_t)cH * sizeof(__nv_bfloat16);
            for (int g2 = 0; g2 < cHkv; ++g2) {
                QTTS_CHECK_CUDA(cudaMemcpy(dst + (size_t)(256 * g2) * cH, wqkv + (size_t)(128 * g2) * cH, 128 * row,
                                           cudaMemcpyDeviceToDevice));
                QTTS_CHECK_CUDA(cudaMemcpy(dst + (size_t)(256 * g2 + 128) * cH,
                                           wqkv + (size_t)(cHq * 64 + 64 * g2) * cH, 64 * row, cudaMemcpyDeviceToDevice));
                QTTS_CHECK_CUDA(cudaMemcpy(dst + (size_t)(256 * g2 + 192) * cH,
                                           wqkv + (size_t)(cHq * 64 + cHkv * 64 + 64 * g2) * cH, 64 * row,
                                           cudaMemcpyDeviceToDevice));
            }
            wqkv_pair = dst;
            if (e->cp_pair) wqkv = dst;
        }
        QTTS_TRY(gemm_plan(&g.qkv, e->cxn, crows, cH, wqkv, e->cp_qkv_rows, QTTS_EPI_QKV_ROPE, e->cq, nullptr, &q,
                           e->cxn_lo));
        if (e->cp_pair) {
            g.qkv.p.pair.on = 1;
            g.qkv.p.pair.out = e->cattn;
            g.qkv.p.pair.out_lo = e->cattn_lo;
            g.qkv.p.pair.scale_log2 = 1.4426950408889634f / sqrtf((float)cD);
        }
        if (wqkv_pair) {
            QTTS_TRY(gemm_plan(&g.qkv_pair, e->cxn, crows, cH, wqkv_pair, e->cp_qkv_rows, QTTS_EPI_QKV_ROPE, e->cq,
                               nullptr, &q, e->cxn_lo));
            g.qkv_pair.p.pair.on = 1;
            g.qkv_pair.p.pair.out = e->cattn;
            g.qkv_pair.p.pair.out_lo = e->cattn_lo;
            g.qkv_pair.p.pair.scale_log2 = 1.4426950408889634f / sqrtf((float)cD);
        }
        QTTS_TRY(gemm_plan(&g.o, e->cattn, crows, cHq * cD, bf(d.cp_w_o, (size_t)l * cH * cHq * cD), cH,
                           QTTS_EPI_RESIDUAL, e->cx, nullptr, nullptr, e->cattn_lo));
        QTTS_TRY(gemm_plan(&g.gu, e->cxn, crows, cH, bf(d.cp_w_gate_up, (size_t)l * 2 * cI * cH), 2 * cI,
                           QTTS_EPI_SWIGLU, e->cact, nullptr, nullptr, e->cxn_lo, e->cact_lo));
        QTTS_TRY(gemm_plan(&g.down, e->cact, crows, cI, bf(d.cp_w_down, (size_t)l * cH * cI), cH, QTTS_EPI_RESIDUAL,
                           e->cx, nullptr, nullptr, e->cact_lo));
        fold_norm_out(g.o, bf(d.cp_w_post_norm, (size_t)l * cH), e->cxn, e->cxn_lo, e->css);
        fold_norm_in(g.gu, e->css, cH, d.cp_rms_eps);
        fold_norm_in(g.qkv, e->css, cH, d.cp_rms_eps);
        if (wqkv_pair) fold_norm_in(g.qkv_pair, e->css, cH, d.cp_rms_eps);
        // the last layer's down projection folds the final norm (used from stage 1 on, where
        // every row is a stream's last position)
        fold_norm_out(g.down, l + 1 < d.cp_layers ? bf(d.cp_w_in_norm, (size_t)(l + 1) * cH) : bf(d.cp_w_final_norm, 0),
                      e->cxn, e->cxn_lo, e->css);
    }
    // stage 0 projects [talker hidden (hi/lo), codec embedding]; later stages only embeddings (exact in bf16)
    QTTS_TRY(gemm_plan(&e->cp_proj_pair, e->cp_in, crows, H, d.cp_w_proj, cH, QTTS_EPI_F32, e->cx, d.cp_b_proj,
                       nullptr, e->cp_in_lo));
    {
        // stages 1..S-1 feed a codec embedding row through the (linear) projection: do it once
        // for every row of their embedding tables
        const int rows = (S - 1) * d.cp_vocab;
        QTTS_TRY(dev_alloc(e, &e->cp_tab, (size_t)rows * cH));
        GemmPlan tab;
        QTTS_TRY(gemm_plan(&tab, d.cp_w_codec_emb, rows, H, d.cp_w_proj, cH, QTTS_EPI_F32, e->cp_tab, d.cp_b_proj,
                           nullptr));
        QTTS_TRY(gemm_run(tab, rows, 0));
        QTTS_CHECK_CUDA(cudaStreamSynchronize(0));
    }
    // the first layer's input norm folded into the projection
    fold_norm_out(e->cp_proj_pair, bf(d.cp_w_in_norm, 0), e->cxn, e->cxn_lo, e->css);
    // Stages >= 1 as one cluster kernel per stage (opt-in: QTTS_CP_CLUSTER=1; the default is the
    // per-GEMM path), for the code predictor's shape (hidden 1024, 16 x 64 heads, 8 kv heads,
    // SwiGLU 3072, 5 layers, 2048-entry heads)
    {
        const char* v = getenv("QTTS_CP_CLUSTER");
        e->cp_cluster = (v && *v == '1') && cH == kCpcH && cI == kCpcI && cHq == kCpcHq && cHkv == kCpcHkv &&
                        cD == kCpcD && d.cp_layers == kCpcL && d.cp_vocab == kCpcV && d.cp_rope_cos != nullptr;
        if (e->cp_cluster) {
            const size_t nq = (size_t)kCpcQkv * cH / 8, no = (size_t)cH * cH / 8, ngu = (size_t)2 * cI * cH / 8,
                         nd = (size_t)cH * cI / 8, nh = (size_t)d.cp_vocab * cH / 8;  // uint4 per matrix
            QTTS_TRY(dev_alloc(e, &e->cpc_qkv, nq * kCpcL));
            QTTS_TRY(dev_alloc(e, &e->cpc_o, no * kCpcL));
            QTTS_TRY(dev_alloc(e, &e->cpc_gu, ngu * kCpcL));
            QTTS_TRY(dev_alloc(e, &e->cpc_down, nd * kCpcL));
            QTTS_TRY(dev_alloc(e, &e->cpc_head, nh * S));
            for (int l = 0; l < kCpcL; ++l) {
                QTTS_TRY(pack_a_frag(bf(d.cp_w_qkv, (size_t)l * kCpcQkv * cH), cH, 0, kCpcQkv, cH, e->cpc_qkv + l * nq, 0));
                QTTS_TRY(pack_a_frag(bf(d.cp_w_o, (size_t)l * cH * cH), cH, 0, cH, cH, e->cpc_o + l * no, 0));
                QTTS_TRY(pack_a_frag(bf(d.cp_w_gate_up, (size_t)l * 2 * cI * cH), cH, 0, 2 * cI, cH,
                                     e->cpc_gu + l * ngu, 0));
                // down: per CTA r the columns (SwiGLU features) [192 r, +192) it computes
                for (int r = 0; r < kCpcCtas; ++r)
                    QTTS_TRY(pack_a_frag(bf(d.cp_w_down, (size_t)l * cH * cI), cI, kCpcFeat * r, cH, kCpcFeat,
                                         e->cpc_down + l * nd + (size_t)r * cH * kCpcFeat / 8, 0));
            }
            for (int st = 0; st < S; ++st)
                QTTS_TRY(pack_a_frag(bf(d.cp_w_lm_head, (size_t)st * d.cp_vocab * cH), cH, 0, d.cp_vocab, cH,
                                     e->cpc_head + st * nh, 0));
            QTTS_CHECK_CUDA(cudaStreamSynchronize(0));
        }
    }
    e->cp_heads.resize(S);
    for (int s = 0; s < S; ++s) {
        // stage 0 reads the final norm of rows 2b+1 (a norm kernel); later stages the folded one
        const bool folded = s > 0;
        QTTS_TRY(gemm_plan(&e->cp_heads[s], folded ? e->cxn : e->chid, folded ? crows : bmax, cH,
                           bf(d.cp_w_lm_head, (size_t)s * d.cp_vocab * cH), d.cp_vocab, QTTS_EPI_F32, e->clogits,
                           nullptr, nullptr, folded ? e->cxn_lo : e->chid_lo));
        if (folded) fold_norm_in(e->cp_heads[s], e->css, cH, d.cp_rms_eps);
    }
    if (e->cp_persist) {
        // per stage s >= 1: [QKV pair, O, gate/up, down] x layers, lm_head
        e->cpp_phases = 4 * d.cp_layers + 1;
        if (e->cpp_phases > kCppMaxPhases) {
            set_error("cp_persist: %d phases (max %d)", e->cpp_phases, kCppMaxPhases);
            return QTTS_ERR_UNSUPPORTED;
        }
        std::vector<CpPhase> prog((size_t)(S - 1) * e->cpp_phases);
        for (int s = 1; s < S; ++s) {
            CpPhase* ph = prog.data() + (size_t)(s - 1) * e->cpp_phases;
            const int32_t* m = e->cp_meta + (size_t)s * 4 * crows;
            // tiles per cluster: gate/up's 48 tiles as 4 tiles x split-K 2 (one round over the
            // clusters), the others split-K 8 (paired QKV: 2 x 4)
            const int gu_members = env_int("QTTS_CPP_GU_MEMBERS", 4);
            for (int l = 0; l < d.cp_layers; ++l) {
                const LayerGemms& g = e->cg[l];
                QTTS_TRY(cp_phase_from_plan(ph, g.qkv_pair, true, 2));
                ph->p.qkv.row_pos = m + crows;
                ph->p.qkv.slot_mapping = m;
                QTTS_TRY(cp_phase_from_plan(ph + 1, g.o, false, 1));
                QTTS_TRY(cp_phase_from_plan(ph + 2, g.gu, false, gu_members));
                QTTS_TRY(cp_phase_from_plan(ph + 3, g.down, false, 1));
                ph += 4;
            }
            QTTS_TRY(cp_phase_from_plan(ph, e->cp_heads[s], false, 1));
        }
        QTTS_TRY(dev_alloc(e, &e->cpp_prog, prog.size()));
        QTTS_CHECK_CUDA(cudaMemcpy(e->cpp_prog, prog.data(), prog.size() * sizeof(CpPhase), cudaMemcpyHostToDevice));
        QTTS_TRY(dev_alloc(e, &e->cpp_bar, 2));
        QTTS_CHECK_CUDA(cudaMemset(e->cpp_bar, 0, 2 * sizeof(unsigned)));
    }
    QTTS_TRY(gemm_plan(&e->head, e->hid, bmax, H, d.w_codec_head, d.vocab, QTTS_EPI_F32, nullptr, nullptr, nullptr,
                       e->hid_lo));
    // A projection prefetches the next one's weights into L2 while its own chain of latencies
    // runs.  QTTS_L2_CHAIN=1 (default): the code predictor's qkv -> o -> gate/up -> down -> next
    // layer's qkv (the last down -> the first qkv of the next stage; the lm_head is small),
    // whose 124 MB of weights per stage about fill L2; 2: the talker's projections as well
    // (qkv -> o -> gate/up -> down -> next qkv, the last -> the codec head), measured 3.6 %
    // slower on the talker, whose weights stream from HBM at a rate the prefetch does not
    // raise; 0: off.
    const int l2_chain = env_int("QTTS_L2_CHAIN", 1);
    if (l2_chain >= 2) {
        for (int l = 0; l < d.layers; ++l) {
            LayerGemms& g = e->tg[l];
            gemm_chain_l2(g.qkv, g.o);
            gemm_chain_l2(g.o, g.gu);
            gemm_chain_l2(g.gu, g.down);
            gemm_chain_l2(g.down, l + 1 < d.layers ? e->tg[l + 1].qkv : e->head);
        }
    }
    if (l2_chain >= 1) {
        for (int l = 0; l < d.cp_layers; ++l) {
            LayerGemms& g = e->cg[l];
            const LayerGemms& n = e->cg[(l + 1) % d.cp_layers];
            gemm_chain_l2(g.qkv, g.o);
            if (e->cp_qkv_pair) gemm_chain_l2(g.qkv_pair, g.o);
            gemm_chain_l2(g.o, g.gu);
            gemm_chain_l2(g.gu, g.down);
            gemm_chain_l2(g.down, e->cp_persist ? n.qkv_pair : n.qkv);
        }
    }
    return QTTS_OK;
}

inline int run_plan(const GemmPlan& g, int M, cudaStream_t st, void* out = nullptr) {
    return gemm_run(g, M, st, out);
}

inline int engine_step_impl(qtts_engine* e, const qtts_step_io& io, cudaStream_t st) {
    const qtts_model_desc& d = e->d;
    const int H = d.hidden, D = d.head_dim, Hq = d.heads, Hkv = d.kv_heads, I = d.inter;
    const int nr = io.n_rows, nn = io.n_new, R = nr * nn;
    if (nr <= 0 || nn <= 0 || nr > e->bmax || R > e->rmax) {
        set_error("engine_step: n_rows=%d n_new=%d outside max_batch=%d / max rows=%d", nr, nn, e->bmax, e->rmax);
        return QTTS_ERR_INVALID;
    }
    if (!io.slots || !io.x_in || !io.status) {
        set_error("engine_step: slots, x_in and status are required");
        return QTTS_ERR_INVALID;
    }
    if (io.sample && (!io.token_counts || !io.full_codec_out || !io.next_x_out || !io.logits_out)) {
        set_error("engine_step: sampling needs token_counts, logits_out, full_codec_out and next_x_out");
        return QTTS_ERR_INVALID;
    }
    const SchedView sv = view_of(&d.pool);
    // ---- scheduler: reserve KV positions, copy shared blocks
    QTTS_LAUNCH(sched_append_kernel, dim3(1), dim3(kSchedThreads), 0, st, sv, io.slots, nr, nn, e->mapping,
                e->row_ctx, e->row_pos, e->cow_src, e->cow_dst, io.status);
    const size_t block_elems = (size_t)d.layers * 2 * Hkv * d.pool.block_size * D;
    QTTS_LAUNCH(kv_copy_blocks_kernel, dim3(64, nr), dim3(256), 0, st, reinterpret_cast<uint4*>(d.kv_pool),
                block_elems / 8, (const int32_t*)e->cow_src, (const int32_t*)e->cow_dst, d.pool.num_blocks);
    QTTS_LAUNCH(expand_rows_kernel, dim3(ceil_div(R, 256)), dim3(256), 0, st, io.slots, nr, nn, e->row_slot);
    const int32_t* smap = io.slot_indexed ? io.slots : nullptr;
    QTTS_LAUNCH(load_x_kernel, dim3(ceil_div(R * H, 1024)), dim3(256), 0, st, io.x_in, e->x, R, H,
                (io.slot_indexed && nn == 1) ? smap : (const int32_t*)nullptr);

    AttnParams ap = {};
    ap.q = e->qbuf;
    ap.kv = reinterpret_cast<const kv_t*>(d.kv_pool);
    ap.num_heads = Hq;
    ap.kv_heads = Hkv;
    ap.num_layers = d.layers;
    ap.block_size = d.pool.block_size;
    ap.num_blocks = d.pool.num_blocks;
    ap.block_table = d.pool.block_table;
    ap.mbps = d.pool.max_blocks_per_seq;
    ap.row_slot = e->row_slot;
    ap.row_ctx = e->row_ctx;
    ap.max_splits = e->max_splits;
    ap.split_blocks = e->attn_split;
    ap.scale_log2 = 1.4426950408889634f / sqrtf((float)D);
    ap.ws_o = e->ws_o;
    ap.ws_ml = e->ws_ml;
    ap.out = e->attn;
    ap.out_lo = e->attn_lo;
    ap.R = R;
    ap.rows_per_stream = nn;
    // decode steps: the scheduler wrote the rows' metadata (and any copied blocks) at least two
    // launches before each layer's attention; only each row's newest key comes from the QKV
    // projection right before it
    ap.meta_settled = (nn == 1 && attn_early()) ? 1 : 0;

    // ---- talker layers
    for (int l = 0; l < d.layers; ++l) {
        const LayerGemms& g = e->tg[l];
        if (l == 0)  // later input norms are folded into the previous layer's down projection
            QTTS_TRY(launch_rmsnorm(e->x, R, H, H, bf(d.w_in_norm, 0), d.rms_eps, e->xn, st, e->xn_lo));
        QTTS_TRY(run_plan(g.qkv, R, st));
        ap.layer = l;
        if (nn > 1 && D == 128 && attn_use_tc() && attn_prefill_tiles())
            QTTS_TRY(launch_prefill_attention(ap, st));  // query tiles of the chunk share each KV block
        else
            QTTS_TRY(launch_attention(ap, D, st));
        QTTS_TRY(run_plan(g.o, R, st));  // + post-attention norm (folded)
        QTTS_TRY(run_plan(g.gu, R, st));
        QTTS_TRY(run_plan(g.down, R, st));
    }
    // ---- final norm of each stream's last new token, codec head
    QTTS_TRY(launch_rmsnorm(e->x + (size_t)(nn - 1) * H, nr, H, nn * H, d.w_final_norm, d.rms_eps, e->hid, st,
                            e->hid_lo));
    if (io.hidden_out)
        QTTS_CHECK_CUDA(cudaMemcpyAsync(io.hidden_out, e->hid, (size_t)nr * H * 2, cudaMemcpyDeviceToDevice, st));
    if (io.logits_out) QTTS_TRY(run_plan(e->head, nr, st, io.logits_out));
    if (!io.sample) return QTTS_OK;

    // ---- talker sampling head
    const int G = 1 + d.cp_stages;
    SampleParams sp = {};
    sp.logits = io.logits_out;
    sp.R = nr;
    sp.V = d.vocab;
    sp.ld = d.vocab;
    sp.topk = d.topk;
    sp.gumbel = io.gumbel;
    sp.gumbel_ld = d.topk;
    sp.seed = io.noise_seed;
    sp.noise_key = io.noise_key;
    sp.noise_step = io.noise_step;
    sp.step = io.noise_step ? 0 : io.step * 16;
    sp.temperature = io.temperature;
    sp.penalty = io.penalty;
    sp.counts = io.token_counts;
    sp.counts_row = smap;
    sp.eos_id = d.eos_id;
    sp.tok_out = io.full_codec_out;
    sp.tok_ld = G;
    QTTS_TRY(launch_sample(sp, st));

    // ---- code predictor
    const int cH = d.cp_hidden, cD = d.cp_head_dim, cHq = d.cp_heads, cHkv = d.cp_kv_heads;
    const int crows = 2 * e->bmax;
    AttnParams cap = {};
    cap.q = e->cq;
    cap.kv = e->cp_kv;
    cap.num_heads = cHq;
    cap.kv_heads = cHkv;
    cap.num_layers = d.cp_layers;
    cap.block_size = 16;
    cap.num_blocks = e->bmax;
    cap.block_table = e->cp_table;
    cap.mbps = 1;
    cap.max_splits = 1;
    cap.split_blocks = QTTS_ATTN_SPLIT_BLOCKS;
    cap.scale_log2 = 1.4426950408889634f / sqrtf((float)cD);
    cap.ws_o = e->cws_o;
    cap.ws_ml = e->cws_ml;
    cap.out = e->cattn;
    cap.out_lo = e->cattn_lo;
    cap.static_meta = 1;  // cp_meta and cp_table are written once, at build time

    // the tokens the next stage consumes: sampled, or forced by a parity test
    const int64_t* codes_in = io.force_codes ? io.force_codes : io.full_codec_out;
    CpClusterParams cpc = {};
    if (e->cp_cluster) {
        cpc.nr = nr;
        cpc.bmax = e->bmax;
        cpc.x_in = e->cx;
        cpc.logits = e->clogits;
        cpc.kv = e->cp_kv;
        const size_t nq = (size_t)kCpcQkv * cH / 8, no = (size_t)cH * cH / 8, ngu = (size_t)2 * d.cp_inter * cH / 8,
                     nd = (size_t)cH * d.cp_inter / 8;
        for (int l = 0; l < kCpcL; ++l) {
            cpc.w_qkv[l] = e->cpc_qkv + l * nq;
            cpc.w_o[l] = e->cpc_o + l * no;
            cpc.w_gu[l] = e->cpc_gu + l * ngu;
            cpc.w_down[l] = e->cpc_down + l * nd;
        }
        cpc.in_norm = bf(d.cp_w_in_norm, 0);
        cpc.post_norm = bf(d.cp_w_post_norm, 0);
        cpc.q_norm = bf(d.cp_w_q_norm, 0);
        cpc.k_norm = bf(d.cp_w_k_norm, 0);
        cpc.final_norm = bf(d.cp_w_final_norm, 0);
        cpc.rope_cos = d.cp_rope_cos;
        cpc.rope_sin = d.cp_rope_sin;
        cpc.eps = d.cp_rms_eps;
    }
    for (int s = 0; s < d.cp_stages; ++s) {
        const int rows = s == 0 ? 2 * nr : nr;
        const int32_t* m = e->cp_meta + (size_t)s * 4 * crows;
        if (s > 0 && e->cp_persist) {
            // the stage's 5 layers and lm_head in one persistent launch: logits -> e->clogits
            QTTS_TRY(launch_cp_persist(e->cpp_prog + (size_t)(s - 1) * e->cpp_phases, e->cpp_phases, nr, e->cpp_bar,
                                       st));
        } else if (s > 0 && e->cp_cluster) {
            // the stage's 5 layers and lm_head in one cluster launch: logits -> e->clogits
            cpc.stage = s;
            cpc.w_head = e->cpc_head + (size_t)s * d.cp_vocab * cH / 8;
            QTTS_TRY(launch_cp_cluster_stage(cpc, st));
        } else {
        if (s == 0) {
            QTTS_LAUNCH(cp_stage0_rows_kernel, dim3(nr), dim3(128), 0, st, (const __nv_bfloat16*)e->hid,
                        (const __nv_bfloat16*)e->hid_lo, bf(d.w_codec_emb, 0), d.vocab, H, codes_in, G, e->cp_in,
                        e->cp_in_lo);
            QTTS_TRY(run_plan(e->cp_proj_pair, rows, st));
        }  // stages 1..: the previous stage's sampling kernel wrote the input (next_table below)
        cap.row_slot = m + 3 * crows;
        cap.row_ctx = m + 2 * crows;
        cap.R = rows;
        for (int l = 0; l < d.cp_layers; ++l) {
            const LayerGemms& g = e->cg[l];
            GemmPlan q = g.qkv;  // input norm folded into the projection / previous down GEMM
            q.p.qkv.row_pos = m + crows;
            q.p.qkv.slot_mapping = m;
            QTTS_TRY(run_plan(q, rows, st));
            cap.layer = l;
            if (!e->cp_pair) QTTS_TRY(launch_short_attention(cap, cD, st));  // <= 16 keys per row
            QTTS_TRY(run_plan(g.o, rows, st));  // + post-attention norm (folded)
            QTTS_TRY(run_plan(g.gu, rows, st));
            QTTS_TRY(run_plan(g.down, rows, st));
        }
        // final norm: stage 0 normalises each stream's last position (row 2b+1) with a kernel;
        // from stage 1 on it is folded into the last down projection and the head
        if (s == 0)
            QTTS_TRY(launch_rmsnorm(e->cx + cH, nr, cH, 2 * cH, d.cp_w_final_norm, d.cp_rms_eps, e->chid, st,
                                    e->chid_lo));
        QTTS_TRY(run_plan(e->cp_heads[s], nr, st));
        }  // per-GEMM stage
        SampleParams cs = {};
        cs.logits = e->clogits;
        cs.R = nr;
        cs.V = d.cp_vocab;
        cs.ld = d.cp_vocab;
        cs.topk = d.topk < d.cp_vocab ? d.topk : d.cp_vocab;
        cs.gumbel = io.cp_gumbel ? io.cp_gumbel + (size_t)s * d.topk : nullptr;
        cs.gumbel_ld = d.cp_stages * d.topk;
        cs.seed = io.noise_seed;
        cs.noise_key = io.noise_key;
        cs.noise_step = io.noise_step;
        cs.step = (io.noise_step ? 0 : io.step * 16) + 1 + s;
        cs.temperature = io.temperature;
        cs.penalty = nullptr;
        cs.counts = nullptr;
        cs.counts_row = smap;  // per-stream temperature / noise state
        cs.eos_id = -1;
        cs.tok_out = io.full_codec_out + 1 + s;
        cs.tok_ld = G;
        if (s + 1 < d.cp_stages) {  // the next stage's input: its projected embedding of this code
            cs.next_table = (const float*)e->cp_tab + (size_t)s * d.cp_vocab * cH;
            cs.next_V = d.cp_vocab;
            cs.next_H = cH;
            cs.next_ids = codes_in + 1 + s;
            cs.next_ld = G;
            cs.next_gamma = bf(d.cp_w_in_norm, 0);
            cs.next_x = e->cx;
            cs.next_xn = e->cxn;
            cs.next_xn_lo = e->cxn_lo;
            cs.next_ss = e->css;
        }
        QTTS_TRY(launch_sample(cs, st));
        if (io.cp_logits_out)
            QTTS_CHECK_CUDA(cudaMemcpy2DAsync(io.cp_logits_out + (size_t)s * d.cp_vocab,
                                              (size_t)d.cp_stages * d.cp_vocab * sizeof(float), e->clogits,
                                              (size_t)d.cp_vocab * sizeof(float), (size_t)d.cp_vocab * sizeof(float),
                                              nr, cudaMemcpyDeviceToDevice, st));
    }
    // ---- codec embedding sum -> next input
    QTTS_LAUNCH(codec_sum_kernel, dim3(nr), dim3(256), G * sizeof(int64_t), st, (const int64_t*)io.full_codec_out,
                G, bf(d.w_codec_emb, 0), d.vocab, bf(d.cp_w_codec_emb, 0), d.cp_vocab, H, io.text_add,
                io.codec_sum_out, io.next_x_out, smap, io.noise_step);
    return QTTS_OK;
}

inline int engine_step(qtts_engine* e, qtts_step_io& io, cudaStream_t st) {
    g_launch_count = 0;
    const int rc = engine_step_impl(e, io, st);
    io.launches = g_launch_count;
    return rc;
}

}  // namespace qtts
