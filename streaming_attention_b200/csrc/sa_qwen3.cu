// sa_qwen3.cu -- Qwen3 forward on B200: weights, KV cache and the layer
// schedule behind the C ABI (sa_qwen3_*).
//
// Replaces tensor_cpp's qwen3_forward (qwen3_ops.cpp:537-614),
// qwen3_forward_with_cache (:936-1014) with the STANDARD attention type, and
// the KVCache it advances (kv_cache.h:27-238).
//
// Numerics: weights are held in bf16 (the reference loads bf16 checkpoints,
// qwen3_loader.cpp:157-164, so bf16 weights are exact); activations, the
// residual stream and the KV cache are fp32 like the reference.  Prompt
// projections run on tcgen05 tensor cores with each fp32 activation split
// into two bf16 terms (sa_gemm.cu); single-token decode runs GEMVs that
// stream the bf16 weights against fp32 activations.  Greedy decode therefore
// follows the fp32 reference token for token.
#include <cuda_bf16.h>
#include <cmath>
#include <cstring>
#include <map>
#include <set>
#include <utility>
#include <vector>

#include "sa_internal.h"
#include "sa_qwen3.h"

struct sa_qwen3 {
    sa_ctx* ctx = nullptr;
    int device = 0;                      // the context's GPU (the model may outlive the context object)
    sa_qwen3_config c{};
    // head-parallel rank (sa_qwen3_create_tp; world 1 = the whole model):
    // this rank's q heads, KV heads and intermediate features, and the
    // vocabulary rows [v0, v0 + vn) of its share of the decode lm_head
    int tp_rank = 0, tp_world = 1;
    int hq = 0, hkv = 0, inter = 0;
    int v0 = 0, vn = 0;
    int QD = 0, KD = 0, NQKV = 0;        // local: hq * D, hkv * D, QD + 2 KD
    // weights (device)
    __nv_bfloat16* embed = nullptr;      // [V, H]
    __nv_bfloat16* lm_head = nullptr;    // [V, H] (== embed when tied)
    float* final_norm = nullptr;         // [H]
    struct Layer {
        float* in_norm = nullptr;        // [H]
        float* post_norm = nullptr;      // [H]
        float* q_norm = nullptr;         // [D]
        float* k_norm = nullptr;         // [D]
        __nv_bfloat16* wqkv = nullptr;   // [QD + 2 KD, H]  rows: q | k | v
        __nv_bfloat16* wo = nullptr;     // [H, QD]
        __nv_bfloat16* wgu = nullptr;    // [2 I, H]  blocks of [gate 32; up 32]
        __nv_bfloat16* wd = nullptr;     // [H, I]
    };
    std::vector<Layer> layers;
    bool loaded_embed = false;
    std::vector<bool> loaded_layer;
    // KV cache (fp32) [L][hkv][max_seq][D] and its current length
    float* kc = nullptr;
    float* vc = nullptr;
    int cache_len = 0;
    float* cos_t = nullptr;              // [max_seq, D/2]
    float* sin_t = nullptr;
    // activations for up to cap_m tokens
    int cap_m = 0;
    float* x = nullptr;                  // [M, H]
    float* qkv = nullptr;                // [M, NQKV]
    float* q = nullptr;                  // [M, QD]
    float* attn = nullptr;               // [M, QD]
    float* act = nullptr;                // [M, I]  (decode path)
    float* xn = nullptr;                 // [M, H]  (final norm, decode path)
    __nv_bfloat16 *a_hi = nullptr, *a_lo = nullptr, *b_hi = nullptr, *b_lo = nullptr;   // [M, max(QD, I, H)]
    float* logits = nullptr;             // [logits_rows, V]
    int logits_rows = 0;
    int64_t* ids = nullptr;              // [M]
    float* gemm_ws = nullptr;            // split-K partial planes of the prompt GEMMs
    float* rowsq = nullptr;              // [H / 128 + 1][M] row sums of x^2 per GEMM tile (deferred RMSNorm)
    size_t gemm_ws_floats = 0;
    // streams: `cur` is where launches go (the context's stream, or the
    // model's own capturable stream inside graph-using calls)
    cudaStream_t own = nullptr;
    cudaStream_t cur = nullptr;
    cudaEvent_t ev_in = nullptr, ev_out = nullptr;
    // device-side decode state: [0] cache length, [1] tokens recorded
    int* d_state = nullptr;
    int64_t* d_toks = nullptr;           // [toks_cap]
    int toks_cap = 0;
    float* dec_scratch = nullptr;        // split partials for the decode step (max plan)
    unsigned* dec_cnt = nullptr;         // [hkv] attention + [hq + hkv] QKV-epilogue arrival counters
    unsigned long long* d_amax = nullptr;  // argmax key of the last lm_head GEMV (0 between uses)
    // single-launch decode step (sa_qwen3_mega.cu): set up on first use;
    // mega_grid < 0 once found unsupported
    int mega_grid = 0;
    sa::MegaLayer* d_mlayers = nullptr;  // [L]
    float* mpart = nullptr;              // attention split partials
    unsigned* mhead_cnt = nullptr;       // [hkv]
    unsigned* mgbar = nullptr;           // grid barrier words [4]
    // CUDA graphs: the single-token decode step; cache-free prefill per (S, logits mode)
    cudaGraphExec_t dec_graph = nullptr;
    std::map<std::pair<int, int>, cudaGraphExec_t> pf_graphs;
    std::set<std::pair<int, int>> pf_seen;
    // head-parallel exchange: this rank's buffer (flags [2][world], then
    // blocks [2][world][tp_rows * hidden]) and the peers' (CUDA IPC mappings)
    void* tp_buf = nullptr;
    size_t tp_flag_bytes = 0;            // flags + word areas, the offset of the receive blocks
    int tp_rows = 0;
    void* tp_peer[sa::TP_MAX] = {};
    bool tp_connected = false;
    unsigned* tp_seq = nullptr;          // [1] exchange instances completed
    unsigned* tp_cnt = nullptr;          // [1] producer arrival counter
    float* tp_part = nullptr;            // [cap_m, hidden] prompt-path partial sums
    float* tp_x2 = nullptr;              // [hidden] decode-path residual, other half of the ping-pong
    float* x_last = nullptr;             // residual after the last run_layers (m->x or tp_x2)
    bool x_last_ll = false;              // its pending exchange came as words (single-token path)
    // sequence-parallel rank (sa_qwen3_create_sp; the whole model on every
    // rank): prompts are split over the ranks by tokens; this rank's buffer
    // holds the flags [2][world] (256 bytes) and then the residual rows of a
    // prompt [sp_rows][hidden]; the peers' buffers and K/V caches are mapped
    int sp_rank = 0, sp_world = 1;
    void* sp_buf = nullptr;
    int sp_rows = 0;
    void* sp_peer_buf[sa::TP_MAX] = {};
    float* sp_peer_kc[sa::TP_MAX] = {};
    float* sp_peer_vc[sa::TP_MAX] = {};
    bool sp_connected = false;
    unsigned* sp_seq = nullptr;          // [1] exchange instances completed
    unsigned* sp_cnt = nullptr;          // [1] producer arrival counter
    unsigned char uuid[16] = {};         // the GPU's UUID (ranks must be on different GPUs)
    // long prompts' tensor-core attention: bf16 q [tc_cap, QD] and token-major
    // K / V [max_seq, KD] operands (allocated on first use)
    __nv_bfloat16* tc_q = nullptr;
    __nv_bfloat16* tc_k = nullptr;
    __nv_bfloat16* tc_v = nullptr;
    int tc_cap = 0;
};

namespace sa {

static int dmalloc(void** p, size_t bytes) {
    if (cudaMalloc(p, bytes) != cudaSuccess) {
        cudaGetLastError();
        return set_error(SA_ERR_OOM, "cudaMalloc of %zu bytes failed", bytes);
    }
    return SA_OK;
}

template <typename T>
static int dalloc(T** p, size_t n) { return dmalloc(reinterpret_cast<void**>(p), n * sizeof(T)); }

static uint16_t f2bf(float f) {
    uint32_t u;
    std::memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40);
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

// Copy n fp32 host values to the device (blocking).
static int upload_f32(float* dst, const float* src, size_t n, cudaStream_t st) {
    SA_CUDA_TRY(cudaMemcpyAsync(dst, src, n * 4, cudaMemcpyHostToDevice, st));
    SA_CUDA_TRY(cudaStreamSynchronize(st));
    return SA_OK;
}

static void free_model(sa_qwen3* m) {
    cudaFree(m->embed);
    if (m->lm_head != m->embed) cudaFree(m->lm_head);
    cudaFree(m->final_norm);
    for (auto& L : m->layers) {
        cudaFree(L.in_norm); cudaFree(L.post_norm); cudaFree(L.q_norm); cudaFree(L.k_norm);
        cudaFree(L.wqkv); cudaFree(L.wo); cudaFree(L.wgu); cudaFree(L.wd);
    }
    cudaFree(m->kc); cudaFree(m->vc); cudaFree(m->cos_t); cudaFree(m->sin_t);
    cudaFree(m->x); cudaFree(m->qkv); cudaFree(m->q); cudaFree(m->attn); cudaFree(m->act); cudaFree(m->xn);
    cudaFree(m->a_hi); cudaFree(m->a_lo); cudaFree(m->b_hi); cudaFree(m->b_lo); cudaFree(m->rowsq);
    cudaFree(m->logits); cudaFree(m->ids); cudaFree(m->gemm_ws);
    cudaFree(m->d_state); cudaFree(m->d_toks); cudaFree(m->dec_scratch); cudaFree(m->dec_cnt); cudaFree(m->d_amax);
    cudaFree(m->d_mlayers); cudaFree(m->mpart); cudaFree(m->mhead_cnt); cudaFree(m->mgbar);
    for (int r = 0; r < sa::TP_MAX; ++r)
        if (m->tp_peer[r] && r != m->tp_rank) cudaIpcCloseMemHandle(m->tp_peer[r]);
    cudaFree(m->tp_buf); cudaFree(m->tp_seq); cudaFree(m->tp_cnt); cudaFree(m->tp_part); cudaFree(m->tp_x2);
    for (int r = 0; r < sa::TP_MAX; ++r) {
        if (r == m->sp_rank) continue;
        if (m->sp_peer_buf[r]) cudaIpcCloseMemHandle(m->sp_peer_buf[r]);
        if (m->sp_peer_kc[r]) cudaIpcCloseMemHandle(m->sp_peer_kc[r]);
        if (m->sp_peer_vc[r]) cudaIpcCloseMemHandle(m->sp_peer_vc[r]);
    }
    cudaFree(m->sp_buf); cudaFree(m->sp_seq); cudaFree(m->sp_cnt);
    cudaFree(m->tc_q); cudaFree(m->tc_k); cudaFree(m->tc_v);
    if (m->dec_graph) cudaGraphExecDestroy(m->dec_graph);
    for (auto& kv : m->pf_graphs) cudaGraphExecDestroy(kv.second);
    if (m->ev_in) cudaEventDestroy(m->ev_in);
    if (m->ev_out) cudaEventDestroy(m->ev_out);
    if (m->own) cudaStreamDestroy(m->own);
}

// Graphs hold buffer addresses; drop them whenever a buffer is reallocated.
static void invalidate_graphs(sa_qwen3* m) {
    if (m->dec_graph) cudaGraphExecDestroy(m->dec_graph);
    m->dec_graph = nullptr;
    for (auto& kv : m->pf_graphs) cudaGraphExecDestroy(kv.second);
    m->pf_graphs.clear();
    m->pf_seen.clear();
}

// Activation buffers for up to M tokens (grow-only).
static int ensure_acts(sa_qwen3* m, int M) {
    if (M <= m->cap_m) return SA_OK;
    SA_CUDA_TRY(cudaStreamSynchronize(m->cur));
    SA_CUDA_TRY(cudaStreamSynchronize(m->ctx->stream));
    invalidate_graphs(m);
    cudaFree(m->x); cudaFree(m->qkv); cudaFree(m->q); cudaFree(m->attn); cudaFree(m->act); cudaFree(m->xn);
    cudaFree(m->a_hi); cudaFree(m->a_lo); cudaFree(m->b_hi); cudaFree(m->b_lo); cudaFree(m->ids);
    cudaFree(m->tp_part);
    cudaFree(m->rowsq);
    m->tp_part = nullptr;
    m->rowsq = nullptr;
    const sa_qwen3_config& c = m->c;
    const size_t wmax = (size_t)std::max(std::max(m->QD, m->inter), c.hidden);
    int rc = SA_OK;
    if (!rc) rc = dalloc(&m->x, (size_t)M * c.hidden);
    if (!rc) rc = dalloc(&m->qkv, (size_t)M * m->NQKV);
    if (!rc) rc = dalloc(&m->q, (size_t)M * m->QD);
    if (!rc) rc = dalloc(&m->attn, (size_t)M * m->QD);
    if (!rc) rc = dalloc(&m->act, (size_t)M * m->inter);
    if (!rc && m->tp_world > 1) rc = dalloc(&m->tp_part, (size_t)M * c.hidden);
    if (!rc) rc = dalloc(&m->xn, (size_t)M * c.hidden);
    if (!rc) rc = dalloc(&m->a_hi, (size_t)M * wmax);
    if (!rc) rc = dalloc(&m->a_lo, (size_t)M * wmax);
    if (!rc) rc = dalloc(&m->b_hi, (size_t)M * wmax);
    if (!rc) rc = dalloc(&m->b_lo, (size_t)M * wmax);
    if (!rc) rc = dalloc(&m->ids, (size_t)M);
    if (!rc) rc = dalloc(&m->rowsq, (size_t)M * (c.hidden / 128 + 1));
    if (rc) { m->cap_m = 0; return rc; }
    m->cap_m = M;
    return SA_OK;
}

static int ensure_logits(sa_qwen3* m, int rows) {
    if (rows <= m->logits_rows) return SA_OK;
    SA_CUDA_TRY(cudaStreamSynchronize(m->cur));
    SA_CUDA_TRY(cudaStreamSynchronize(m->ctx->stream));
    invalidate_graphs(m);
    cudaFree(m->logits);
    m->logits = nullptr;
    int rc = dalloc(&m->logits, (size_t)rows * m->c.vocab);
    m->logits_rows = rc ? 0 : rows;
    return rc;
}

// Prompt projection on the tensor cores with the tile / split plan for its
// shape.  With split_ok the plan may split K: then the partial planes are left
// in m->gemm_ws for the next kernel and *splits (when given) is the plane
// count; otherwise `mode` is applied and *splits is 1.
static int gemm(sa_qwen3* m, const __nv_bfloat16* hi, const __nv_bfloat16* lo, long long lda,
                const __nv_bfloat16* w, int M, int N, int K, int mode, float* C, long long ldc,
                __nv_bfloat16* ohi, __nv_bfloat16* olo, long long ldo, bool split_ok = false, int* splits = nullptr,
                const GemmEpi* epi = nullptr) {
    // fused epilogues: the plan run_layers chose them by (it must be unsplit)
    const GemmPlan plan = gemm_plan(m->ctx->device, m->ctx->num_sms, M, N, K, (split_ok && splits) || epi);
    if (epi && plan.splits != 1) return set_error(SA_ERR_ARG, "gemm: fused epilogue on a split plan");
    const size_t need = plan.splits > 1 ? (size_t)plan.splits * M * N : 0;
    if (need > m->gemm_ws_floats) {
        // grow-only; graphs captured with the old buffer are dropped
        SA_CUDA_TRY(cudaStreamSynchronize(m->cur));
        invalidate_graphs(m);
        cudaFree(m->gemm_ws);
        m->gemm_ws = nullptr;
        m->gemm_ws_floats = 0;
        int rc = dalloc(&m->gemm_ws, need);
        if (rc) return rc;
        m->gemm_ws_floats = need;
    }
    if (splits) *splits = plan.splits;
    return gemm_launch(m->cur, m->ctx->status, hi, lo, lda, w, M, N, K, mode, C, ldc, ohi, olo, ldo, plan,
                       m->gemm_ws, m->gemm_ws_floats, epi);
}

#define SA_RC(expr) do { int rc_ = (expr); if (rc_) return rc_; } while (0)

// Prompts of at least this many tokens run their attention on the tcgen05
// tensor cores (bf16 q / K / V, fp32 accumulation, sa_prefill.cu); shorter
// ones on the fp32 CUDA-core prompt-attention kernel, whose cost grows with
// the square of the prompt.  SA_QWEN3_TC_ATTN_MIN overrides the crossover.
static int tc_attn_min_rows() {
    static const int v = [] {
        const char* e = std::getenv("SA_QWEN3_TC_ATTN_MIN");
        return e ? std::atoi(e) : 256;
    }();
    return v;
}

// The tensor-core attention's operand buffers for M query rows.
static int ensure_tc(sa_qwen3* m, int M) {
    if (m->tc_k && M <= m->tc_cap) return SA_OK;
    SA_CUDA_TRY(cudaStreamSynchronize(m->cur));
    SA_CUDA_TRY(cudaStreamSynchronize(m->ctx->stream));
    invalidate_graphs(m);
    cudaFree(m->tc_q);
    m->tc_q = nullptr;
    m->tc_cap = 0;
    if (!m->tc_k) {
        SA_RC(dalloc(&m->tc_k, (size_t)m->c.max_seq * m->KD));
        SA_RC(dalloc(&m->tc_v, (size_t)m->c.max_seq * m->KD));
    }
    SA_RC(dalloc(&m->tc_q, (size_t)M * m->QD));
    m->tc_cap = M;
    return SA_OK;
}


// Tokens ids (device) at positions pos0 .. pos0+M-1 through every layer.
// Their K/V go to cache rows kv_row0 + (0 .. M-1) and attention reads rows
// from kv_row0 - pos0: with the cache, kv_row0 = pos0 = cache length; a
// cache-free forward (positions from 0) uses the rows after the live prefix
// as scratch, kv_row0 = cache length, so the cache is left as it was.
// M == 1 uses the GEMV path; pos_dev makes the position a device value.
// Exchange operands of instance k of the current segment (head-parallel).
static TpArgs tp_args(sa_qwen3* m, int k) {
    TpArgs t;
    t.rank = m->tp_rank;
    t.world = m->tp_world;
    for (int r = 0; r < m->tp_world; ++r) {
        char* base = static_cast<char*>(m->tp_peer[r]);
        t.flags[r] = reinterpret_cast<unsigned*>(base);
        t.ll[r] = reinterpret_cast<unsigned long long*>(base + 256);
        t.recv[r] = reinterpret_cast<float*>(base + m->tp_flag_bytes);
    }
    t.ll_stride = m->c.hidden;
    t.slot_floats = (long long)m->tp_rows * m->c.hidden;
    t.seq = m->tp_seq;
    t.k = k;
    t.cnt = m->tp_cnt;
    t.status = m->ctx->status;
    return t;
}

// Exchange operands of instance k of the current sequence-parallel segment:
// the flags of every rank's buffer, the sequence word and arrival counter.
static TpArgs sp_args(sa_qwen3* m, int k) {
    TpArgs t;
    t.rank = m->sp_rank;
    t.world = m->sp_world;
    for (int r = 0; r < m->sp_world; ++r) t.flags[r] = static_cast<unsigned*>(m->sp_peer_buf[r]);
    t.seq = m->sp_seq;
    t.k = k;
    t.cnt = m->sp_cnt;
    t.status = m->ctx->status;
    return t;
}
static float* sp_xrows(sa_qwen3* m, int r) {
    return reinterpret_cast<float*>(static_cast<char*>(m->sp_peer_buf[r]) + 256);
}

// Head-parallel ranks run the same schedule on their share of the heads and
// intermediate features; each layer exchanges two partial sums of the
// residual update (o_proj, down_proj: instances 2l and 2l + 1 of the
// segment), which the next normed projection adds in before its norm.  In
// the single-token path the residual alternates between m->x and m->tp_x2
// (the consuming GEMV reads one and writes the other); m->x_last records
// where it ends.  The prompt path updates m->x in place.
//
// Sequence-parallel ranks (sp) run the prompt path on their own tokens at
// their global positions; after QK-norm, RoPE and the cache append of a
// layer, the rank's new K/V rows go to the same rows of every other rank's
// cache (instance l of the segment) and every rank waits for all ranks'
// rows before the causal attention, which then sees the whole prefix.
static int run_layers(sa_qwen3* m, int M, int pos0, const int* pos_dev = nullptr, int kv_row0 = -1,
                      bool sp = false) {
    if (kv_row0 < 0) kv_row0 = pos0;
    const sa_qwen3_config& c = m->c;
    cudaStream_t st = m->cur;
    const int H = c.hidden, I = m->inter, D = c.head_dim;
    const float scale = 1.0f / sqrtf((float)D);
    const size_t layer_kv = (size_t)m->hkv * c.max_seq * D;
    const bool tp = m->tp_world > 1;
    float* xc = m->x;          // single-token path: the residual the next consumer reads
    float* xo = m->tp_x2;
    SA_RC(launch_embedding(st, m->ids, M, m->embed, c.vocab, H, m->x, m->ctx->status));
    int resid = 0;   // partial planes of the last down_proj not yet added to x
    // Prompt path, one GPU or sequence-parallel: unsplit GEMMs take the fused
    // epilogues (GemmEpi).  QKV with QK-norm + RoPE + cache append
    // (fuse_qkv); an unsplit o_proj / down_proj whose consumer is unsplit
    // too writes the consumer's A operand with its RMSNorm deferred
    // (defer_gu: o_proj -> gate/up, defer_qkv: down_proj -> the next QKV).
    // The plans are those gemm() picks for these shapes.
    bool fuse_qkv = false, defer_gu = false, defer_qkv = false;
    int parts_o = 0, parts_d = 0;
    if (M > 1 && !tp && D == 128) {
        const int dev = m->ctx->device, sms = m->ctx->num_sms;
        const GemmPlan pq = gemm_plan(dev, sms, M, m->NQKV, H, true), po = gemm_plan(dev, sms, M, H, m->QD, true);
        const GemmPlan pg = gemm_plan(dev, sms, M, 2 * I, H, true), pd = gemm_plan(dev, sms, M, H, I, true);
        fuse_qkv = pq.splits == 1 && pq.bn % 128 == 0 && m->NQKV % pq.bn == 0;
        defer_gu = po.splits == 1 && po.bn % 128 == 0 && H % po.bn == 0 && pg.splits == 1;
        defer_qkv = fuse_qkv && pd.splits == 1 && pd.bn % 128 == 0 && H % pd.bn == 0;
        parts_o = H / po.bn;
        parts_d = H / pd.bn;
    }
    const bool tc_attn = M > 1 && M >= tc_attn_min_rows();
    const bool tc_direct = fuse_qkv && tc_attn && !sp;   // the QKV epilogue writes the bf16 operands
    // bf16 hi/lo activation buffers: `qkv_in` holds the QKV GEMM's A operand
    // (RMSNorm'd x, or hi/lo(g . x) after a deferred down_proj); the
    // attention output goes to a; a GEMM never writes the buffer it reads.
    __nv_bfloat16 *qkv_hi = m->a_hi, *qkv_lo = m->a_lo;
    for (int l = 0; l < c.n_layers; ++l) {
        const sa_qwen3::Layer& L = m->layers[l];
        float* kc = m->kc + l * layer_kv;
        float* vc = m->vc + l * layer_kv;
        const int shift = kv_row0 - pos0;                     // cache row - RoPE position
        const float* ka = kc + (size_t)shift * D;             // attention view of this sequence
        const float* va = vc + (size_t)shift * D;
        if (M == 1) {
            QkvEpi e;
            e.hq = m->hq; e.hkv = m->hkv; e.max_seq = c.max_seq; e.pos0 = pos0; e.row_shift = shift;
            e.pos_dev = pos_dev;
            e.qn = L.q_norm; e.kn = L.k_norm; e.cos_t = m->cos_t; e.sin_t = m->sin_t;
            e.q_out = m->q; e.kc = kc; e.vc = vc;
            e.cnt = m->dec_cnt + m->hkv;
            if (tp && l > 0) {
                TpArgs t = tp_args(m, 2 * l - 1);
                t.x_out = xo;
                t.use_ll = 1;
                SA_RC(launch_gemv2_tp(st, QW_EPI_QKV, true, L.wqkv, m->NQKV, H, xc, L.in_norm, c.eps, m->qkv,
                                      nullptr, &e, t, true));
                std::swap(xc, xo);
            } else {
                SA_RC(launch_gemv2(st, QW_EPI_QKV, true, L.wqkv, m->NQKV, H, xc, L.in_norm, c.eps, m->qkv, nullptr,
                                   &e));
            }
            SA_RC(decode_dev_launch(st, m->ctx->status, m->ctx->num_sms, m->q, ka, va, (long long)c.max_seq * D,
                                    pos_dev, pos0 + 1, c.max_seq - shift, D, m->hq, m->hkv, scale, m->attn,
                                    m->dec_scratch, m->dec_cnt));
            if (tp) {
                SA_RC(launch_gemv2_tp(st, QW_EPI_XCHG, false, L.wo, H, m->QD, m->attn, nullptr, 0.f, nullptr, nullptr,
                                      nullptr, tp_args(m, 2 * l), false));
                TpArgs t = tp_args(m, 2 * l);
                t.x_out = xo;
                t.use_ll = 1;
                SA_RC(launch_gemv2_tp(st, QW_EPI_SWIGLU, true, L.wgu, I, H, xc, L.post_norm, c.eps, m->act, nullptr,
                                      nullptr, t, true));
                std::swap(xc, xo);
                SA_RC(launch_gemv2_tp(st, QW_EPI_XCHG, false, L.wd, H, I, m->act, nullptr, 0.f, nullptr, nullptr,
                                      nullptr, tp_args(m, 2 * l + 1), false));
            } else {
                SA_RC(launch_gemv2(st, QW_EPI_RESID, false, L.wo, H, m->QD, m->attn, nullptr, 0.f, m->x, nullptr));
                SA_RC(launch_gemv2(st, QW_EPI_SWIGLU, true, L.wgu, I, H, m->x, L.post_norm, c.eps, m->act, nullptr));
                SA_RC(launch_gemv2(st, QW_EPI_RESID, false, L.wd, H, I, m->act, nullptr, 0.f, m->x, nullptr));
            }
        } else {
            // split GEMMs leave partial planes (m->gemm_ws) that the next
            // kernel adds: `resid` counts the planes of a pending residual add
            const bool deferred_in = defer_qkv && l > 0;   // qkv_in = hi/lo(in_norm . x), rows unscaled
            if (tp && l > 0)
                SA_RC(launch_rmsnorm_hilo_tp(st, m->x, L.in_norm, M, H, c.eps, m->a_hi, m->a_lo, tp_args(m, 2 * l - 1)));
            else if (!deferred_in)
                SA_RC(launch_rmsnorm_hilo(st, m->x, L.in_norm, M, H, c.eps, m->a_hi, m->a_lo, m->gemm_ws, resid));
            if (!deferred_in) {
                qkv_hi = m->a_hi;
                qkv_lo = m->a_lo;
            }
            resid = 0;
            if (fuse_qkv) {
                GemmEpi e;
                if (deferred_in) {
                    e.rowsq_in = m->rowsq;
                    e.rowsq_parts = parts_d;
                    e.norm_k = (float)H;
                    e.eps = c.eps;
                }
                e.hq = m->hq; e.hkv = m->hkv; e.max_seq = c.max_seq; e.pos0 = pos0; e.row_shift = shift;
                e.qn = L.q_norm; e.kn = L.k_norm; e.cos_t = m->cos_t; e.sin_t = m->sin_t;
                e.kc = kc; e.vc = vc;
                if (tc_direct) {
                    e.q_bf = m->tc_q; e.k_bf = m->tc_k; e.v_bf = m->tc_v;
                } else {
                    e.q_out = m->q;
                }
                SA_RC(gemm(m, qkv_hi, qkv_lo, H, L.wqkv, M, m->NQKV, H, QW_EPI_QKV_ROWS, nullptr, 0, nullptr, nullptr,
                           0, false, nullptr, &e));
            } else {
                int sq = 1;
                SA_RC(gemm(m, qkv_hi, qkv_lo, H, L.wqkv, M, m->NQKV, H, QW_EPI_STORE, m->qkv, m->NQKV, nullptr, nullptr,
                           0, true, &sq));
                SA_RC(launch_qknorm_rope_append(st, sq > 1 ? m->gemm_ws : m->qkv, sq, M, m->hq, m->hkv, L.q_norm,
                                                L.k_norm, m->cos_t, m->sin_t, pos0, nullptr, shift, m->q, kc, vc,
                                                c.max_seq));
            }
            if (sp) {
                SpCopy cp;
                cp.nreg = 2;
                cp.src[0] = kc + (size_t)kv_row0 * D;
                cp.src[1] = vc + (size_t)kv_row0 * D;
                for (int r = 0; r < m->sp_world; ++r) {
                    if (r == m->sp_rank) continue;
                    cp.dst[0][r] = m->sp_peer_kc[r] + l * layer_kv + (size_t)kv_row0 * D;
                    cp.dst[1][r] = m->sp_peer_vc[r] + l * layer_kv + (size_t)kv_row0 * D;
                }
                cp.nblk = m->hkv;
                cp.blk_floats = (long long)M * D;
                cp.stride = (long long)c.max_seq * D;
                SA_RC(launch_sp_rows_scatter(st, cp, sp_args(m, l), m->ctx->num_sms));
                SA_RC(launch_sp_wait(st, sp_args(m, l)));
            }
            if (tc_attn) {
                // rows [0, pos0 + M) of the attention view as bf16 operands
                // (only the cached prefix when the QKV epilogue wrote the
                // new rows), the causal prefill on the tensor cores with its
                // output as the o_proj GEMM's hi/lo planes
                const int T = pos0 + M;
                if (!tc_direct)
                    SA_RC(launch_tc_pack(st, m->q, M, m->QD, ka, va, c.max_seq, m->hkv, T, m->tc_q, m->tc_k, m->tc_v,
                                         m->ctx->num_sms));
                else if (pos0 > 0)
                    SA_RC(launch_tc_pack(st, nullptr, 0, m->QD, ka, va, c.max_seq, m->hkv, pos0, m->tc_q, m->tc_k,
                                         m->tc_v, m->ctx->num_sms));
                SA_RC(prefill_launch(st, m->ctx->status, m->tc_q, m->tc_k, m->tc_v, m->a_hi, SA_BF16, M, T, pos0,
                                     m->hq, m->hkv, m->QD, m->KD, m->QD, scale, m->a_lo));
            } else {
                SA_RC(prompt_attn_launch(st, m->ctx->status, m->q, m->QD, ka, va, (long long)c.max_seq * D,
                                         (long long)m->hkv * c.max_seq - shift, pos0 + 1, M, D, m->hq, m->hkv, scale,
                                         nullptr, m->QD, m->a_hi, m->a_lo));
            }
            // gate/up reads gu_in and writes the SwiGLU output to gu_out
            __nv_bfloat16 *gu_in_hi = m->a_hi, *gu_in_lo = m->a_lo, *gu_out_hi = m->b_hi, *gu_out_lo = m->b_lo;
            if (tp) {
                SA_RC(gemm(m, m->a_hi, m->a_lo, m->QD, L.wo, M, H, m->QD, QW_EPI_STORE, m->tp_part, H, nullptr, nullptr,
                           0));
                SA_RC(launch_tp_scatter(st, m->tp_part, M, H, tp_args(m, 2 * l), m->ctx->num_sms));
                SA_RC(launch_rmsnorm_hilo_tp(st, m->x, L.post_norm, M, H, c.eps, m->a_hi, m->a_lo, tp_args(m, 2 * l)));
            } else if (defer_gu) {
                GemmEpi e;
                e.g = L.post_norm;
                e.rowsq_out = m->rowsq;
                SA_RC(gemm(m, m->a_hi, m->a_lo, m->QD, L.wo, M, H, m->QD, QW_EPI_RESID_NORM, m->x, H, m->b_hi, m->b_lo,
                           H, false, nullptr, &e));
                gu_in_hi = m->b_hi; gu_in_lo = m->b_lo; gu_out_hi = m->a_hi; gu_out_lo = m->a_lo;
            } else {
                int so = 1;
                SA_RC(gemm(m, m->a_hi, m->a_lo, m->QD, L.wo, M, H, m->QD, QW_EPI_RESID, m->x, H, nullptr, nullptr, 0,
                           true, &so));
                SA_RC(launch_rmsnorm_hilo(st, m->x, L.post_norm, M, H, c.eps, m->a_hi, m->a_lo, m->gemm_ws,
                                          so > 1 ? so : 0));
            }
            int sg = 1;
            if (defer_gu) {
                GemmEpi e;
                e.rowsq_in = m->rowsq;
                e.rowsq_parts = parts_o;
                e.norm_k = (float)H;
                e.eps = c.eps;
                SA_RC(gemm(m, gu_in_hi, gu_in_lo, H, L.wgu, M, 2 * I, H, QW_EPI_SWIGLU, nullptr, 0, gu_out_hi, gu_out_lo,
                           I, false, nullptr, &e));
            } else {
                SA_RC(gemm(m, gu_in_hi, gu_in_lo, H, L.wgu, M, 2 * I, H, QW_EPI_SWIGLU, nullptr, 0, gu_out_hi, gu_out_lo,
                           I, true, &sg));
            }
            if (sg > 1) SA_RC(launch_swiglu_hilo(st, m->gemm_ws, sg, M, I, gu_out_hi, gu_out_lo, I, m->ctx->num_sms));
            if (tp) {
                SA_RC(gemm(m, gu_out_hi, gu_out_lo, I, L.wd, M, H, I, QW_EPI_STORE, m->tp_part, H, nullptr, nullptr, 0));
                SA_RC(launch_tp_scatter(st, m->tp_part, M, H, tp_args(m, 2 * l + 1), m->ctx->num_sms));
            } else if (defer_qkv && l + 1 < c.n_layers) {
                // the next layer's QKV A operand, in whichever buffer this
                // GEMM does not read
                GemmEpi e;
                e.g = m->layers[l + 1].in_norm;
                e.rowsq_out = m->rowsq;
                qkv_hi = gu_out_hi == m->a_hi ? m->b_hi : m->a_hi;
                qkv_lo = gu_out_hi == m->a_hi ? m->b_lo : m->a_lo;
                SA_RC(gemm(m, gu_out_hi, gu_out_lo, I, L.wd, M, H, I, QW_EPI_RESID_NORM, m->x, H, qkv_hi, qkv_lo, H,
                           false, nullptr, &e));
            } else {
                int sd = 1;
                SA_RC(gemm(m, gu_out_hi, gu_out_lo, I, L.wd, M, H, I, QW_EPI_RESID, m->x, H, nullptr, nullptr, 0, true,
                           &sd));
                resid = sd > 1 ? sd : 0;
            }
        }
    }
    if (resid) SA_RC(launch_resid_add(st, m->x, m->gemm_ws, resid, M, H, m->ctx->num_sms));
    m->x_last = M == 1 ? xc : m->x;
    m->x_last_ll = M == 1;
    return SA_OK;
}

// Final norm + lm_head for rows [r0, r0 + n) of the residual stream.  With
// `token` (n == 1 only) the argmax of the logits is also written there
// (first index of the maximum, as ops::argmax).  Head-parallel ranks first
// add the last layer's exchanged down_proj sums (instance 2L - 1); with
// `token` each rank takes the argmax over its vocabulary slice and the
// ranks' maxima are exchanged (instance 2L), which also closes the segment.
// `xsrc` (the single-GPU path only) reads the residual rows from there
// instead of m->x: the rows a sequence-parallel prompt gathered.
static int run_head(sa_qwen3* m, int r0, int n, int64_t* token = nullptr, const float* xsrc = nullptr) {
    const sa_qwen3_config& c = m->c;
    cudaStream_t st = m->cur;
    const size_t H = c.hidden;
    SA_RC(ensure_logits(m, n));
    if (m->tp_world > 1) {
        const int L2 = 2 * c.n_layers;
        TpArgs t = tp_args(m, L2 - 1);
        t.row = r0;
        t.use_ll = m->x_last_ll ? 1 : 0;
        if (n == 1) {
            const float* xin = m->x_last + (m->x_last == m->x ? (size_t)r0 * H : 0);
            t.x_out = m->x_last == m->tp_x2 ? m->x : m->tp_x2;
            if (token) {
                t.n_base = m->v0;
                SA_RC(launch_gemv2_tp(st, QW_EPI_STORE, true, m->lm_head + (size_t)m->v0 * H, m->vn, (int)H, xin,
                                      m->final_norm, c.eps, m->logits, m->d_amax, nullptr, t, true));
                SA_RC(launch_tp_amax_token(st, m->d_amax, token, tp_args(m, L2), L2 + 1));
            } else {
                SA_RC(launch_gemv2_tp(st, QW_EPI_STORE, true, m->lm_head, c.vocab, (int)H, xin, m->final_norm, c.eps,
                                      m->logits, nullptr, nullptr, t, true));
            }
        } else {
            SA_RC(launch_rmsnorm_hilo_tp(st, m->x + (size_t)r0 * H, m->final_norm, n, (int)H, c.eps, m->a_hi, m->a_lo,
                                         t));
            SA_RC(gemm(m, m->a_hi, m->a_lo, c.hidden, m->lm_head, n, c.vocab, c.hidden, QW_EPI_STORE, m->logits,
                       c.vocab, nullptr, nullptr, 0));
        }
        return SA_OK;
    }
    const float* xs = xsrc ? xsrc : m->x;
    if (n == 1) {
        SA_RC(launch_gemv2(st, QW_EPI_STORE, true, m->lm_head, c.vocab, c.hidden, xs + (size_t)r0 * c.hidden,
                           m->final_norm, c.eps, m->logits, token ? m->d_amax : nullptr));
        if (token) SA_RC(launch_amax_to_token(st, m->d_amax, token));
    } else {
        SA_RC(launch_rmsnorm_hilo(st, const_cast<float*>(xs) + (size_t)r0 * c.hidden, m->final_norm, n, c.hidden, c.eps,
                                  m->a_hi, m->a_lo));
        SA_RC(gemm(m, m->a_hi, m->a_lo, c.hidden, m->lm_head, n, c.vocab, c.hidden, QW_EPI_STORE, m->logits, c.vocab,
                   nullptr, nullptr, 0));
    }
    return SA_OK;
}

// This rank's tokens [s0, s1) of an S-token sequence-parallel prompt.
static void sp_share(const sa_qwen3* m, int S, int* s0, int* s1) {
    *s0 = (int)((long long)S * m->sp_rank / m->sp_world);
    *s1 = (int)((long long)S * (m->sp_rank + 1) / m->sp_world);
}
static bool sp_split(const sa_qwen3* m, int S) { return m->sp_world > 1 && S >= 2 * m->sp_world; }

// A sequence-parallel prompt of S tokens at positions pos0.. and cache rows
// kv_row0.. (m->ids holds this rank's tokens): this rank's layers with the
// per-layer K/V exchanges (instances 0..L-1), then every rank's final
// residual rows gathered in every rank's row buffer (instance L), which
// *x_all points to; the segment's L + 1 instances are then counted.
static int run_prompt_sp(sa_qwen3* m, int S, int pos0, int kv_row0, const float** x_all) {
    const int L = m->c.n_layers, H = m->c.hidden;
    int s0, s1;
    sp_share(m, S, &s0, &s1);
    SA_RC(run_layers(m, s1 - s0, pos0 + s0, nullptr, kv_row0 + s0, true));
    SpCopy cp;
    cp.nreg = 1;
    cp.src[0] = m->x;
    for (int r = 0; r < m->sp_world; ++r) cp.dst[0][r] = sp_xrows(m, r) + (size_t)s0 * H;
    cp.nblk = 1;
    cp.blk_floats = (long long)(s1 - s0) * H;
    SA_RC(launch_sp_rows_scatter(m->cur, cp, sp_args(m, L), m->ctx->num_sms));
    SA_RC(launch_sp_wait(m->cur, sp_args(m, L)));
    SA_RC(launch_tp_seq_add(m->cur, m->sp_seq, L + 1));
    *x_all = sp_xrows(m, m->sp_rank);
    return SA_OK;
}

// Close a head-parallel segment that did not end with the token exchange
// (which closes its own): the sequence word advances by the 2L instances.
static int tp_close_segment(sa_qwen3* m) {
    if (m->tp_world > 1) SA_RC(launch_tp_seq_add(m->cur, m->tp_seq, 2 * m->c.n_layers));
    return SA_OK;
}

}  // namespace sa

using namespace sa;

namespace sa {

// Allocate rank `rank` of a `world`-way head-parallel model (world 1: the
// whole model).
int qwen3_create_model(sa_ctx* ctx, const sa_qwen3_config* cfg, int rank, int world, sa_qwen3** out) {
    SA_CHECK_ARG(ctx && cfg && out, "sa_qwen3_create: null argument");
    *out = nullptr;
    const sa_qwen3_config& c = *cfg;
    SA_CHECK_ARG(c.head_dim == 128, "sa_qwen3_create: head_dim %d (128 supported)", c.head_dim);
    SA_CHECK_ARG(c.hidden > 0 && c.hidden % 256 == 0 && c.inter % 64 == 0 && c.vocab > 0 && c.n_layers > 0,
                 "sa_qwen3_create: hidden=%d inter=%d vocab=%d layers=%d", c.hidden, c.inter, c.vocab, c.n_layers);
    SA_CHECK_ARG(c.hkv > 0 && c.hq % c.hkv == 0 && (c.hq / c.hkv == 1 || c.hq / c.hkv == 2 || c.hq / c.hkv == 4),
                 "sa_qwen3_create: hq=%d hkv=%d", c.hq, c.hkv);
    SA_CHECK_ARG(c.max_seq > 0, "sa_qwen3_create: max_seq=%d", c.max_seq);
    SA_CHECK_ARG(world >= 1 && world <= TP_MAX && rank >= 0 && rank < world,
                 "sa_qwen3_create_tp: rank %d of world %d (1..%d)", rank, world, TP_MAX);
    SA_CHECK_ARG(c.hkv % world == 0 && c.inter % (64 * world) == 0 && c.vocab >= world,
                 "sa_qwen3_create_tp: hkv=%d and inter/64=%d must divide over %d ranks", c.hkv, c.inter / 64, world);
    DeviceGuard guard(ctx->device);
    gemm_prepare(ctx->device);   // occupancy queries outside any later stream capture
    sa_qwen3* m = new sa_qwen3();
    m->ctx = ctx;
    m->device = ctx->device;
    m->c = c;
    m->tp_rank = rank;
    m->tp_world = world;
    m->hq = c.hq / world;
    m->hkv = c.hkv / world;
    m->inter = c.inter / world;
    m->v0 = (int)((long long)c.vocab * rank / world);
    m->vn = (int)((long long)c.vocab * (rank + 1) / world) - m->v0;
    m->QD = m->hq * c.head_dim;
    m->KD = m->hkv * c.head_dim;
    m->NQKV = m->QD + 2 * m->KD;
    m->layers.resize(c.n_layers);
    m->loaded_layer.assign(c.n_layers, false);
    const size_t H = c.hidden, I = m->inter, D = c.head_dim;
    int rc = SA_OK;
    if (!rc) rc = dalloc(&m->embed, (size_t)c.vocab * H);
    if (!rc) rc = dalloc(&m->final_norm, H);
    for (int l = 0; l < c.n_layers && !rc; ++l) {
        auto& L = m->layers[l];
        rc = dalloc(&L.in_norm, H);
        if (!rc) rc = dalloc(&L.post_norm, H);
        if (!rc) rc = dalloc(&L.q_norm, D);
        if (!rc) rc = dalloc(&L.k_norm, D);
        if (!rc) rc = dalloc(&L.wqkv, (size_t)m->NQKV * H);
        if (!rc) rc = dalloc(&L.wo, H * m->QD);
        if (!rc) rc = dalloc(&L.wgu, 2 * I * H);
        if (!rc) rc = dalloc(&L.wd, H * I);
    }
    const size_t kv = (size_t)c.n_layers * m->hkv * c.max_seq * D;
    if (!rc) rc = dalloc(&m->kc, kv);
    if (!rc) rc = dalloc(&m->vc, kv);
    if (!rc) rc = dalloc(&m->cos_t, (size_t)c.max_seq * D / 2);
    if (!rc) rc = dalloc(&m->sin_t, (size_t)c.max_seq * D / 2);
    if (!rc && cudaStreamCreateWithFlags(&m->own, cudaStreamNonBlocking) != cudaSuccess)
        rc = set_error(SA_ERR_CUDA, "stream create");
    if (!rc && (cudaEventCreateWithFlags(&m->ev_in, cudaEventDisableTiming) != cudaSuccess ||
                cudaEventCreateWithFlags(&m->ev_out, cudaEventDisableTiming) != cudaSuccess))
        rc = set_error(SA_ERR_CUDA, "event create");
    m->toks_cap = c.max_seq + 1;
    if (!rc) rc = dalloc(&m->d_state, 2);
    if (!rc) rc = dalloc(&m->d_toks, (size_t)m->toks_cap);
    if (!rc) rc = dalloc(&m->dec_scratch,
                         decode_dev_scratch_floats(ctx->num_sms, c.max_seq, (int)D, m->hq, m->hkv, nullptr));
    if (!rc) rc = dalloc(&m->dec_cnt, (size_t)(m->hq + 2 * m->hkv));
    if (!rc) rc = dalloc(&m->d_amax, 1);
    if (!rc && cudaMemsetAsync(m->d_amax, 0, sizeof(unsigned long long), ctx->stream) != cudaSuccess)
        rc = set_error(SA_ERR_CUDA, "memset");
    if (!rc && cudaMemsetAsync(m->dec_cnt, 0, (m->hq + 2 * m->hkv) * sizeof(unsigned), ctx->stream) != cudaSuccess)
        rc = set_error(SA_ERR_CUDA, "memset");
    if (!rc && world > 1) {
        // exchange buffer: flags, then two slots of `world` blocks of tp_rows rows
        m->tp_rows = std::min(c.max_seq, 8192);
        m->tp_flag_bytes = 256 + 2 * (size_t)world * H * sizeof(unsigned long long);
        const size_t bytes = m->tp_flag_bytes + 2 * (size_t)world * m->tp_rows * H * sizeof(float);
        rc = dmalloc(&m->tp_buf, bytes);
        if (!rc && cudaMemsetAsync(m->tp_buf, 0, bytes, ctx->stream) != cudaSuccess)
            rc = set_error(SA_ERR_CUDA, "memset");
        if (!rc) rc = dalloc(&m->tp_seq, 1);
        if (!rc) rc = dalloc(&m->tp_cnt, 1);
        if (!rc) rc = dalloc(&m->tp_x2, H);
        if (!rc && (cudaMemsetAsync(m->tp_seq, 0, sizeof(unsigned), ctx->stream) != cudaSuccess ||
                    cudaMemsetAsync(m->tp_cnt, 0, sizeof(unsigned), ctx->stream) != cudaSuccess))
            rc = set_error(SA_ERR_CUDA, "memset");
    }
    m->cur = ctx->stream;
    if (!rc) rc = launch_rope_table(ctx->stream, c.max_seq, (int)D, c.theta, m->cos_t, m->sin_t);
    if (!rc && cudaMemsetAsync(m->kc, 0, kv * 4, ctx->stream) != cudaSuccess) rc = set_error(SA_ERR_CUDA, "memset");
    if (!rc && cudaMemsetAsync(m->vc, 0, kv * 4, ctx->stream) != cudaSuccess) rc = set_error(SA_ERR_CUDA, "memset");
    if (!rc && cudaStreamSynchronize(ctx->stream) != cudaSuccess) rc = set_error(SA_ERR_CUDA, "sync");
    if (rc) {
        free_model(m);
        delete m;
        return rc;
    }
    m->lm_head = m->embed;
    *out = m;
    return SA_OK;
}

}  // namespace sa

SA_API int sa_qwen3_create(sa_ctx* ctx, const sa_qwen3_config* cfg, sa_qwen3** out) {
    clear_error();
    return qwen3_create_model(ctx, cfg, 0, 1, out);
}

SA_API int sa_qwen3_create_tp(sa_ctx* ctx, const sa_qwen3_config* cfg, int rank, int world, sa_qwen3** out) {
    clear_error();
    return qwen3_create_model(ctx, cfg, rank, world, out);
}

SA_API int sa_qwen3_tp_handle(sa_qwen3* m, void* handle) {
    clear_error();
    SA_CHECK_ARG(m && handle, "sa_qwen3_tp_handle: null argument");
    SA_CHECK_ARG(m->tp_world > 1, "sa_qwen3_tp_handle: not a head-parallel model (world 1)");
    static_assert(sizeof(cudaIpcMemHandle_t) <= SA_TP_HANDLE_BYTES, "IPC handle size");
    DeviceGuard guard(m->device);
    cudaIpcMemHandle_t h;
    SA_CUDA_TRY(cudaIpcGetMemHandle(&h, m->tp_buf));
    std::memset(handle, 0, SA_TP_HANDLE_BYTES);
    std::memcpy(handle, &h, sizeof(h));
    return SA_OK;
}

SA_API int sa_qwen3_tp_connect(sa_qwen3* m, const void* handles) {
    clear_error();
    SA_CHECK_ARG(m && handles, "sa_qwen3_tp_connect: null argument");
    SA_CHECK_ARG(m->tp_world > 1, "sa_qwen3_tp_connect: not a head-parallel model (world 1)");
    SA_CHECK_ARG(!m->tp_connected, "sa_qwen3_tp_connect: already connected");
    DeviceGuard guard(m->device);
    const unsigned char* hb = static_cast<const unsigned char*>(handles);
    for (int r = 0; r < m->tp_world; ++r) {
        if (r == m->tp_rank) {
            m->tp_peer[r] = m->tp_buf;
            continue;
        }
        cudaIpcMemHandle_t h;
        std::memcpy(&h, hb + (size_t)r * SA_TP_HANDLE_BYTES, sizeof(h));
        void* p = nullptr;
        const cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess) {
            cudaGetLastError();
            for (int q = 0; q < r; ++q)
                if (q != m->tp_rank && m->tp_peer[q]) cudaIpcCloseMemHandle(m->tp_peer[q]);
            std::fill(m->tp_peer, m->tp_peer + TP_MAX, nullptr);
            return set_error(SA_ERR_CUDA, "sa_qwen3_tp_connect: opening rank %d's buffer failed: %s", r,
                             cudaGetErrorString(e));
        }
        m->tp_peer[r] = p;
    }
    m->tp_connected = true;
    return SA_OK;
}

namespace sa {
namespace {
constexpr uint32_t QSP_MAGIC = 0x50535133u;   // "3QSP"
struct QspHandle {                            // the SA_QWEN3_SP_HANDLE_BYTES blob
    cudaIpcMemHandle_t buf, kc, vc;
    unsigned char uuid[16];
    int32_t rank, world, max_seq, hidden, n_layers, hkv;
    uint32_t magic;
};
static_assert(sizeof(QspHandle) <= SA_QWEN3_SP_HANDLE_BYTES, "handle size");
}  // namespace
}  // namespace sa

SA_API int sa_qwen3_create_sp(sa_ctx* ctx, const sa_qwen3_config* cfg, int rank, int world, sa_qwen3** out) {
    clear_error();
    SA_CHECK_ARG(ctx && cfg && out, "sa_qwen3_create_sp: null argument");
    SA_CHECK_ARG(world >= 1 && world <= TP_MAX && rank >= 0 && rank < world,
                 "sa_qwen3_create_sp: rank %d of world %d (1..%d)", rank, world, TP_MAX);
    SA_RC(qwen3_create_model(ctx, cfg, 0, 1, out));
    sa_qwen3* m = *out;
    m->sp_rank = rank;
    m->sp_world = world;
    if (world == 1) return SA_OK;
    DeviceGuard guard(ctx->device);
    cudaDeviceProp prop;
    m->sp_rows = std::min(cfg->max_seq, 8192);
    const size_t bytes = 256 + (size_t)m->sp_rows * cfg->hidden * sizeof(float);
    int rc = SA_OK;
    if (cudaGetDeviceProperties(&prop, ctx->device) != cudaSuccess) rc = set_error(SA_ERR_CUDA, "device properties");
    if (!rc) rc = dmalloc(&m->sp_buf, bytes);
    if (!rc) rc = dalloc(&m->sp_seq, 1);
    if (!rc) rc = dalloc(&m->sp_cnt, 1);
    if (!rc && (cudaMemset(m->sp_buf, 0, bytes) != cudaSuccess || cudaMemset(m->sp_seq, 0, 4) != cudaSuccess ||
                cudaMemset(m->sp_cnt, 0, 4) != cudaSuccess))
        rc = set_error(SA_ERR_CUDA, "memset");
    if (rc) {
        sa_qwen3_destroy(m);
        *out = nullptr;
        return rc;
    }
    std::memcpy(m->uuid, &prop.uuid, sizeof(m->uuid));
    m->sp_peer_buf[rank] = m->sp_buf;
    m->sp_peer_kc[rank] = m->kc;
    m->sp_peer_vc[rank] = m->vc;
    return SA_OK;
}

SA_API int sa_qwen3_sp_handle(sa_qwen3* m, void* handle) {
    clear_error();
    SA_CHECK_ARG(m && handle, "sa_qwen3_sp_handle: null argument");
    SA_CHECK_ARG(m->sp_world > 1, "sa_qwen3_sp_handle: not a sequence-parallel model (world 1)");
    DeviceGuard guard(m->device);
    QspHandle h;
    std::memset(&h, 0, sizeof(h));
    SA_CUDA_TRY(cudaIpcGetMemHandle(&h.buf, m->sp_buf));
    SA_CUDA_TRY(cudaIpcGetMemHandle(&h.kc, m->kc));
    SA_CUDA_TRY(cudaIpcGetMemHandle(&h.vc, m->vc));
    std::memcpy(h.uuid, m->uuid, sizeof(h.uuid));
    h.rank = m->sp_rank;
    h.world = m->sp_world;
    h.max_seq = m->c.max_seq;
    h.hidden = m->c.hidden;
    h.n_layers = m->c.n_layers;
    h.hkv = m->c.hkv;
    h.magic = QSP_MAGIC;
    std::memset(handle, 0, SA_QWEN3_SP_HANDLE_BYTES);
    std::memcpy(handle, &h, sizeof(h));
    return SA_OK;
}

SA_API int sa_qwen3_sp_connect(sa_qwen3* m, const void* handles) {
    clear_error();
    SA_CHECK_ARG(m && handles, "sa_qwen3_sp_connect: null argument");
    SA_CHECK_ARG(m->sp_world > 1, "sa_qwen3_sp_connect: not a sequence-parallel model (world 1)");
    SA_CHECK_ARG(!m->sp_connected, "sa_qwen3_sp_connect: already connected");
    DeviceGuard guard(m->device);
    const unsigned char* hb = static_cast<const unsigned char*>(handles);
    auto fail = [&](int code, const char* fmt, int r, const char* what) {
        for (int q = 0; q < TP_MAX; ++q) {
            if (q == m->sp_rank) continue;
            if (m->sp_peer_buf[q]) cudaIpcCloseMemHandle(m->sp_peer_buf[q]);
            if (m->sp_peer_kc[q]) cudaIpcCloseMemHandle(m->sp_peer_kc[q]);
            if (m->sp_peer_vc[q]) cudaIpcCloseMemHandle(m->sp_peer_vc[q]);
            m->sp_peer_buf[q] = nullptr;
            m->sp_peer_kc[q] = m->sp_peer_vc[q] = nullptr;
        }
        return set_error(code, fmt, r, what);
    };
    for (int r = 0; r < m->sp_world; ++r) {
        QspHandle h;
        std::memcpy(&h, hb + (size_t)r * SA_QWEN3_SP_HANDLE_BYTES, sizeof(h));
        if (h.magic != QSP_MAGIC) return fail(SA_ERR_ARG, "sa_qwen3_sp_connect: handle %d %s", r, "is not a model handle");
        if (h.rank != r || h.world != m->sp_world || h.max_seq != m->c.max_seq || h.hidden != m->c.hidden ||
            h.n_layers != m->c.n_layers || h.hkv != m->c.hkv)
            return fail(SA_ERR_ARG, "sa_qwen3_sp_connect: handle %d %s", r,
                        "names another rank, world size or model shape");
        if (r == m->sp_rank) continue;
        if (std::memcmp(h.uuid, m->uuid, sizeof(h.uuid)) == 0)
            return fail(SA_ERR_ARG, "sa_qwen3_sp_connect: handle %d %s", r,
                        "is on this rank's GPU (the ranks wait for one another: one GPU per rank)");
        void *pb = nullptr, *pk = nullptr, *pv = nullptr;
        if (cudaIpcOpenMemHandle(&pb, h.buf, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess ||
            cudaIpcOpenMemHandle(&pk, h.kc, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess ||
            cudaIpcOpenMemHandle(&pv, h.vc, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
            const cudaError_t e = cudaGetLastError();
            if (pb) cudaIpcCloseMemHandle(pb);
            if (pk) cudaIpcCloseMemHandle(pk);
            return fail(SA_ERR_CUDA, "sa_qwen3_sp_connect: opening rank %d's buffers failed: %s", r,
                        cudaGetErrorString(e));
        }
        m->sp_peer_buf[r] = pb;
        m->sp_peer_kc[r] = static_cast<float*>(pk);
        m->sp_peer_vc[r] = static_cast<float*>(pv);
    }
    m->sp_connected = true;
    return SA_OK;
}

SA_API int sa_qwen3_destroy(sa_qwen3* m) {
    clear_error();
    if (!m) return SA_OK;
    // the context may already be destroyed: use only the model's own state
    DeviceGuard guard(m->device);
    cudaDeviceSynchronize();
    free_model(m);
    delete m;
    return SA_OK;
}

namespace sa {

static float h2f(uint16_t h) {   // IEEE half -> float (exact)
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1Fu, man = h & 0x3FFu;
    uint32_t bits;
    if (exp == 0x1Fu) {
        bits = sign | 0x7F800000u | (man << 13);
    } else if (exp == 0) {
        if (man == 0) {
            bits = sign;
        } else {   // subnormal: renormalise
            int e = -1;
            do { man <<= 1; ++e; } while (!(man & 0x400u));
            bits = sign | ((uint32_t)(127 - 15 - e) << 23) | ((man & 0x3FFu) << 13);
        }
    } else {
        bits = sign | ((exp + 127 - 15) << 23) | (man << 13);
    }
    float f;
    std::memcpy(&f, &bits, 4);
    return f;
}

static float src_at(QwSrc s, size_t i) {
    if (s.type == QW_SRC_F32) return static_cast<const float*>(s.p)[i];
    const uint16_t u = static_cast<const uint16_t*>(s.p)[i];
    if (s.type == QW_SRC_F16) return h2f(u);
    uint32_t bits = (uint32_t)u << 16;
    float f;
    std::memcpy(&f, &bits, 4);
    return f;
}

// rows x cols elements of `src` starting at element `off` -> device bf16 rows
// of pitch dpitch_elems (2-D copy; bf16 sources go straight from host memory).
static int upload_rows(__nv_bfloat16* dst, size_t dpitch_elems, QwSrc src, size_t off, size_t rows,
                       size_t cols, size_t spitch_elems, cudaStream_t st) {
    if (src.type == QW_SRC_BF16) {
        SA_CUDA_TRY(cudaMemcpy2DAsync(dst, dpitch_elems * 2, static_cast<const uint16_t*>(src.p) + off,
                                      spitch_elems * 2, cols * 2, rows, cudaMemcpyHostToDevice, st));
        SA_CUDA_TRY(cudaStreamSynchronize(st));
        return SA_OK;
    }
    std::vector<uint16_t> tmp(rows * cols);
    for (size_t r = 0; r < rows; ++r)
        for (size_t c = 0; c < cols; ++c) tmp[r * cols + c] = f2bf(src_at(src, off + r * spitch_elems + c));
    SA_CUDA_TRY(cudaMemcpy2DAsync(dst, dpitch_elems * 2, tmp.data(), cols * 2, cols * 2, rows,
                                  cudaMemcpyHostToDevice, st));
    SA_CUDA_TRY(cudaStreamSynchronize(st));
    return SA_OK;
}

static int upload_gain(float* dst, QwSrc src, size_t n, cudaStream_t st) {
    std::vector<float> tmp(n);
    for (size_t i = 0; i < n; ++i) tmp[i] = src_at(src, i);
    return upload_f32(dst, tmp.data(), n, st);
}

int qwen3_upload_embed(sa_qwen3* m, QwSrc embed, QwSrc final_norm, QwSrc lm_head) {
    const size_t V = m->c.vocab, H = m->c.hidden;
    cudaStream_t st = m->ctx->stream;
    SA_RC(upload_rows(m->embed, H, embed, 0, V, H, H, st));
    SA_RC(upload_gain(m->final_norm, final_norm, H, st));
    bool tied = lm_head.p == nullptr || lm_head.p == embed.p;
    if (!tied && lm_head.type == embed.type) {
        const size_t bytes = V * H * (embed.type == QW_SRC_F32 ? 4 : 2);
        tied = std::memcmp(lm_head.p, embed.p, bytes) == 0;
    }
    if (tied) {
        if (m->lm_head != m->embed) cudaFree(m->lm_head);
        m->lm_head = m->embed;
    } else {
        if (m->lm_head == m->embed) SA_RC(dalloc(&m->lm_head, V * H));
        SA_RC(upload_rows(m->lm_head, H, lm_head, 0, V, H, H, st));
    }
    m->loaded_embed = true;
    return SA_OK;
}

int qwen3_upload_layer(sa_qwen3* m, int layer, QwSrc in_norm, QwSrc wq, QwSrc wk, QwSrc wv, QwSrc q_norm,
                       QwSrc k_norm, QwSrc wo, QwSrc post_norm, QwSrc w_gate, QwSrc w_up, QwSrc w_down) {
    const sa_qwen3_config& c = m->c;
    const size_t H = c.hidden, I = c.inter, D = c.head_dim;
    // this rank's share: q / k / v rows of its heads, the matching o_proj
    // columns, gate / up rows and down_proj columns of its intermediate features
    const size_t QDl = m->QD, KDl = m->KD, Il = m->inter, QDg = (size_t)c.hq * D, r = m->tp_rank;
    auto& L = m->layers[layer];
    cudaStream_t st = m->ctx->stream;
    SA_RC(upload_gain(L.in_norm, in_norm, H, st));
    SA_RC(upload_gain(L.post_norm, post_norm, H, st));
    SA_RC(upload_gain(L.q_norm, q_norm, D, st));
    SA_RC(upload_gain(L.k_norm, k_norm, D, st));
    // [q; k; v] rows, as qwen3_loader.cpp builds qkv_projs
    SA_RC(upload_rows(L.wqkv, H, wq, r * QDl * H, QDl, H, H, st));
    SA_RC(upload_rows(L.wqkv + QDl * H, H, wk, r * KDl * H, KDl, H, H, st));
    SA_RC(upload_rows(L.wqkv + (QDl + KDl) * H, H, wv, r * KDl * H, KDl, H, H, st));
    SA_RC(upload_rows(L.wo, QDl, wo, r * QDl, H, QDl, QDg, st));
    // gate/up interleaved in blocks of 32 rows: [gate 32b..32b+31 ; up 32b..32b+31]:
    // the blocks of gate land at even block slots, those of up at odd ones
    SA_RC(upload_rows(L.wgu, 2 * 32 * H, w_gate, r * Il * H, Il / 32, 32 * H, 32 * H, st));
    SA_RC(upload_rows(L.wgu + 32 * H, 2 * 32 * H, w_up, r * Il * H, Il / 32, 32 * H, 32 * H, st));
    SA_RC(upload_rows(L.wd, Il, w_down, r * Il, H, Il, I, st));
    m->loaded_layer[layer] = true;
    return SA_OK;
}

}  // namespace sa

SA_API int sa_qwen3_set_embed(sa_qwen3* m, const float* embed, const float* final_norm, const float* lm_head) {
    clear_error();
    SA_CHECK_ARG(m && embed && final_norm, "sa_qwen3_set_embed: null argument");
    DeviceGuard guard(m->ctx->device);
    return qwen3_upload_embed(m, {embed, QW_SRC_F32}, {final_norm, QW_SRC_F32}, {lm_head, QW_SRC_F32});
}

SA_API int sa_qwen3_set_layer(sa_qwen3* m, int layer, const float* in_norm, const float* wq, const float* wk,
                              const float* wv, const float* q_norm, const float* k_norm, const float* wo,
                              const float* post_norm, const float* w_gate, const float* w_up, const float* w_down) {
    clear_error();
    SA_CHECK_ARG(m && layer >= 0 && layer < m->c.n_layers, "sa_qwen3_set_layer: layer %d", layer);
    SA_CHECK_ARG(in_norm && wq && wk && wv && q_norm && k_norm && wo && post_norm && w_gate && w_up && w_down,
                 "sa_qwen3_set_layer: null weight");
    DeviceGuard guard(m->ctx->device);
    auto F = [](const float* p) { return QwSrc{p, QW_SRC_F32}; };
    return qwen3_upload_layer(m, layer, F(in_norm), F(wq), F(wk), F(wv), F(q_norm), F(k_norm), F(wo),
                              F(post_norm), F(w_gate), F(w_up), F(w_down));
}

SA_API int sa_qwen3_reset(sa_qwen3* m) {
    clear_error();
    SA_CHECK_ARG(m, "sa_qwen3_reset: null model");
    m->cache_len = 0;   // rows past cache_len are never read; no zeroing needed
    return SA_OK;
}

SA_API int sa_qwen3_cache_len(sa_qwen3* m) { return m ? m->cache_len : -1; }

// Host [hkv][seq_stride][D] <-> device rows 0..rows-1 of one layer's cache
// ([hkv][max_seq][D]), one 2-D copy per tensor on the context's stream.
static int copy_kv_layer(sa_qwen3* m, int layer, float* hk, float* hv, int rows, int seq_stride, bool to_host) {
    const size_t D = m->c.head_dim;
    const size_t layer_kv = (size_t)m->hkv * m->c.max_seq * D;
    float* dk = m->kc + (size_t)layer * layer_kv;
    float* dv = m->vc + (size_t)layer * layer_kv;
    if (rows == 0) return SA_OK;
    const size_t hpitch = (size_t)seq_stride * D * 4, dpitch = (size_t)m->c.max_seq * D * 4;
    const size_t width = (size_t)rows * D * 4;
    cudaStream_t st = m->ctx->stream;
    if (to_host) {
        SA_CUDA_TRY(cudaMemcpy2DAsync(hk, hpitch, dk, dpitch, width, m->hkv, cudaMemcpyDeviceToHost, st));
        SA_CUDA_TRY(cudaMemcpy2DAsync(hv, hpitch, dv, dpitch, width, m->hkv, cudaMemcpyDeviceToHost, st));
    } else {
        SA_CUDA_TRY(cudaMemcpy2DAsync(dk, dpitch, hk, hpitch, width, m->hkv, cudaMemcpyHostToDevice, st));
        SA_CUDA_TRY(cudaMemcpy2DAsync(dv, dpitch, hv, hpitch, width, m->hkv, cudaMemcpyHostToDevice, st));
    }
    return sync_and_check(m->ctx);
}

SA_API int sa_qwen3_read_kv(sa_qwen3* m, int layer, float* k_out, float* v_out, int seq_stride) {
    clear_error();
    SA_CHECK_ARG(m && k_out && v_out, "sa_qwen3_read_kv: null argument");
    SA_CHECK_ARG(layer >= 0 && layer < m->c.n_layers, "sa_qwen3_read_kv: layer %d of %d", layer, m->c.n_layers);
    SA_CHECK_ARG(seq_stride >= m->cache_len, "sa_qwen3_read_kv: seq_stride %d < cache length %d", seq_stride,
                 m->cache_len);
    DeviceGuard guard(m->ctx->device);
    return copy_kv_layer(m, layer, k_out, v_out, m->cache_len, seq_stride, true);
}

SA_API int sa_qwen3_write_kv(sa_qwen3* m, int layer, const float* k, const float* v, int len, int seq_stride) {
    clear_error();
    SA_CHECK_ARG(m && (len == 0 || (k && v)), "sa_qwen3_write_kv: null argument");
    SA_CHECK_ARG(layer >= 0 && layer < m->c.n_layers, "sa_qwen3_write_kv: layer %d of %d", layer, m->c.n_layers);
    SA_CHECK_ARG(len >= 0 && len <= m->c.max_seq && seq_stride >= len,
                 "sa_qwen3_write_kv: len %d (max_seq %d, seq_stride %d)", len, m->c.max_seq, seq_stride);
    DeviceGuard guard(m->ctx->device);
    return copy_kv_layer(m, layer, const_cast<float*>(k), const_cast<float*>(v), len, seq_stride, false);
}

SA_API int sa_qwen3_set_cache_len(sa_qwen3* m, int len) {
    clear_error();
    SA_CHECK_ARG(m, "sa_qwen3_set_cache_len: null model");
    SA_CHECK_ARG(len >= 0 && len <= m->c.max_seq, "sa_qwen3_set_cache_len: len %d (max_seq %d)", len, m->c.max_seq);
    m->cache_len = len;
    return SA_OK;
}

// Run `body` on the model's own (capturable) stream, ordered after the
// context's stream and before anything the caller issues on it afterwards.
template <typename F>
static int on_own_stream(sa_qwen3* m, F body) {
    SA_CUDA_TRY(cudaEventRecord(m->ev_in, m->ctx->stream));
    SA_CUDA_TRY(cudaStreamWaitEvent(m->own, m->ev_in, 0));
    m->cur = m->own;
    int rc = body();
    m->cur = m->ctx->stream;
    if (cudaEventRecord(m->ev_out, m->own) != cudaSuccess ||
        cudaStreamWaitEvent(m->ctx->stream, m->ev_out, 0) != cudaSuccess)
        return rc ? rc : set_error(SA_ERR_CUDA, "stream join failed");
    return rc;
}

// Capture `body` (launches on m->own) into a graph; *exec receives it.
template <typename F>
static int capture(sa_qwen3* m, cudaGraphExec_t* exec, F body) {
    cudaGraph_t g = nullptr;
    SA_CUDA_TRY(cudaStreamBeginCapture(m->own, cudaStreamCaptureModeThreadLocal));
    const int rc = body();
    const cudaError_t e = cudaStreamEndCapture(m->own, &g);
    if (rc) {
        if (g) cudaGraphDestroy(g);
        return rc;
    }
    if (e != cudaSuccess) return set_error(SA_ERR_CUDA, "graph capture failed: %s", cudaGetErrorString(e));
    const cudaError_t e2 = cudaGraphInstantiate(exec, g, 0);
    cudaGraphDestroy(g);
    if (e2 != cudaSuccess) {
        *exec = nullptr;
        return set_error(SA_ERR_CUDA, "graph instantiate failed: %s", cudaGetErrorString(e2));
    }
    return SA_OK;
}

SA_API int sa_qwen3_forward(sa_qwen3* m, const int64_t* ids, int S, int use_cache, float* logits, int logits_mode,
                            unsigned flags) {
    clear_error();
    SA_CHECK_ARG(m && ids, "sa_qwen3_forward: null argument");
    SA_CHECK_ARG(S >= 1, "sa_qwen3_forward: S = %d", S);
    SA_CHECK_ARG(logits_mode >= 0 && logits_mode <= 2, "sa_qwen3_forward: logits_mode %d", logits_mode);
    SA_CHECK_ARG(logits_mode == 2 || logits, "sa_qwen3_forward: logits is NULL");
    SA_CHECK_ARG(m->loaded_embed, "sa_qwen3_forward: embedding not loaded");
    for (int l = 0; l < m->c.n_layers; ++l)
        SA_CHECK_ARG(m->loaded_layer[l], "sa_qwen3_forward: layer %d not loaded", l);
    SA_CHECK_ARG(m->tp_world == 1 || m->tp_connected, "sa_qwen3_forward: head-parallel ranks not connected");
    SA_CHECK_ARG(m->tp_world == 1 || S <= m->tp_rows, "sa_qwen3_forward: S = %d > %d rows per head-parallel forward",
                 S, m->tp_rows);
    SA_CHECK_ARG(m->sp_world == 1 || m->sp_connected, "sa_qwen3_forward: sequence-parallel ranks not connected");
    SA_CHECK_ARG(!sp_split(m, S) || S <= m->sp_rows,
                 "sa_qwen3_forward: S = %d > %d rows per sequence-parallel forward", S, m->sp_rows);
    DeviceGuard guard(m->ctx->device);
    m->cur = m->ctx->stream;
    const int pos0 = use_cache ? m->cache_len : 0;
    const int kv_row0 = m->cache_len;      // cache-free forwards use the rows after the live prefix
    if (kv_row0 + S > m->c.max_seq)
        return set_error(SA_ERR_FULL, "KV cache full, cannot place %d tokens after %d cached (max_seq %d)", S,
                         m->cache_len, m->c.max_seq);
    const bool host = flags & SA_HOST_PTRS;
    if (host)
        for (int s = 0; s < S; ++s)
            if (ids[s] < 0 || ids[s] >= m->c.vocab)
                return set_error(SA_ERR_RANGE, "Embedding index out of range: ids[%d] = %lld", s, (long long)ids[s]);
    SA_RC(ensure_acts(m, S));
    if (S >= tc_attn_min_rows()) SA_RC(ensure_tc(m, S));
    const int r0 = logits_mode == 1 ? S - 1 : 0, n = logits_mode == 1 ? 1 : S;
    if (logits_mode != 2) SA_RC(ensure_logits(m, n));
    const cudaMemcpyKind in_kind = host ? cudaMemcpyHostToDevice : cudaMemcpyDeviceToDevice;
    const bool sp = sp_split(m, S);
    int s0 = 0, s1 = S;
    if (sp) sp_share(m, S, &s0, &s1);
    int rc = on_own_stream(m, [&]() -> int {
        SA_CUDA_TRY(cudaMemcpyAsync(m->ids, ids + s0, (size_t)(s1 - s0) * 8, in_kind, m->own));
        auto body = [&]() -> int {
            if (sp) {
                const float* xa = nullptr;
                SA_RC(run_prompt_sp(m, S, pos0, kv_row0, &xa));
                if (logits_mode != 2) SA_RC(run_head(m, r0, n, nullptr, xa));
                return SA_OK;
            }
            SA_RC(run_layers(m, S, pos0, nullptr, kv_row0));
            if (logits_mode != 2) SA_RC(run_head(m, r0, n));
            return tp_close_segment(m);
        };
        if (use_cache) return body();
        // qwen3_forward without a cache has a fixed schedule per (S, logits
        // mode): the second call of a shape captures it, later ones replay
        const std::pair<int, int> key{S, logits_mode * 1048576 + kv_row0};
        auto it = m->pf_graphs.find(key);
        if (it == m->pf_graphs.end() && m->pf_seen.count(key)) {
            cudaGraphExec_t ex = nullptr;
            SA_RC(capture(m, &ex, body));
            it = m->pf_graphs.emplace(key, ex).first;
        }
        if (it != m->pf_graphs.end()) {
            SA_CUDA_TRY(cudaGraphLaunch(it->second, m->own));
            return SA_OK;
        }
        m->pf_seen.insert(key);
        return body();
    });
    if (rc) return rc;
    if (use_cache) m->cache_len = pos0 + S;
    if (logits_mode != 2)
        SA_CUDA_TRY(cudaMemcpyAsync(logits, m->logits, (size_t)n * m->c.vocab * 4,
                                    host ? cudaMemcpyDeviceToHost : cudaMemcpyDeviceToDevice, m->ctx->stream));
    if (host) return sync_and_check(m->ctx);
    return SA_OK;
}

// One decode step driven entirely by device state: the token in ids[0] at
// cache position d_state[0] goes through every layer (K/V appended), the
// lm_head GEMV and argmax write the next token back to ids[0], which is
// recorded at d_toks[d_state[1]]; then both counters advance.
static int decode_step_dev(sa_qwen3* m) {
    SA_RC(run_layers(m, 1, 0, m->d_state));
    SA_RC(run_head(m, 0, 1, m->ids));
    SA_RC(launch_advance(m->cur, m->d_state, m->ids, m->d_toks, m->toks_cap, 1, true));
    return SA_OK;
}

// The single-launch decode step's buffers and per-layer weight table; false
// when this model or device cannot use it (the graph of separate kernels
// serves then).
static bool mega_ready(sa_qwen3* m) {
    if (m->mega_grid < 0 || m->tp_world > 1) return false;
    if (m->mega_grid > 0) return true;
    const sa_qwen3_config& c = m->c;
    const int grid = mega_supported(c, m->ctx->num_sms) ? mega_grid(m->ctx->device) : 0;
    if (grid < c.hkv) {
        m->mega_grid = -1;
        return false;
    }
    std::vector<MegaLayer> ls(c.n_layers);
    for (int l = 0; l < c.n_layers; ++l) {
        const auto& L = m->layers[l];
        ls[l] = MegaLayer{L.wqkv, L.wo, L.wgu, L.wd, L.in_norm, L.post_norm, L.q_norm, L.k_norm};
    }
    const size_t part = (size_t)c.hkv * (grid / c.hkv) * (c.hq / c.hkv) * (c.head_dim + 2);
    bool ok = dmalloc(reinterpret_cast<void**>(&m->d_mlayers), ls.size() * sizeof(MegaLayer)) == SA_OK &&
              dalloc(&m->mpart, part) == SA_OK && dalloc(&m->mhead_cnt, (size_t)c.hkv) == SA_OK &&
              dalloc(&m->mgbar, 4) == SA_OK;
    ok = ok && cudaMemcpy(m->d_mlayers, ls.data(), ls.size() * sizeof(MegaLayer), cudaMemcpyHostToDevice) ==
                   cudaSuccess &&
         cudaMemset(m->mhead_cnt, 0, (size_t)c.hkv * sizeof(unsigned)) == cudaSuccess &&
         cudaMemset(m->mgbar, 0, 4 * sizeof(unsigned)) == cudaSuccess;
    if (!ok) {
        cudaGetLastError();
        clear_error();
        m->mega_grid = -1;
        return false;
    }
    m->mega_grid = grid;
    return true;
}

static int launch_mega_step(sa_qwen3* m, cudaStream_t st) {
    const sa_qwen3_config& c = m->c;
    MegaParams q;
    q.layers = m->d_mlayers;
    q.L = c.n_layers; q.H = c.hidden; q.I = c.inter; q.hq = c.hq; q.hkv = c.hkv; q.V = c.vocab;
    q.max_seq = c.max_seq; q.eps = c.eps;
    q.embed = m->embed; q.lm_head = m->lm_head; q.final_norm = m->final_norm;
    q.kc = m->kc; q.vc = m->vc; q.cos_t = m->cos_t; q.sin_t = m->sin_t;
    q.x = m->x; q.qkv = m->qkv; q.attn = m->attn; q.act = m->act; q.part = m->mpart;
    q.head_cnt = m->mhead_cnt; q.amax = m->d_amax; q.gbar = m->mgbar;
    q.state = m->d_state; q.ids = m->ids; q.toks = m->d_toks; q.toks_cap = m->toks_cap;
    q.status = m->ctx->status;
    return launch_decode_mega(st, m->mega_grid, q);
}

SA_API int sa_qwen3_generate(sa_qwen3* m, const int64_t* prompt, int S, int n_new, int64_t* out_tokens,
                             unsigned flags) {
    clear_error();
    SA_CHECK_ARG(m && prompt && out_tokens && S >= 1 && n_new >= 0, "sa_qwen3_generate: bad argument");
    SA_CHECK_ARG(m->loaded_embed, "sa_qwen3_generate: embedding not loaded");
    for (int l = 0; l < m->c.n_layers; ++l)
        SA_CHECK_ARG(m->loaded_layer[l], "sa_qwen3_generate: layer %d not loaded", l);
    SA_CHECK_ARG(m->tp_world == 1 || m->tp_connected, "sa_qwen3_generate: head-parallel ranks not connected");
    SA_CHECK_ARG(m->tp_world == 1 || S <= m->tp_rows, "sa_qwen3_generate: S = %d > %d prompt rows (head-parallel)",
                 S, m->tp_rows);
    SA_CHECK_ARG(m->sp_world == 1 || m->sp_connected, "sa_qwen3_generate: sequence-parallel ranks not connected");
    SA_CHECK_ARG(!sp_split(m, S) || S <= m->sp_rows, "sa_qwen3_generate: S = %d > %d prompt rows (sequence-parallel)",
                 S, m->sp_rows);
    DeviceGuard guard(m->ctx->device);
    m->cur = m->ctx->stream;
    if (m->cache_len + S + n_new > m->c.max_seq + 1)
        return set_error(SA_ERR_FULL, "KV cache full: %d + %d prompt + %d new > max_seq %d", m->cache_len, S, n_new,
                         m->c.max_seq);
    const bool host = flags & SA_HOST_PTRS;
    if (host)
        for (int s = 0; s < S; ++s)
            if (prompt[s] < 0 || prompt[s] >= m->c.vocab)
                return set_error(SA_ERR_RANGE, "Embedding index out of range: prompt[%d]", s);
    SA_RC(ensure_acts(m, S));
    if (S >= tc_attn_min_rows()) SA_RC(ensure_tc(m, S));
    SA_RC(ensure_logits(m, 1));
    const int pos0 = m->cache_len;
    int rc = on_own_stream(m, [&]() -> int {
        cudaStream_t st = m->own;
        const bool sp = sp_split(m, S);
        int s0 = 0, s1 = S;
        if (sp) sp_share(m, S, &s0, &s1);
        SA_CUDA_TRY(cudaMemcpyAsync(m->ids, prompt + s0, (size_t)(s1 - s0) * 8,
                                    host ? cudaMemcpyHostToDevice : cudaMemcpyDeviceToDevice, st));
        // the prompt: split over sequence-parallel ranks (their gathered
        // residual rows then feed the head on every rank), else whole
        const float* xa = nullptr;
        if (sp)
            SA_RC(run_prompt_sp(m, S, pos0, pos0, &xa));
        else
            SA_RC(run_layers(m, S, pos0));
        if (n_new == 0) {
            SA_RC(run_head(m, S - 1, 1, nullptr, xa));
            return sp ? SA_OK : tp_close_segment(m);
        }
        SA_RC(run_head(m, S - 1, 1, m->ids, xa));
        const int state[2] = {pos0 + S, 0};
        SA_CUDA_TRY(cudaMemcpyAsync(m->d_state, state, sizeof(state), cudaMemcpyHostToDevice, st));
        SA_RC(launch_advance(st, m->d_state, m->ids, m->d_toks, m->toks_cap, 0, false));   // first new token
        if (n_new > 1 && mega_ready(m)) {
            // one cooperative launch per token (sa_qwen3_mega.cu)
            SA_CUDA_TRY(cudaMemsetAsync(m->mgbar, 0, 4 * sizeof(unsigned), st));
            for (int t = 1; t < n_new; ++t) SA_RC(launch_mega_step(m, st));
        } else {
            if (n_new > 1 && !m->dec_graph)
                SA_RC(capture(m, &m->dec_graph, [&]() { return decode_step_dev(m); }));
            for (int t = 1; t < n_new; ++t) SA_CUDA_TRY(cudaGraphLaunch(m->dec_graph, st));
        }
        SA_CUDA_TRY(cudaMemcpyAsync(out_tokens, m->d_toks, (size_t)n_new * 8,
                                    host ? cudaMemcpyDeviceToHost : cudaMemcpyDeviceToDevice, st));
        return SA_OK;
    });
    if (rc) return rc;
    m->cache_len = pos0 + S + (n_new > 0 ? n_new - 1 : 0);
    if (host) return sync_and_check(m->ctx);
    return SA_OK;
}
