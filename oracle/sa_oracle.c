/*
 * sa_oracle.c -- CPU restatement of the reference's streaming-attention and
 * Qwen3 forward arithmetic.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity checker for the CUDA
 * path.  Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline
 * leg may load it.  The product library (libsa_cuda.so) never links or calls
 * it; there is no CPU fallback anywhere in the product.
 *
 * Parity pin: every function here is checked against the reference's own
 * implementation compiled from its sources (oracle/_ref/libsa_ref.so, built by
 * oracle/Makefile) and against the committed fixtures in tests/golden/ that
 * were generated from that build (tests/golden/make_golden.py).
 *
 * All arithmetic is fp32 in the reference's loop order (sequential dot
 * products, libm expf/sqrtf/powf/cosf/sinf), so agreement with the reference
 * is at the level of rounding of the compiler's FMA contraction.  Citations
 * are path:line inside the reference project.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define ORC_EXPORT __attribute__((visibility("default")))

/* ------------------------------------------------------------------------ */
/* Online softmax block update.                                              */
/* Follows utils/softmax_online.h:40-87 (state init m=-inf, l=1 at :22-28).  */
/* The output accumulator is kept normalised by l after every block.         */
/* ------------------------------------------------------------------------ */
ORC_EXPORT void orc_online_block(const float* scores, const float* values,
                                 float* m, float* l, float* out,
                                 int n, int d) {
    float m_new = *m;
    for (int i = 0; i < n; ++i) m_new = fmaxf(m_new, scores[i]);
    float sum_exp = 0.0f;
    for (int i = 0; i < n; ++i) sum_exp += expf(scores[i] - m_new);
    float scale_old = expf(*m - m_new);
    float l_new = (*l) * scale_old + sum_exp;
    float alpha_old = ((*l) * scale_old) / l_new;
    float alpha_new = 1.0f / l_new;
    for (int j = 0; j < d; ++j) out[j] *= alpha_old;
    for (int i = 0; i < n; ++i) {
        float w = alpha_new * expf(scores[i] - m_new);
        const float* vr = values + (size_t)i * d;
        for (int j = 0; j < d; ++j) out[j] += w * vr[j];
    }
    *m = m_new;
    *l = l_new;
}

/* ------------------------------------------------------------------------ */
/* Naive three-pass attention, unscaled scores (scale=1 reproduces it).      */
/* Follows attention/src/naive_serial.cpp:18-72.                             */
/* ------------------------------------------------------------------------ */
ORC_EXPORT void orc_naive_attention(const float* q, const float* k, const float* v,
                                    int T, int d, float scale, float* out) {
    float* s = (float*)malloc(sizeof(float) * (T > 0 ? T : 1));
    for (int i = 0; i < T; ++i) {
        float acc = 0.0f;
        const float* kr = k + (size_t)i * d;
        for (int j = 0; j < d; ++j) acc += q[j] * kr[j];
        s[i] = acc * scale;
    }
    float mx = -INFINITY;
    for (int i = 0; i < T; ++i) mx = fmaxf(mx, s[i]);
    float sum = 0.0f;
    for (int i = 0; i < T; ++i) { s[i] = expf(s[i] - mx); sum += s[i]; }
    for (int i = 0; i < T; ++i) s[i] /= sum;
    for (int j = 0; j < d; ++j) out[j] = 0.0f;
    for (int i = 0; i < T; ++i) {
        const float* vr = v + (size_t)i * d;
        for (int j = 0; j < d; ++j) out[j] += s[i] * vr[j];
    }
    free(s);
}

/* ------------------------------------------------------------------------ */
/* Partial state over rows [t0, t1) in blocks of `block` rows.               */
/* Follows attention/src/streaming_omp.cpp:53-89 (process_blocks_serial).    */
/* A `scale` multiplies each score (1.0 reproduces the unscaled reference).  */
/* Empty ranges leave the initial state (m=-inf, l=1, O=0).                  */
/* ------------------------------------------------------------------------ */
ORC_EXPORT void orc_partial(const float* q, const float* k, const float* v,
                            int t0, int t1, int d, int block, float scale,
                            float* m, float* l, float* o) {
    *m = -INFINITY;
    *l = 1.0f;
    for (int j = 0; j < d; ++j) o[j] = 0.0f;
    float* s = (float*)malloc(sizeof(float) * (block > 0 ? block : 1));
    int n = t1 - t0;
    for (int b = 0; b < (n + block - 1) / block; ++b) {
        int bs = t0 + b * block;
        int be = bs + block < t1 ? bs + block : t1;
        for (int i = 0; i < be - bs; ++i) {
            const float* kr = k + (size_t)(bs + i) * d;
            float acc = 0.0f;
            for (int j = 0; j < d; ++j) acc += q[j] * kr[j];
            s[i] = acc * scale;
        }
        orc_online_block(s, v + (size_t)bs * d, m, l, o, be - bs, d);
    }
    free(s);
}

/* Streaming single-query attention: attention/src/streaming_serial.cpp:20-71 */
ORC_EXPORT void orc_streaming_attention(const float* q, const float* k, const float* v,
                                        int T, int d, int block, float scale, float* out) {
    float m, l;
    orc_partial(q, k, v, 0, T, d, block, scale, &m, &l, out);
}

/* ------------------------------------------------------------------------ */
/* Associative merge of two partial states (left <- left (+) right).         */
/* Follows attention/src/streaming_omp.cpp:27-48 (merge_partial_results);    */
/* the same merge is used across ranks at streaming_mpi.cpp:295-305.         */
/* ------------------------------------------------------------------------ */
ORC_EXPORT void orc_merge(float* m, float* l, float* o,
                          float m2, float l2, const float* o2, int d) {
    float m_new = fmaxf(*m, m2);
    float sl = expf(*m - m_new);
    float sr = expf(m2 - m_new);
    float l_new = (*l) * sl + l2 * sr;
    float al = ((*l) * sl) / l_new;
    float ar = (l2 * sr) / l_new;
    for (int j = 0; j < d; ++j) o[j] = o[j] * al + o2[j] * ar;
    *m = m_new;
    *l = l_new;
}

/* ------------------------------------------------------------------------ */
/* Chunked streaming attention with the reference's OpenMP chunk arithmetic, */
/* run sequentially: n_chunks = max(1, min(threads, ceil(T/(2*block)))),     */
/* chunk = ceil(T/n_chunks), then merge in chunk order into a fresh state.   */
/* Follows attention/src/streaming_omp.cpp:99-154.                           */
/* ------------------------------------------------------------------------ */
ORC_EXPORT void orc_streaming_chunked(const float* q, const float* k, const float* v,
                                      int T, int d, int block, int n_threads,
                                      float scale, float* out) {
    int n_chunks = (T + block * 2 - 1) / (block * 2);
    if (n_threads < n_chunks) n_chunks = n_threads;
    if (n_chunks < 1) n_chunks = 1;
    int chunk = (T + n_chunks - 1) / n_chunks;
    float M = -INFINITY, L = 1.0f;
    float* po = (float*)malloc(sizeof(float) * d);
    for (int j = 0; j < d; ++j) out[j] = 0.0f;
    for (int c = 0; c < n_chunks; ++c) {
        int ts = c * chunk;
        int te = ts + chunk < T ? ts + chunk : T;
        float pm, pl;
        if (ts >= te) { pm = -INFINITY; pl = 1.0f; for (int j = 0; j < d; ++j) po[j] = 0.0f; }
        else orc_partial(q, k, v, ts, te, d, block, scale, &pm, &pl, po);
        orc_merge(&M, &L, out, pm, pl, po, d);
    }
    free(po);
}

/* ------------------------------------------------------------------------ */
/* GQA single-token decode over a head-major KV cache.                       */
/* q: [hq, d]; k, v: head h at k + h*kv_head_stride, rows of d; out [hq, d].  */
/* Query head h reads KV head h / (hq/hkv): the repeat_kv mapping of         */
/* tensor_cpp/src/qwen3_ops.cpp:194-234 (h_out = h*n_rep + r).  The score is */
/* scaled before the softmax as in tensor_cpp/src/ops.cpp:544 (the decode    */
/* wrapper at ops.cpp:1010 scales the output instead, which is wrong).       */
/* Per head it is the streaming recurrence of streaming_serial.cpp:20-71.    */
/* ------------------------------------------------------------------------ */
ORC_EXPORT void orc_gqa_decode(const float* q, const float* k, const float* v,
                               long long kv_head_stride, int T, int d, int hq, int hkv,
                               int block, float scale, float* out) {
    int rep = hq / hkv;
    for (int h = 0; h < hq; ++h) {
        int kh = h / rep;
        orc_streaming_attention(q + (size_t)h * d, k + (size_t)kh * kv_head_stride,
                                v + (size_t)kh * kv_head_stride, T, d, block, scale,
                                out + (size_t)h * d);
    }
}

/* ------------------------------------------------------------------------ */
/* Causal block-wise prefill (online softmax per query row).                 */
/* Follows tensor_cpp/src/ops.cpp:1027-1112 (process_q_block_causal) and     */
/* :1383-1450 (self_attention_streaming_blockwise), generalised with a query */
/* position offset: key j is visible to query i iff j <= q_pos0 + i.         */
/* Layouts are token-major with explicit strides (elements):                 */
/*   q[i, h, :] at q + i*q_tok + h*q_head, k/v likewise, out likewise.       */
/* GQA: query head h reads KV head h / (hq/hkv).                             */
/* ------------------------------------------------------------------------ */
ORC_EXPORT void orc_causal_prefill(const float* q, const float* k, const float* v,
                                   float* out, int Sq, int Skv, int q_pos0,
                                   int hq, int hkv, int d,
                                   long long q_tok, long long q_head,
                                   long long kv_tok, long long kv_head,
                                   long long o_tok, long long o_head,
                                   int kv_block, float scale) {
    int rep = hq / hkv;
    #pragma omp parallel for collapse(2) schedule(dynamic, 4)
    for (int h = 0; h < hq; ++h) {
        for (int i = 0; i < Sq; ++i) {
            int kh = h / rep;
            const float* qi = q + (size_t)i * q_tok + (size_t)h * q_head;
            float* oi = out + (size_t)i * o_tok + (size_t)h * o_head;
            float m = -INFINITY, l = 1.0f;
            float* s = (float*)malloc(sizeof(float) * kv_block);
            float* vb = (float*)malloc(sizeof(float) * (size_t)kv_block * d);
            for (int j = 0; j < d; ++j) oi[j] = 0.0f;
            int last = q_pos0 + i;               /* inclusive */
            if (last > Skv - 1) last = Skv - 1;
            for (int b0 = 0; b0 <= last; b0 += kv_block) {
                int b1 = b0 + kv_block - 1 < last ? b0 + kv_block - 1 : last;
                int n = b1 - b0 + 1;
                for (int r = 0; r < n; ++r) {
                    const float* kr = k + (size_t)(b0 + r) * kv_tok + (size_t)kh * kv_head;
                    const float* vr = v + (size_t)(b0 + r) * kv_tok + (size_t)kh * kv_head;
                    float acc = 0.0f;
                    for (int j = 0; j < d; ++j) acc += qi[j] * kr[j];
                    s[r] = acc * scale;
                    memcpy(vb + (size_t)r * d, vr, sizeof(float) * d);
                }
                orc_online_block(s, vb, &m, &l, oi, n, d);
            }
            free(s);
            free(vb);
        }
    }
}

/* ======================================================================== */
/* Qwen3 forward                                                             */
/* ======================================================================== */

/* x / sqrt(mean(x^2) + eps) * w per row: tensor_cpp/src/ops.cpp:375-418 */
ORC_EXPORT void orc_rms_norm(const float* x, const float* w, int rows, int n,
                             float eps, float* y) {
    for (int r = 0; r < rows; ++r) {
        const float* xr = x + (size_t)r * n;
        float* yr = y + (size_t)r * n;
        float ms = 0.0f;
        for (int i = 0; i < n; ++i) ms += xr[i] * xr[i];
        ms /= (float)n;
        float rms = sqrtf(ms + eps);
        for (int i = 0; i < n; ++i) yr[i] = xr[i] / rms;
        if (w) for (int i = 0; i < n; ++i) yr[i] *= w[i];
    }
}

/* y[s, o] = sum_i x[s, i] * W[o, i]: tensor_cpp/src/ops.cpp:315-369.       */
/* Every output is one sum over i in increasing order, as the reference's   */
/* loop forms it; the register tiles below only interleave independent      */
/* sums (4 rows x ORC_OB outputs) so that they overlap in the FMA pipeline  */
/* -- the bits of every output are those of the plain loop.                */
#define ORC_OB 8
#define ORC_MAX_D 256   /* head_dim bound of the Qwen3 forward */
static void lin_tile(const float* x, const float* W, int in_f, int out_f, int s0, int ns,
                     int o0, float* y) {
    int no = out_f - o0 < ORC_OB ? out_f - o0 : ORC_OB;
    if (no == ORC_OB && ns == 4) {
        float acc[4][ORC_OB] = {{0}};
        const float* x0 = x + (size_t)s0 * in_f;
        const float* w0 = W + (size_t)o0 * in_f;
        for (int i = 0; i < in_f; ++i) {
            float xv[4];
            for (int a = 0; a < 4; ++a) xv[a] = x0[(size_t)a * in_f + i];
            for (int b = 0; b < ORC_OB; ++b) {
                float w = w0[(size_t)b * in_f + i];
                for (int a = 0; a < 4; ++a) acc[a][b] += xv[a] * w;
            }
        }
        for (int a = 0; a < 4; ++a)
            for (int b = 0; b < ORC_OB; ++b) y[(size_t)(s0 + a) * out_f + o0 + b] = acc[a][b];
        return;
    }
    for (int a = 0; a < ns; ++a) {
        const float* xr = x + (size_t)(s0 + a) * in_f;
        if (no == ORC_OB) {
            float acc[ORC_OB] = {0};
            const float* w0 = W + (size_t)o0 * in_f;
            for (int i = 0; i < in_f; ++i)
                for (int b = 0; b < ORC_OB; ++b) acc[b] += xr[i] * w0[(size_t)b * in_f + i];
            for (int b = 0; b < ORC_OB; ++b) y[(size_t)(s0 + a) * out_f + o0 + b] = acc[b];
        } else {
            for (int b = 0; b < no; ++b) {
                const float* wr = W + (size_t)(o0 + b) * in_f;
                float acc = 0.0f;
                for (int i = 0; i < in_f; ++i) acc += xr[i] * wr[i];
                y[(size_t)(s0 + a) * out_f + o0 + b] = acc;
            }
        }
    }
}

ORC_EXPORT void orc_linear(const float* x, const float* W, int rows, int in_f, int out_f,
                           float* y) {
    int nrb = (rows + 3) / 4, nob = (out_f + ORC_OB - 1) / ORC_OB;
    #pragma omp parallel for collapse(2) schedule(static)
    for (int rb = 0; rb < nrb; ++rb)
        for (int ob = 0; ob < nob; ++ob) {
            int s0 = rb * 4;
            int ns = rows - s0 < 4 ? rows - s0 : 4;
            lin_tile(x, W, in_f, out_f, s0, ns, ob * ORC_OB, y);
        }
}

/* inv_freq_i = 1/theta^(i/D); cos/sin[pos, i] = cos/sin(pos*inv_freq_i)     */
/* tensor_cpp/src/qwen3_ops.cpp:70-104 (theta 1e6 from :564 and :959).        */
ORC_EXPORT void orc_rope_tables(int n_pos, int head_dim, float theta,
                                float* cos_t, float* sin_t) {
    int half = head_dim / 2;
    float* inv = (float*)malloc(sizeof(float) * half);
    for (int i = 0; i < half; ++i)
        inv[i] = 1.0f / powf(theta, (float)i / (float)head_dim);
    for (int p = 0; p < n_pos; ++p)
        for (int i = 0; i < half; ++i) {
            float a = (float)p * inv[i];
            cos_t[(size_t)p * half + i] = cosf(a);
            sin_t[(size_t)p * half + i] = sinf(a);
        }
    free(inv);
}

/* Per-head RMS norm (eps inside the sqrt, qwen3_ops.cpp:355-369) followed by */
/* rotate-half RoPE at position pos (qwen3_ops.cpp:30-64, 110-188).          */
static void qk_norm_rope(float* x, const float* w, int d, float eps,
                         const float* cos_row, const float* sin_row) {
    float ss = 0.0f;
    for (int i = 0; i < d; ++i) ss += x[i] * x[i];
    float rms = sqrtf(ss / (float)d + eps);
    float tmp[512];
    for (int i = 0; i < d; ++i) tmp[i] = (x[i] / rms) * w[i];
    int half = d / 2;
    for (int i = 0; i < half; ++i) {
        float c = cos_row[i], s = sin_row[i];
        float x1 = tmp[i], x2 = tmp[half + i];
        x[i] = x1 * c + (-x2) * s;
        x[half + i] = x2 * c + x1 * s;
    }
}

typedef struct {
    int vocab, hidden, n_layers, hq, hkv, head_dim, inter;
    float eps, theta;
} orc_qwen3_cfg;

/* Offsets of one layer's tensors inside the packed per-layer fp32 block:    */
/* in_norm[H] q[Hq*D,H] k[Hkv*D,H] v[Hkv*D,H] q_norm[D] k_norm[D]            */
/* o[H,Hq*D] post_norm[H] gate[I,H] up[I,H] down[H,I]                        */
ORC_EXPORT long long orc_qwen3_layer_floats(const orc_qwen3_cfg* c) {
    long long H = c->hidden, D = c->head_dim, I = c->inter;
    return H + (long long)c->hq * D * H + 2LL * c->hkv * D * H + 2 * D +
           H * (long long)c->hq * D + H + 3LL * I * H;
}

/*
 * One forward over S new tokens at cache position `pos0` (0 = prefill).
 * Follows qwen3_forward_with_cache (tensor_cpp/src/qwen3_ops.cpp:936-1014) and
 * qwen3_decoder_layer_with_cache (:620-934) with the STANDARD attention type:
 * RMSNorm -> Q/K/V linear -> QK-norm -> RoPE at offset pos0 -> cache append ->
 * masked softmax attention (ops.cpp:514-641, scale 1/sqrt(D)) -> o_proj ->
 * residual -> RMSNorm -> SwiGLU MLP (qwen3_ops.cpp:265-296) -> residual.
 * Generalisation: S>1 with pos0>0 uses the causal rule j <= pos0+i (the
 * reference assumes one new token when the cache is non-empty, :809,826).
 * With pos0 = 0 and no cache this is qwen3_forward (:537-614).
 * kc/vc: [n_layers, hkv, max_seq, D] or NULL (no cache; then pos0 must be 0).
 * logits: [S, vocab] if all_logits else [1, vocab] for the last token only.
 */
ORC_EXPORT int orc_qwen3_forward(const orc_qwen3_cfg* c, const float* embed,
                                 const float* layer_w, const float* final_norm,
                                 const float* lm_head, const int64_t* ids, int S,
                                 float* kc, float* vc, int max_seq, int pos0,
                                 int all_logits, float* logits) {
    const int H = c->hidden, D = c->head_dim, HQ = c->hq, HKV = c->hkv, I = c->inter;
    if (D > ORC_MAX_D) return -4;
    const int QD = HQ * D, KD = HKV * D;
    const int total = pos0 + S;
    if (!kc && pos0 != 0) return -1;
    if (kc && total > max_seq) return -2;
    for (int s = 0; s < S; ++s)
        if (ids[s] < 0 || ids[s] >= c->vocab) return -3;

    float* x = (float*)malloc(sizeof(float) * (size_t)S * H);
    float* xn = (float*)malloc(sizeof(float) * (size_t)S * H);
    float* q = (float*)malloc(sizeof(float) * (size_t)S * QD);
    float* kk = (float*)malloc(sizeof(float) * (size_t)S * KD);
    float* vv = (float*)malloc(sizeof(float) * (size_t)S * KD);
    float* att = (float*)malloc(sizeof(float) * (size_t)S * QD);
    float* tmp = (float*)malloc(sizeof(float) * (size_t)S * (H > I ? H : I));
    float* g = (float*)malloc(sizeof(float) * (size_t)S * I);
    float* u = (float*)malloc(sizeof(float) * (size_t)S * I);
    float* cos_t = (float*)malloc(sizeof(float) * (size_t)total * (D / 2));
    float* sin_t = (float*)malloc(sizeof(float) * (size_t)total * (D / 2));
    /* full K/V history for this layer (token-major [total, HKV, D]) */
    float* kh = (float*)malloc(sizeof(float) * (size_t)total * KD);
    float* vh = (float*)malloc(sizeof(float) * (size_t)total * KD);
    orc_rope_tables(total, D, c->theta, cos_t, sin_t);

    /* embedding: ops.cpp:278-309 */
    for (int s = 0; s < S; ++s)
        memcpy(x + (size_t)s * H, embed + (size_t)ids[s] * H, sizeof(float) * H);

    long long LF = orc_qwen3_layer_floats(c);
    float scale = 1.0f / sqrtf((float)D);
    for (int L = 0; L < c->n_layers; ++L) {
        const float* w = layer_w + (size_t)L * LF;
        const float* in_norm = w;            w += H;
        const float* wq = w;                 w += (size_t)QD * H;
        const float* wk = w;                 w += (size_t)KD * H;
        const float* wv = w;                 w += (size_t)KD * H;
        const float* qn = w;                 w += D;
        const float* kn = w;                 w += D;
        const float* wo = w;                 w += (size_t)H * QD;
        const float* post_norm = w;          w += H;
        const float* wg = w;                 w += (size_t)I * H;
        const float* wu = w;                 w += (size_t)I * H;
        const float* wd = w;

        orc_rms_norm(x, in_norm, S, H, c->eps, xn);
        orc_linear(xn, wq, S, H, QD, q);
        orc_linear(xn, wk, S, H, KD, kk);
        orc_linear(xn, wv, S, H, KD, vv);
        for (int s = 0; s < S; ++s) {
            int p = pos0 + s;
            for (int h = 0; h < HQ; ++h)
                qk_norm_rope(q + (size_t)s * QD + h * D, qn, D, 1e-6f,
                             cos_t + (size_t)p * (D / 2), sin_t + (size_t)p * (D / 2));
            for (int h = 0; h < HKV; ++h)
                qk_norm_rope(kk + (size_t)s * KD + h * D, kn, D, 1e-6f,
                             cos_t + (size_t)p * (D / 2), sin_t + (size_t)p * (D / 2));
        }
        /* history: cached prefix + new rows; then append (kv_cache.h:94-130) */
        for (int t = 0; t < pos0; ++t)
            for (int h = 0; h < HKV; ++h) {
                size_t src = (((size_t)L * HKV + h) * max_seq + t) * D;
                memcpy(kh + (size_t)t * KD + h * D, kc + src, sizeof(float) * D);
                memcpy(vh + (size_t)t * KD + h * D, vc + src, sizeof(float) * D);
            }
        for (int s = 0; s < S; ++s)
            for (int h = 0; h < HKV; ++h) {
                memcpy(kh + (size_t)(pos0 + s) * KD + h * D, kk + (size_t)s * KD + h * D, sizeof(float) * D);
                memcpy(vh + (size_t)(pos0 + s) * KD + h * D, vv + (size_t)s * KD + h * D, sizeof(float) * D);
                if (kc) {
                    size_t dst = (((size_t)L * HKV + h) * max_seq + pos0 + s) * D;
                    memcpy(kc + dst, kk + (size_t)s * KD + h * D, sizeof(float) * D);
                    memcpy(vc + dst, vv + (size_t)s * KD + h * D, sizeof(float) * D);
                }
            }
        /* masked softmax attention, one query row at a time (ops.cpp:514-641) */
        int rep = HQ / HKV;
        #pragma omp parallel for collapse(2) schedule(dynamic, 2)
        for (int s = 0; s < S; ++s) {
            for (int h = 0; h < HQ; ++h) {
                float* sc = (float*)malloc(sizeof(float) * total);
                const float* qi = q + (size_t)s * QD + h * D;
                int kvh = h / rep;
                int last = pos0 + s;
                float mx = -INFINITY;
                /* scores: one sum over e per key, 8 keys interleaved */
                int j = 0;
                for (; j + 8 <= total; j += 8) {
                    float acc[8] = {0};
                    const float* k0 = kh + (size_t)j * KD + kvh * D;
                    for (int e = 0; e < D; ++e)
                        for (int b = 0; b < 8; ++b) acc[b] += qi[e] * k0[(size_t)b * KD + e];
                    for (int b = 0; b < 8; ++b) sc[j + b] = acc[b] * scale + (j + b <= last ? 0.0f : -INFINITY);
                }
                for (; j < total; ++j) {
                    const float* kr = kh + (size_t)j * KD + kvh * D;
                    float acc = 0.0f;
                    for (int e = 0; e < D; ++e) acc += qi[e] * kr[e];
                    sc[j] = acc * scale + (j <= last ? 0.0f : -INFINITY);
                }
                for (j = 0; j < total; ++j) mx = fmaxf(mx, sc[j]);
                float sum = 0.0f;
                for (j = 0; j < total; ++j) { sc[j] = expf(sc[j] - mx); sum += sc[j]; }
                for (j = 0; j < total; ++j) sc[j] /= sum;
                float* oi = att + (size_t)s * QD + h * D;
                /* P.V: one sum over j per output column, the columns side by side */
                float acc[ORC_MAX_D];
                for (int e = 0; e < D; ++e) acc[e] = 0.0f;
                for (j = 0; j < total; ++j) {
                    const float* vr = vh + (size_t)j * KD + kvh * D;
                    for (int e = 0; e < D; ++e) acc[e] += sc[j] * vr[e];
                }
                for (int e = 0; e < D; ++e) oi[e] = acc[e];
                free(sc);
            }
        }
        orc_linear(att, wo, S, QD, H, tmp);
        for (size_t i = 0; i < (size_t)S * H; ++i) x[i] = x[i] + tmp[i];
        orc_rms_norm(x, post_norm, S, H, c->eps, xn);
        orc_linear(xn, wg, S, H, I, g);
        orc_linear(xn, wu, S, H, I, u);
        for (size_t i = 0; i < (size_t)S * I; ++i) {
            float sg = g[i] * (1.0f / (1.0f + expf(-g[i])));
            g[i] = sg * u[i];
        }
        orc_linear(g, wd, S, I, H, tmp);
        for (size_t i = 0; i < (size_t)S * H; ++i) x[i] = x[i] + tmp[i];
    }
    orc_rms_norm(x, final_norm, S, H, c->eps, xn);
    if (all_logits) orc_linear(xn, lm_head, S, H, c->vocab, logits);
    else orc_linear(xn + (size_t)(S - 1) * H, lm_head, 1, H, c->vocab, logits);

    free(x); free(xn); free(q); free(kk); free(vv); free(att); free(tmp);
    free(g); free(u); free(cos_t); free(sin_t); free(kh); free(vh);
    return 0;
}

/* bf16 round-to-nearest-even of an fp32 value (for building bf16 inputs the */
/* oracle also sees exactly); NaN is passed through quiet.                   */
ORC_EXPORT void orc_round_bf16(const float* x, float* y, long long n) {
    for (long long i = 0; i < n; ++i) {
        uint32_t u;
        memcpy(&u, &x[i], 4);
        if ((u & 0x7fffffffu) > 0x7f800000u) { u |= 0x00400000u; }
        else { u += 0x7fffu + ((u >> 16) & 1u); }
        u &= 0xffff0000u;
        memcpy(&y[i], &u, 4);
    }
}
