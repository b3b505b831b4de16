// ref_shim.cpp -- extern "C" entry points onto the reference implementation.
//
// TEST INFRASTRUCTURE ONLY.  oracle/Makefile compiles this file together with
// the reference's own sources (attention/src/*.cpp and tensor_cpp/src/*.cpp,
// read in place from the reference tree) into oracle/_ref/libsa_ref.so.  It
// lets the Python tests pin oracle/sa_oracle.c against the reference itself,
// and lets bench.py time the reference's CPU path as its baseline arm.
// Nothing in the product library links or calls this.
//
// Each wrapper only converts raw pointers to the reference's containers
// (std::vector / tensor_cpp::Tensor) and back; the arithmetic is entirely the
// reference's.
#include <cstdint>
#include <cstring>
#include <cmath>
#include <exception>
#include <string>
#include <vector>

#include "attention.h"                 // attention/src/attention.h
#include "tensor_cpp/ops.h"            // tensor_cpp/include/tensor_cpp/ops.h
#include "tensor_cpp/qwen3_ops.h"
#include "tensor_cpp/qwen3_loader.h"
#include "tensor_cpp/qwen3_ops_avx.h"
#include "tensor_cpp/kv_cache.h"

using tensor_cpp::Shape;
using tensor_cpp::Tensor;
// TensorL is declared at global scope (tensor_cpp/include/tensor_cpp/ops.h:35)
namespace q3 = tensor_cpp::qwen3;

#define REF_EXPORT extern "C" __attribute__((visibility("default")))

static thread_local std::string g_err;
REF_EXPORT const char* ref_last_error() { return g_err.c_str(); }

static void put(const std::vector<float>& r, float* out) {
    std::memcpy(out, r.data(), r.size() * sizeof(float));
}

// ---- attention/src/attention.h:27-208 ------------------------------------
REF_EXPORT void ref_naive_attention_serial(const float* q, const float* k, const float* v,
                                           int T, int d, float* out) {
    put(naive_attention_serial(q, k, v, T, d), out);
}
REF_EXPORT void ref_naive_attention_omp(const float* q, const float* k, const float* v,
                                        int T, int d, int threads, float* out) {
    put(naive_attention_omp(q, k, v, T, d, threads), out);
}
REF_EXPORT void ref_streaming_attention_serial(const float* q, const float* k, const float* v,
                                               int T, int d, int block, float* out) {
    put(streaming_attention_serial(q, k, v, T, d, block), out);
}
REF_EXPORT void ref_streaming_attention_omp(const float* q, const float* k, const float* v,
                                            int T, int d, int block, int threads, float* out) {
    put(streaming_attention_omp(q, k, v, T, d, block, threads), out);
}

// GQA decode on the reference's CPU path: one streaming_attention_omp call per
// query head on its KV head's rows (the repeat_kv mapping h -> h / n_rep of
// tensor_cpp/src/qwen3_ops.cpp:194-234, without materialising the copy).  The
// attention.h kernels do not scale scores, so q is pre-scaled by `scale`.
REF_EXPORT void ref_gqa_decode_omp(const float* q, const float* k, const float* v,
                                   long long kv_head_stride, int T, int d, int hq, int hkv,
                                   int block, int threads, float scale, float* out) {
    int rep = hq / hkv;
    std::vector<float> qs(d);
    for (int h = 0; h < hq; ++h) {
        for (int j = 0; j < d; ++j) qs[j] = q[(size_t)h * d + j] * scale;
        int kh = h / rep;
        put(streaming_attention_omp(qs.data(), k + (size_t)kh * kv_head_stride,
                                    v + (size_t)kh * kv_head_stride, T, d, block, threads),
            out + (size_t)h * d);
    }
}

// ---- tensor_cpp ops: causal prefill ------------------------------------
// q [1, hq, S, d]; k/v [1, hkv, S, d] (head-major, as the reference holds
// them); repeat_kv (qwen3_ops.cpp:194) then the block-wise causal online
// softmax (ops.cpp:1383-1450) or the masked standard attention (ops.cpp:514).
REF_EXPORT int ref_causal_prefill(const float* q, const float* k, const float* v, int S,
                                  int hq, int hkv, int d, float scale, int q_block,
                                  int kv_block, int standard, float* out) {
    try {
        Tensor tq(std::vector<float>(q, q + (size_t)hq * S * d), Shape({1, (size_t)hq, (size_t)S, (size_t)d}));
        Tensor tk(std::vector<float>(k, k + (size_t)hkv * S * d), Shape({1, (size_t)hkv, (size_t)S, (size_t)d}));
        Tensor tv(std::vector<float>(v, v + (size_t)hkv * S * d), Shape({1, (size_t)hkv, (size_t)S, (size_t)d}));
        Tensor kr = q3::repeat_kv(tk, hq / hkv);
        Tensor vr = q3::repeat_kv(tv, hq / hkv);
        Tensor o;
        if (standard == 1) {
            Tensor mask = q3::create_causal_mask(S).view(Shape({1, 1, (size_t)S, (size_t)S}));
            o = tensor_cpp::ops::self_attention(tq, kr, vr, &mask, scale);
        } else if (standard == 2) {
            o = tensor_cpp::ops::self_attention_streaming_blockwise_avx2(tq, kr, vr, scale, q_block, kv_block);
        } else {
            o = tensor_cpp::ops::self_attention_streaming_blockwise(tq, kr, vr, scale, q_block, kv_block);
        }
        std::memcpy(out, o.data(), o.size() * sizeof(float));
        return 0;
    } catch (const std::exception& e) {
        g_err = e.what();
        return -1;
    }
}

// ---- Qwen3 ---------------------------------------------------------------
struct RefCfg {  // mirrors orc_qwen3_cfg in oracle/sa_oracle.c
    int vocab, hidden, n_layers, hq, hkv, head_dim, inter;
    float eps, theta;
};

struct RefModel {
    RefCfg c;
    Tensor embed, norm, lm_head;
    std::vector<q3::Qwen3LayerWeights> layers;
};

static Tensor mk(const float*& p, size_t r, size_t c) {
    size_t n = r * (c ? c : 1);
    Tensor t(std::vector<float>(p, p + n), c ? Shape({r, c}) : Shape({r}));
    p += n;
    return t;
}

// Packed per-layer layout is the one documented at orc_qwen3_layer_floats.
REF_EXPORT void* ref_qwen3_create(const RefCfg* c, const float* embed, const float* layer_w,
                                  const float* final_norm, const float* lm_head) {
    auto* m = new RefModel();
    m->c = *c;
    size_t H = c->hidden, D = c->head_dim, I = c->inter, QD = c->hq * D, KD = c->hkv * D;
    m->embed = Tensor(std::vector<float>(embed, embed + (size_t)c->vocab * H), Shape({(size_t)c->vocab, H}));
    m->norm = Tensor(std::vector<float>(final_norm, final_norm + H), Shape({H}));
    m->lm_head = Tensor(std::vector<float>(lm_head, lm_head + (size_t)c->vocab * H), Shape({(size_t)c->vocab, H}));
    const float* p = layer_w;
    for (int L = 0; L < c->n_layers; ++L) {
        q3::Qwen3LayerWeights w;
        w.input_layernorm_weight = mk(p, H, 0);
        w.q_proj = mk(p, QD, H);
        w.k_proj = mk(p, KD, H);
        w.v_proj = mk(p, KD, H);
        w.q_norm_weight = mk(p, D, 0);
        w.k_norm_weight = mk(p, D, 0);
        w.o_proj = mk(p, H, QD);
        w.post_attention_layernorm_weight = mk(p, H, 0);
        w.gate_proj = mk(p, I, H);
        w.up_proj = mk(p, I, H);
        w.down_proj = mk(p, H, I);
        // combined [q; k; v] rows, as qwen3_loader.cpp:257-283 builds it
        std::vector<float> qkv;
        qkv.reserve((QD + 2 * KD) * H);
        qkv.insert(qkv.end(), w.q_proj.data(), w.q_proj.data() + QD * H);
        qkv.insert(qkv.end(), w.k_proj.data(), w.k_proj.data() + KD * H);
        qkv.insert(qkv.end(), w.v_proj.data(), w.v_proj.data() + KD * H);
        w.qkv_projs = Tensor(std::move(qkv), Shape({QD + 2 * KD, H}));
        m->layers.push_back(std::move(w));
    }
    return m;
}

// The reference's own safetensors loader (load_qwen3_weights,
// qwen3_loader.cpp:140-297): weights and the configuration it implies (the
// loader fixes 28 layers, 16/8 heads, head_dim 128; eps / theta are the
// forwards' 1e-6 / 1e6).
REF_EXPORT void* ref_qwen3_load(const char* path, RefCfg* out_cfg) {
    try {
        q3::Qwen3Weights w = q3::load_qwen3_weights(path);
        auto* m = new RefModel();
        m->c.vocab = (int)w.vocab_size;
        m->c.hidden = (int)w.hidden_size;
        m->c.n_layers = (int)w.num_layers;
        m->c.hq = (int)w.num_attention_heads;
        m->c.hkv = (int)w.num_key_value_heads;
        m->c.head_dim = (int)w.head_dim;
        m->c.inter = (int)w.layers[0].gate_proj.shape()[0];
        m->c.eps = 1e-6f;
        m->c.theta = 1000000.0f;
        m->embed = std::move(w.embed_tokens);
        m->norm = std::move(w.norm_weight);
        m->lm_head = std::move(w.lm_head);
        m->layers = std::move(w.layers);
        if (out_cfg) *out_cfg = m->c;
        return m;
    } catch (const std::exception& e) {
        g_err = e.what();
        return nullptr;
    }
}

REF_EXPORT void ref_qwen3_destroy(void* h) { delete static_cast<RefModel*>(h); }

static TensorL ids_tensor(const int64_t* ids, int S) {
    std::vector<long> v(ids, ids + S);
    return TensorL(v, Shape({1, (size_t)S}));
}

// method: 0 = qwen3_forward (qwen3_ops.cpp:537), 1 = avx2::qwen3_forward_avx
// (qwen3_ops_avx.cpp:383).  logits [S, vocab].
REF_EXPORT int ref_qwen3_forward(void* h, const int64_t* ids, int S, int method, float* logits) {
    auto* m = static_cast<RefModel*>(h);
    try {
        TensorL t = ids_tensor(ids, S);
        Tensor out = method == 1
            ? q3::avx2::qwen3_forward_avx(t, m->embed, m->layers, m->norm, m->lm_head,
                                          m->c.n_layers, m->c.hq, m->c.hkv, m->c.head_dim, m->c.eps)
            : q3::qwen3_forward(t, m->embed, m->layers, m->norm, m->lm_head,
                                m->c.n_layers, m->c.hq, m->c.hkv, m->c.head_dim, m->c.eps);
        std::memcpy(logits, out.data(), out.size() * sizeof(float));
        return 0;
    } catch (const std::exception& e) {
        g_err = e.what();
        return -1;
    }
}

// KV-cache forward (qwen3_ops.cpp:936-1014, STANDARD attention), with the
// reference's KVCache object (kv_cache.h:27-238) owned by the handle.
REF_EXPORT void* ref_kv_create(int layers, int hkv, int head_dim, int max_seq) {
    return new q3::KVCache(layers, 1, hkv, head_dim, max_seq);
}
REF_EXPORT void ref_kv_destroy(void* kv) { delete static_cast<q3::KVCache*>(kv); }
REF_EXPORT long long ref_kv_len(void* kv) { return (long long)static_cast<q3::KVCache*>(kv)->current_seq_len; }

REF_EXPORT int ref_qwen3_forward_cached(void* h, void* kv, const int64_t* ids, int S,
                                        int method, float* logits) {
    auto* m = static_cast<RefModel*>(h);
    try {
        TensorL t = ids_tensor(ids, S);
        auto* cache = static_cast<q3::KVCache*>(kv);
        Tensor out = method == 1
            ? q3::avx2::qwen3_forward_avx_with_cache(t, cache, m->embed, m->layers, m->norm, m->lm_head,
                                                     m->c.n_layers, m->c.hq, m->c.hkv, m->c.head_dim,
                                                     m->c.eps, q3::AttentionType::STANDARD)
            : q3::qwen3_forward_with_cache(t, cache, m->embed, m->layers, m->norm, m->lm_head,
                                           m->c.n_layers, m->c.hq, m->c.hkv, m->c.head_dim,
                                           m->c.eps, q3::AttentionType::STANDARD);
        std::memcpy(logits, out.data(), out.size() * sizeof(float));
        return 0;
    } catch (const std::exception& e) {
        g_err = e.what();
        return -1;
    }
}
