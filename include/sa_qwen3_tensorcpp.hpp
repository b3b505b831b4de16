/*
 * sa_qwen3_tensorcpp.hpp -- the CUDA method for the reference's Qwen3 model
 * API: tensor_cpp::qwen3::cuda::qwen3_forward_cuda and
 * qwen3_forward_cuda_with_cache take exactly the arguments of
 * qwen3::qwen3_forward and qwen3::qwen3_forward_with_cache
 * (tensor_cpp/include/tensor_cpp/qwen3_ops.h:242-333) and return the same
 * logits Tensor [batch, seq_len, vocab] on the host.
 *
 * Header-only, for a build of the reference: include it after
 * "tensor_cpp/qwen3_ops.h" (it uses that header's Tensor, TensorL,
 * Qwen3LayerWeights, KVCache and AttentionType) and link libsa_cuda.so.  The
 * method dispatch of benchmark_qwen3's forward_with_method
 * (tensor_cpp/tests/benchmark/benchmark_qwen3.cpp:262-378) gains one branch
 * that calls these with its own arguments.
 *
 * Contract kept from the reference:
 *  - weights are host fp32 tensors in the reference's shapes; they are
 *    uploaded (as bf16, exact for bf16 checkpoints) once per weights object
 *    (keyed by the addresses of token_embedding and layers) on first use;
 *    q_proj/k_proj/v_proj are used when present, else the rows of qkv_projs;
 *  - forward_with_cache appends the S new tokens' K/V at
 *    kv_cache->current_seq_len and advances it by S (kv_cache.h:94-137), with
 *    RoPE positions starting there; the device cache is kept in a table
 *    keyed by the KVCache* : when the host cache's current_seq_len is 0 the
 *    device cache restarts, and when it differs from the device length (a
 *    cache filled by another method, or a different KVCache) the host
 *    cache's rows 0..current_seq_len-1 are uploaded first.  The host K/V
 *    tensors are written only by sync_kv_to_host(); a cache whose rows live
 *    only on the GPU and had to be dropped (a cache-free forward that needed
 *    the room, another KVCache taking the device cache, a larger max_seq_len
 *    rebuilding the model) is recognised on its next use by its host rows
 *    being unwritten (row current_seq_len-1 of layer 0 all zero, which K
 *    after QK-norm and RoPE never is) and raises std::runtime_error instead
 *    of continuing from them;
 *  - errors are exceptions: std::invalid_argument for shapes the CUDA path
 *    does not take, std::out_of_range for token ids outside the vocabulary
 *    (as ops::embedding, ops.cpp:296), std::runtime_error for a full cache
 *    (kv_cache.h:109-111) and for CUDA failures.
 * Attention type: STANDARD and STREAMING compute the same softmax attention;
 * the GPU always runs its online-softmax kernels.  Batch: 1 with a cache;
 * without a cache each batch row is an independent forward.
 * Threading: one model per weights object, guarded by a mutex.
 */
#ifndef SA_QWEN3_TENSORCPP_HPP
#define SA_QWEN3_TENSORCPP_HPP

#include <algorithm>
#include <cstdint>
#include <map>
#include <memory>
#include <mutex>
#include <stdexcept>
#include <string>
#include <utility>
#include <vector>

#include "sa_cuda.h"

namespace tensor_cpp {
namespace qwen3 {
namespace cuda {

namespace sa_detail {

inline void throw_rc(int rc, const char* what) {
    if (rc == SA_OK) return;
    const std::string msg = std::string(what) + ": " + sa_last_error();
    if (rc == SA_ERR_ARG) throw std::invalid_argument(msg);
    if (rc == SA_ERR_RANGE) throw std::out_of_range(msg);
    throw std::runtime_error(msg);
}

struct Model {
    sa_ctx* ctx = nullptr;
    sa_qwen3* m = nullptr;
    sa_qwen3_config cfg{};
    const KVCache* bound = nullptr;   // the host cache the device cache mirrors
    ~Model() {
        if (m) sa_qwen3_destroy(m);
        if (ctx) sa_ctx_destroy(ctx);
    }
};

struct Registry {
    std::mutex mu;
    std::map<std::pair<const void*, const void*>, std::unique_ptr<Model>> models;
    int device = 0;
};

// The model's device cache is about to be dropped (reset for room or a
// rebuild) or handed to another KVCache.
inline void drop_cache(Model& md) { md.bound = nullptr; }

// Host rows 0..len-1 hold K/V that some method wrote (row len-1 of layer 0,
// every head, is not all zero).
inline bool host_rows_written(const KVCache& kv, size_t len) {
    const float* k = kv.key_cache[0].data();
    for (size_t h = 0; h < kv.num_kv_heads; ++h) {
        const float* row = k + (h * kv.max_seq_len + (len - 1)) * kv.head_dim;
        for (size_t i = 0; i < kv.head_dim; ++i)
            if (row[i] != 0.f) return true;
    }
    return false;
}

inline Registry& registry() {
    static Registry r;
    return r;
}

// Every entry point holds the one adapter lock for its whole call (a model
// runs one forward at a time anyway).
inline std::unique_lock<std::mutex> lock_all() { return std::unique_lock<std::mutex>(registry().mu); }

// Upload one weights object into a new device model holding max_seq tokens.
inline std::unique_ptr<Model> build(const Tensor& token_embedding, const std::vector<Qwen3LayerWeights>& layers,
                                    const Tensor& norm_weight, const Tensor& lm_head, size_t num_layers,
                                    size_t hq, size_t hkv, size_t head_dim, float eps, int max_seq, int device) {
    if (token_embedding.shape().ndim() != 2 || layers.size() < num_layers || num_layers == 0)
        throw std::invalid_argument("qwen3_forward_cuda: embedding must be [vocab, hidden] and layers >= num_layers");
    const size_t V = token_embedding.shape()[0], H = token_embedding.shape()[1];
    const size_t QD = hq * head_dim, KD = hkv * head_dim;
    const Qwen3LayerWeights& l0 = layers[0];
    if (l0.gate_proj.shape().ndim() != 2) throw std::invalid_argument("qwen3_forward_cuda: gate_proj must be 2-D");
    std::unique_ptr<Model> md(new Model);
    md->cfg.vocab = (int)V;
    md->cfg.hidden = (int)H;
    md->cfg.n_layers = (int)num_layers;
    md->cfg.hq = (int)hq;
    md->cfg.hkv = (int)hkv;
    md->cfg.head_dim = (int)head_dim;
    md->cfg.inter = (int)l0.gate_proj.shape()[0];
    md->cfg.eps = eps;
    md->cfg.theta = 1000000.0f;   // the reference's forwards build RoPE with theta 1e6 (qwen3_ops.cpp:560,959)
    md->cfg.max_seq = max_seq;
    throw_rc(sa_ctx_create(device, &md->ctx), "sa_ctx_create");
    throw_rc(sa_qwen3_create(md->ctx, &md->cfg, &md->m), "sa_qwen3_create");
    const bool tied = lm_head.size() == 0 || lm_head.data() == token_embedding.data();
    if (!tied && lm_head.size() != V * H) throw std::invalid_argument("qwen3_forward_cuda: lm_head shape");
    throw_rc(sa_qwen3_set_embed(md->m, token_embedding.data(), norm_weight.data(), tied ? nullptr : lm_head.data()),
             "sa_qwen3_set_embed");
    for (size_t i = 0; i < num_layers; ++i) {
        const Qwen3LayerWeights& L = layers[i];
        const float *wq, *wk, *wv;
        if (L.q_proj.size() == QD * H && L.k_proj.size() == KD * H && L.v_proj.size() == KD * H) {
            wq = L.q_proj.data();
            wk = L.k_proj.data();
            wv = L.v_proj.data();
        } else if (L.qkv_projs.size() == (QD + 2 * KD) * H) {
            // rows [q (QD) | k (KD) | v (KD)] of hidden columns each (qwen3_ops.cpp:470-498)
            wq = L.qkv_projs.data();
            wk = wq + QD * H;
            wv = wk + KD * H;
        } else {
            throw std::invalid_argument("qwen3_forward_cuda: layer " + std::to_string(i) +
                                        " has neither q/k/v_proj nor qkv_projs of the expected size");
        }
        throw_rc(sa_qwen3_set_layer(md->m, (int)i, L.input_layernorm_weight.data(), wq, wk, wv,
                                    L.q_norm_weight.data(), L.k_norm_weight.data(), L.o_proj.data(),
                                    L.post_attention_layernorm_weight.data(), L.gate_proj.data(), L.up_proj.data(),
                                    L.down_proj.data()),
                 "sa_qwen3_set_layer");
    }
    return md;
}

// The model for these weights, (re)built when it cannot hold max_seq tokens.
// Called with the adapter lock held.
inline Model& model_for(const Tensor& token_embedding, const std::vector<Qwen3LayerWeights>& layers,
                        const Tensor& norm_weight, const Tensor& lm_head, size_t num_layers, size_t hq, size_t hkv,
                        size_t head_dim, float eps, int max_seq) {
    Registry& r = registry();
    auto key = std::make_pair((const void*)token_embedding.data(), (const void*)layers.data());
    auto it = r.models.find(key);
    if (it != r.models.end() && it->second->cfg.max_seq >= max_seq) return *it->second;
    if (it != r.models.end()) drop_cache(*it->second);
    const int cap = it != r.models.end() ? std::max(max_seq, 2 * it->second->cfg.max_seq) : std::max(max_seq, 4096);
    auto md = build(token_embedding, layers, norm_weight, lm_head, num_layers, hq, hkv, head_dim, eps, cap, r.device);
    Model& ref = *md;
    r.models[key] = std::move(md);
    return ref;
}

inline std::vector<int64_t> row_ids(const TensorL& ids, size_t b, size_t S) {
    std::vector<int64_t> out(S);
    for (size_t s = 0; s < S; ++s) out[s] = (int64_t)ids[b * S + s];
    return out;
}

}  // namespace sa_detail

/* GPU used for models built from now on (default 0). */
inline void set_device(int device) {
    auto lk = sa_detail::lock_all();
    sa_detail::registry().device = device;
}

/* Free every device model (weights and caches). */
inline void release() {
    auto lk = sa_detail::lock_all();
    sa_detail::Registry& r = sa_detail::registry();
    r.models.clear();
}

namespace sa_detail {

// qwen3_forward_cuda with the adapter lock held.
inline Tensor forward_nocache(const TensorL& input_ids, const Tensor& token_embedding,
                              const std::vector<Qwen3LayerWeights>& layers, const Tensor& norm_weight,
                              const Tensor& lm_head, size_t num_layers, size_t hq, size_t hkv, size_t head_dim,
                              float eps) {
    if (input_ids.shape().ndim() != 2) throw std::invalid_argument("qwen3_forward_cuda: input_ids must be [B, S]");
    const size_t B = input_ids.shape()[0], S = input_ids.shape()[1];
    Model& md = model_for(token_embedding, layers, norm_weight, lm_head, num_layers, hq, hkv, head_dim, eps, (int)S);
    const size_t V = (size_t)md.cfg.vocab;
    Tensor logits(Shape{B, S, V});
    for (size_t b = 0; b < B; ++b) {
        const std::vector<int64_t> ids = row_ids(input_ids, b, S);
        // the cache-free forward uses the rows after the live cache: make room
        if (sa_qwen3_cache_len(md.m) + (int)S > md.cfg.max_seq) {
            drop_cache(md);
            throw_rc(sa_qwen3_reset(md.m), "sa_qwen3_reset");
        }
        throw_rc(sa_qwen3_forward(md.m, ids.data(), (int)S, 0, logits.data() + b * S * V, 0, SA_HOST_PTRS),
                 "qwen3_forward_cuda");
    }
    return logits;
}

}  // namespace sa_detail

/* qwen3::qwen3_forward (qwen3_ops.h:250-261): logits [B, S, vocab] for every
 * position, no cache. */
inline Tensor qwen3_forward_cuda(const TensorL& input_ids, const Tensor& token_embedding,
                                 const std::vector<Qwen3LayerWeights>& layers, const Tensor& norm_weight,
                                 const Tensor& lm_head, size_t num_layers, size_t num_attention_heads,
                                 size_t num_key_value_heads, size_t head_dim, float rms_norm_eps) {
    auto lk = sa_detail::lock_all();
    return sa_detail::forward_nocache(input_ids, token_embedding, layers, norm_weight, lm_head, num_layers,
                                      num_attention_heads, num_key_value_heads, head_dim, rms_norm_eps);
}

/* qwen3::qwen3_forward_with_cache (qwen3_ops.h:319-332). */
inline Tensor qwen3_forward_cuda_with_cache(const TensorL& input_ids, KVCache* kv_cache, const Tensor& token_embedding,
                                            const std::vector<Qwen3LayerWeights>& layers, const Tensor& norm_weight,
                                            const Tensor& lm_head, size_t num_layers, size_t num_attention_heads,
                                            size_t num_key_value_heads, size_t head_dim, float rms_norm_eps,
                                            AttentionType attention_type = AttentionType::STANDARD) {
    (void)attention_type;
    auto lk = sa_detail::lock_all();
    if (!kv_cache)
        return sa_detail::forward_nocache(input_ids, token_embedding, layers, norm_weight, lm_head, num_layers,
                                          num_attention_heads, num_key_value_heads, head_dim, rms_norm_eps);
    if (input_ids.shape().ndim() != 2 || input_ids.shape()[0] != 1)
        throw std::invalid_argument("qwen3_forward_cuda_with_cache: input_ids must be [1, S]");
    if (kv_cache->num_layers != num_layers || kv_cache->num_kv_heads != num_key_value_heads ||
        kv_cache->head_dim != head_dim || kv_cache->batch_size != 1)
        throw std::invalid_argument("qwen3_forward_cuda_with_cache: KVCache shape does not match the model");
    const size_t S = input_ids.shape()[1];
    const size_t len = kv_cache->current_seq_len;
    if (len + S > kv_cache->max_seq_len) throw std::runtime_error("KV cache full, cannot append more tokens");
    sa_detail::Model& md = sa_detail::model_for(token_embedding, layers, norm_weight, lm_head, num_layers,
                                                num_attention_heads, num_key_value_heads, head_dim, rms_norm_eps,
                                                (int)kv_cache->max_seq_len);
    const size_t dev_len = (size_t)sa_qwen3_cache_len(md.m);
    if (len == 0) {
        sa_detail::throw_rc(sa_qwen3_reset(md.m), "sa_qwen3_reset");
    } else if (md.bound == kv_cache && len < dev_len) {
        // the caller rewound current_seq_len: the device's first len rows hold it
        sa_detail::throw_rc(sa_qwen3_set_cache_len(md.m, (int)len), "sa_qwen3_set_cache_len");
    } else if (md.bound != kv_cache || dev_len != len) {
        if (!sa_detail::host_rows_written(*kv_cache, len))
            throw std::runtime_error(
                "qwen3_forward_cuda_with_cache: the KVCache's rows live only on a GPU cache that was dropped "
                "(another cache or a long cache-free forward took it); call sync_kv_to_host() before switching, "
                "or reset() the cache");
        // adopt the host cache: rows 0..len-1 of every layer
        for (size_t l = 0; l < num_layers; ++l)
            sa_detail::throw_rc(sa_qwen3_write_kv(md.m, (int)l, kv_cache->key_cache[l].data(),
                                                  kv_cache->value_cache[l].data(), (int)len,
                                                  (int)kv_cache->max_seq_len),
                                "sa_qwen3_write_kv");
        sa_detail::throw_rc(sa_qwen3_set_cache_len(md.m, (int)len), "sa_qwen3_set_cache_len");
    }
    md.bound = kv_cache;
    const size_t V = (size_t)md.cfg.vocab;
    Tensor logits(Shape{1, S, V});
    const std::vector<int64_t> ids = sa_detail::row_ids(input_ids, 0, S);
    sa_detail::throw_rc(sa_qwen3_forward(md.m, ids.data(), (int)S, 1, logits.data(), 0, SA_HOST_PTRS),
                        "qwen3_forward_cuda_with_cache");
    kv_cache->increment_seq_len(S);
    return logits;
}

/* Write the device cache bound to kv_cache into its host tensors (rows
 * 0..current_seq_len-1 of every layer, KVCache layout). */
inline void sync_kv_to_host(KVCache* kv_cache) {
    auto lk = sa_detail::lock_all();
    sa_detail::Registry& r = sa_detail::registry();
    for (auto& kv : r.models) {
        sa_detail::Model& md = *kv.second;
        if (md.bound != kv_cache) continue;
        for (size_t l = 0; l < kv_cache->num_layers; ++l)
            sa_detail::throw_rc(sa_qwen3_read_kv(md.m, (int)l, kv_cache->key_cache[l].data(),
                                                 kv_cache->value_cache[l].data(), (int)kv_cache->max_seq_len),
                                "sa_qwen3_read_kv");
        return;
    }
    throw std::invalid_argument("sync_kv_to_host: no device cache is bound to this KVCache");
}

}  // namespace cuda
}  // namespace qwen3
}  // namespace tensor_cpp

#endif /* SA_QWEN3_TENSORCPP_HPP */
