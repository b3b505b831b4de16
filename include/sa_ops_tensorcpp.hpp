/*
 * sa_ops_tensorcpp.hpp -- the CUDA method for the reference's attention
 * operators, with their arguments and Tensor types:
 *
 *   tensor_cpp::ops::cuda::self_attention                    ops.h:133-139   (ops.cpp:514-641)
 *   tensor_cpp::ops::cuda::self_attention_streaming          ops.h:250-256   (ops.cpp:964-1017)
 *   tensor_cpp::ops::cuda::self_attention_streaming_blockwise ops.h:272-279  (ops.cpp:1383-1450)
 *   tensor_cpp::ops::mpi::cuda::attention_headwise_standard        ops_mpi.h:238  (ops_mpi.cpp:966-977)
 *   tensor_cpp::ops::mpi::cuda::attention_headwise_online_softmax  ops_mpi.h:272  (ops_mpi.cpp:979-994)
 *   tensor_cpp::ops::mpi::cuda::attention_sequence_online_softmax  ops_mpi.h:326  (ops_mpi.cpp:1000-1212)
 *
 * Header-only, for a build of the reference: include it after
 * "tensor_cpp/ops.h" (it uses that header's Tensor and Shape) and link
 * libsa_cuda.so.  Every operator takes host fp32 tensors and returns a host
 * Tensor; the attention runs in fp32 on the GPU (sa_attn_prompt_f32 of
 * sa_cuda.h: the prompt-attention and decode kernels), so results agree with
 * the reference's to fp32 rounding.
 *
 * Semantics kept from the reference:
 *  - self_attention(q, k, v, mask, scale): q [B, H, Sq, D], k/v [B, H, Sk, D]
 *    (already repeated to H heads), scores scaled and mask[i * Sk + j] added.
 *    The masks the reference builds are supported: none, all zeros, and the
 *    causal 0 / -inf mask of create_causal_mask (qwen3_ops.cpp:240-259),
 *    also offset (query i sees keys j <= i + Sk - Sq); any other mask raises
 *    std::invalid_argument.
 *  - self_attention_streaming: every query sees all keys, with the scale on
 *    the scores.  (The reference multiplies the OUTPUT by the scale,
 *    ops.cpp:1010, which is not attention; the GPU computes the attention the
 *    operator documents, which is also what the Qwen3 decode needs.)
 *  - self_attention_streaming_blockwise: causal, query i sees keys 0..i
 *    (queries past the last key see all keys), block sizes only change
 *    rounding.
 *  - the ops::mpi operators take the reference's arguments without the
 *    communicator and run inside ONE process over `num_gpus` GPUs (0 = all
 *    visible), one host thread per GPU:
 *      head-wise: the KV-head groups are split over the GPUs (each GPU takes
 *        whole groups, so no repeat_kv copy), outputs gathered in host memory
 *        (the Allgatherv); "standard" applies the mask as self_attention,
 *        "online_softmax" is causal as self_attention_mpi_streaming_omp
 *        (ops_mpi.cpp:452-597, which ignores the mask);
 *      sequence: q, k, v are the FULL [B, H, S, D] tensors (the ranks' local
 *        blocks concatenated in rank order); the sequence is cut into 2P
 *        zig-zag chunks, GPU r computing the causal attention of chunks r and
 *        2P-1-r over the keys before them -- the correct result of the
 *        sequence strategy whose reference implementation is wrong (its
 *        statistics all-reduce mixes positions).  global_seq_len must equal S.
 *  - errors are exceptions: std::invalid_argument for shapes / masks the CUDA
 *    path does not take, std::runtime_error for CUDA failures.
 * Threading: one sa_ctx per GPU, created on first use and kept until
 * ops::cuda::release() (or the end of the process); calls are serialised per
 * GPU.
 */
#ifndef SA_OPS_TENSORCPP_HPP
#define SA_OPS_TENSORCPP_HPP

#include <algorithm>
#include <cmath>
#include <cstddef>
#include <exception>
#include <map>
#include <memory>
#include <mutex>
#include <stdexcept>
#include <string>
#include <thread>
#include <vector>

#include "sa_cuda.h"

namespace tensor_cpp {
namespace ops {
namespace cuda {

namespace sa_ops_detail {

inline void throw_rc(int rc, const char* what) {
    if (rc == SA_OK) return;
    const std::string msg = std::string(what) + ": " + sa_last_error();
    if (rc == SA_ERR_ARG) throw std::invalid_argument(msg);
    throw std::runtime_error(msg);
}

struct Device {
    std::mutex mu;
    sa_ctx* ctx = nullptr;
};

struct Devices {
    std::mutex mu;
    std::map<int, std::unique_ptr<Device>> dev;
};

// Never destroyed: a context left at exit goes with the process, and no CUDA
// call runs from a static destructor while the runtime shuts down.  release()
// frees them earlier.
inline Devices& devices() {
    static Devices* d = new Devices;
    return *d;
}

// The GPU's context (created on first use) with its lock held by the caller.
inline Device& device(int id) {
    Devices& ds = devices();
    std::lock_guard<std::mutex> lk(ds.mu);
    std::unique_ptr<Device>& d = ds.dev[id];
    if (!d) d.reset(new Device);
    return *d;
}

inline int device_count() {
    int n = 0;
    throw_rc(sa_device_count(&n), "sa_device_count");
    if (n < 1) throw std::runtime_error("tensor_cpp::ops::cuda: no CUDA device");
    return n;
}

// Which keys query i sees: all of them (full), or j <= i + offset (causal).
struct Visibility {
    bool causal;
    long long offset;
};

// The reference's masks: none / all zeros (full), or the causal 0 / -inf
// pattern with some offset.  Anything else is outside the CUDA path.
inline Visibility classify_mask(const Tensor* mask, size_t Sq, size_t Sk, const char* fn) {
    if (!mask) return {false, 0};
    if (mask->size() < Sq * Sk)
        throw std::invalid_argument(std::string(fn) + ": mask smaller than [q_seq_len, k_seq_len]");
    const float* m = mask->data();
    std::vector<size_t> lead(Sq);
    for (size_t i = 0; i < Sq; ++i) {
        const float* row = m + i * Sk;
        size_t c = 0;
        while (c < Sk && row[c] == 0.0f) ++c;
        for (size_t j = c; j < Sk; ++j)
            if (!(std::isinf(row[j]) && row[j] < 0))
                throw std::invalid_argument(std::string(fn) +
                                            ": only no mask, an all-zero mask or a causal 0/-inf mask "
                                            "is supported on the CUDA path");
        lead[i] = c;
    }
    bool full = true;
    for (size_t i = 0; i < Sq; ++i) full = full && lead[i] == Sk;
    if (full) return {false, 0};
    if (lead[0] == 0) throw std::invalid_argument(std::string(fn) + ": mask hides every key of query 0");
    const long long off = (long long)lead[0] - 1;
    for (size_t i = 0; i < Sq; ++i)
        if (lead[i] != std::min(Sk, (size_t)(off + (long long)i + 1)))
            throw std::invalid_argument(std::string(fn) + ": mask is not causal (0 for j <= i + offset, -inf after)");
    return {true, off};
}

// Rows [row0, row0 + nrows) of query heads [0, hq) (head-major source
// q [hq][Sq_all][D]) against KV heads [0, hkv) (head-major k, v
// [hkv][Sk_all][D], of which the first Sk rows are used) on GPU `dev`;
// writes the same rows of out [hq][Sq_all][D].  Query row i sits at
// position q_pos0 + (i - row0) for the causal limit.
inline void run_rows(int dev, const float* q, const float* k, const float* v, float* out, size_t hq, size_t hkv,
                     size_t Sq_all, size_t Sk_all, size_t D, size_t row0, size_t nrows, size_t Sk, bool causal,
                     long long q_pos0, float scale) {
    if (nrows == 0) return;
    std::vector<float> qt(nrows * hq * D), ot(nrows * hq * D);
    for (size_t h = 0; h < hq; ++h)
        for (size_t i = 0; i < nrows; ++i)
            std::copy_n(q + (h * Sq_all + row0 + i) * D, D, qt.data() + (i * hq + h) * D);
    Device& d = device(dev);
    {
        std::lock_guard<std::mutex> lk(d.mu);
        if (!d.ctx) throw_rc(sa_ctx_create(dev, &d.ctx), "sa_ctx_create");
        throw_rc(sa_attn_prompt_f32(d.ctx, qt.data(), k, v, (int)nrows, (int)Sk, (int)q_pos0, causal ? 1 : 0,
                                    (int)D, (int)hq, (int)hkv, (long long)(hq * D), (long long)(Sk_all * D), scale,
                                    ot.data(), (long long)(hq * D), SA_HOST_PTRS),
                 "sa_attn_prompt_f32");
    }
    for (size_t h = 0; h < hq; ++h)
        for (size_t i = 0; i < nrows; ++i)
            std::copy_n(ot.data() + (i * hq + h) * D, D, out + (h * Sq_all + row0 + i) * D);
}

inline void check4(const Tensor& t, const char* fn, const char* what) {
    if (t.shape().ndim() != 4)
        throw std::invalid_argument(std::string(fn) + ": " + what + " must be [batch, heads, seq_len, head_dim]");
}

// Every batch row, all heads, on one GPU.
inline Tensor attend(const Tensor& query, const Tensor& key, const Tensor& value, Visibility vis, float scale,
                     const char* fn) {
    check4(query, fn, "query");
    check4(key, fn, "key");
    check4(value, fn, "value");
    const size_t B = query.shape()[0], H = query.shape()[1], Sq = query.shape()[2], D = query.shape()[3];
    const size_t Hk = key.shape()[1], Sk = key.shape()[2];
    if (key.shape()[0] != B || key.shape()[3] != D || value.shape()[0] != B || value.shape()[1] != Hk ||
        value.shape()[2] != Sk || value.shape()[3] != D || Hk == 0 || H % Hk != 0 || Sk == 0)
        throw std::invalid_argument(std::string(fn) + ": query/key/value shapes do not match");
    Tensor out(query.shape());
    for (size_t b = 0; b < B; ++b)
        run_rows(0, query.data() + b * H * Sq * D, key.data() + b * Hk * Sk * D, value.data() + b * Hk * Sk * D,
                 out.data() + b * H * Sq * D, H, Hk, Sq, Sk, D, 0, Sq, Sk, vis.causal, vis.offset, scale);
    return out;
}

}  // namespace sa_ops_detail

/* Destroy the per-GPU contexts (device memory and streams); the next call
 * creates them again.  Not to be called while an operator runs. */
inline void release() {
    sa_ops_detail::Devices& ds = sa_ops_detail::devices();
    std::lock_guard<std::mutex> lk(ds.mu);
    for (auto& kv : ds.dev) {
        std::lock_guard<std::mutex> dl(kv.second->mu);
        if (kv.second->ctx) sa_ctx_destroy(kv.second->ctx);
        kv.second->ctx = nullptr;
    }
}

/* ops::self_attention (ops.h:133-139): softmax(scale q k^T + mask) v. */
inline Tensor self_attention(const Tensor& query, const Tensor& key, const Tensor& value,
                             const Tensor* mask = nullptr, float scale = 1.0f) {
    const char* fn = "ops::cuda::self_attention";
    sa_ops_detail::check4(query, fn, "query");
    sa_ops_detail::check4(key, fn, "key");
    const sa_ops_detail::Visibility vis =
        sa_ops_detail::classify_mask(mask, query.shape()[2], key.shape()[2], fn);
    return sa_ops_detail::attend(query, key, value, vis, scale, fn);
}

/* ops::self_attention_streaming (ops.h:250-256): every query sees every key. */
inline Tensor self_attention_streaming(const Tensor& query, const Tensor& key, const Tensor& value,
                                       float scale = 1.0f, int block_size = 64) {
    (void)block_size;
    return sa_ops_detail::attend(query, key, value, {false, 0}, scale, "ops::cuda::self_attention_streaming");
}

/* ops::self_attention_streaming_blockwise (ops.h:272-279): causal, query i
 * sees keys 0..i. */
inline Tensor self_attention_streaming_blockwise(const Tensor& query, const Tensor& key, const Tensor& value,
                                                 float scale = 1.0f, int q_block_size = 32,
                                                 int kv_block_size = 64) {
    (void)q_block_size;
    (void)kv_block_size;
    return sa_ops_detail::attend(query, key, value, {true, 0}, scale,
                                 "ops::cuda::self_attention_streaming_blockwise");
}

}  // namespace cuda

namespace mpi {
namespace cuda {

namespace sa_mpi_detail {

using tensor_cpp::ops::cuda::sa_ops_detail::Visibility;

inline int gpus_for(int num_gpus, size_t parts) {
    int n = tensor_cpp::ops::cuda::sa_ops_detail::device_count();
    if (num_gpus > 0) n = std::min(n, num_gpus);
    return (int)std::max<size_t>(1, std::min<size_t>((size_t)n, parts));
}

// Run job(g) for g < n on one host thread each; rethrow the first failure.
template <typename F>
inline void on_gpus(int n, F job) {
    std::vector<std::thread> th;
    std::vector<std::exception_ptr> err(n);
    for (int g = 0; g < n; ++g)
        th.emplace_back([&, g] {
            try {
                job(g);
            } catch (...) {
                err[g] = std::current_exception();
            }
        });
    for (auto& t : th) t.join();
    for (auto& e : err)
        if (e) std::rethrow_exception(e);
}

inline Tensor headwise(const Tensor& query, const Tensor& key, const Tensor& value, Visibility vis, float scale,
                       int num_attention_heads, int num_key_value_heads, int num_gpus, const char* fn) {
    namespace d = tensor_cpp::ops::cuda::sa_ops_detail;
    d::check4(query, fn, "query");
    d::check4(key, fn, "key");
    d::check4(value, fn, "value");
    const size_t B = query.shape()[0], H = query.shape()[1], Sq = query.shape()[2], D = query.shape()[3];
    const size_t Hk = key.shape()[1], Sk = key.shape()[2];
    if ((int)H != num_attention_heads || (int)Hk != num_key_value_heads || Hk == 0 || H % Hk != 0 ||
        key.shape()[0] != B || key.shape()[3] != D || value.shape()[1] != Hk || value.shape()[2] != Sk)
        throw std::invalid_argument(std::string(fn) + ": tensor shapes do not match the head counts");
    const size_t G = H / Hk;
    const int P = gpus_for(num_gpus, Hk);
    Tensor out(query.shape());
    on_gpus(P, [&](int g) {
        const size_t k0 = Hk * g / P, k1 = Hk * (g + 1) / P;      // this GPU's KV-head groups
        for (size_t b = 0; b < B; ++b)
            d::run_rows(g, query.data() + (b * H + k0 * G) * Sq * D, key.data() + (b * Hk + k0) * Sk * D,
                        value.data() + (b * Hk + k0) * Sk * D, out.data() + (b * H + k0 * G) * Sq * D,
                        (k1 - k0) * G, k1 - k0, Sq, Sk, D, 0, Sq, Sk, vis.causal, vis.offset, scale);
    });
    return out;
}

}  // namespace sa_mpi_detail

/* ops::mpi::attention_headwise_standard (ops_mpi.h:238): heads split over
 * the GPUs, the mask applied as ops::self_attention. */
inline Tensor attention_headwise_standard(const Tensor& query, const Tensor& key, const Tensor& value,
                                          const Tensor* mask, float scale, int num_attention_heads,
                                          int num_key_value_heads, int num_gpus = 0) {
    const char* fn = "ops::mpi::cuda::attention_headwise_standard";
    tensor_cpp::ops::cuda::sa_ops_detail::check4(query, fn, "query");
    tensor_cpp::ops::cuda::sa_ops_detail::check4(key, fn, "key");
    const auto vis = tensor_cpp::ops::cuda::sa_ops_detail::classify_mask(mask, query.shape()[2], key.shape()[2], fn);
    return sa_mpi_detail::headwise(query, key, value, vis, scale, num_attention_heads, num_key_value_heads,
                                   num_gpus, fn);
}

/* ops::mpi::attention_headwise_online_softmax (ops_mpi.h:272): heads split
 * over the GPUs, causal block-wise attention (the mask is not used, as in
 * self_attention_mpi_streaming_omp). */
inline Tensor attention_headwise_online_softmax(const Tensor& query, const Tensor& key, const Tensor& value,
                                                const Tensor* mask, float scale, int num_attention_heads,
                                                int num_key_value_heads, int num_gpus = 0) {
    (void)mask;
    return sa_mpi_detail::headwise(query, key, value, {true, 0}, scale, num_attention_heads, num_key_value_heads,
                                   num_gpus, "ops::mpi::cuda::attention_headwise_online_softmax");
}

/* ops::mpi::attention_sequence_online_softmax (ops_mpi.h:326), one process:
 * the full tensors, the sequence in 2P zig-zag chunks over P GPUs, causal
 * attention of each chunk over the keys before it. */
inline Tensor attention_sequence_online_softmax(const Tensor& query, const Tensor& key, const Tensor& value,
                                                const Tensor* mask, float scale, int num_attention_heads,
                                                int num_key_value_heads, size_t global_seq_len,
                                                int num_gpus = 0) {
    namespace d = tensor_cpp::ops::cuda::sa_ops_detail;
    (void)mask;
    const char* fn = "ops::mpi::cuda::attention_sequence_online_softmax";
    d::check4(query, fn, "query");
    d::check4(key, fn, "key");
    d::check4(value, fn, "value");
    const size_t B = query.shape()[0], H = query.shape()[1], S = query.shape()[2], D = query.shape()[3];
    const size_t Hk = key.shape()[1];
    if ((int)H != num_attention_heads || (int)Hk != num_key_value_heads || Hk == 0 || H % Hk != 0 ||
        key.shape()[2] != S || value.shape()[2] != S || key.shape()[0] != B || value.shape()[1] != Hk)
        throw std::invalid_argument(std::string(fn) + ": tensor shapes do not match the head counts");
    if (global_seq_len != S)
        throw std::invalid_argument(std::string(fn) + ": pass the full [B, H, global_seq_len, D] tensors");
    const int P = sa_mpi_detail::gpus_for(num_gpus, (S + 1) / 2);
    const size_t n = 2 * (size_t)P;
    Tensor out(query.shape());
    sa_mpi_detail::on_gpus(P, [&](int g) {
        for (size_t c : {(size_t)g, n - 1 - (size_t)g}) {
            const size_t r0 = S * c / n, r1 = S * (c + 1) / n;   // chunk c's rows
            for (size_t b = 0; b < B; ++b)
                d::run_rows(g, query.data() + b * H * S * D, key.data() + b * Hk * S * D,
                            value.data() + b * Hk * S * D, out.data() + b * H * S * D, H, Hk, S, S, D, r0,
                            r1 - r0, r1, true, (long long)r0, scale);
        }
    });
    return out;
}

}  // namespace cuda
}  // namespace mpi
}  // namespace ops
}  // namespace tensor_cpp

#endif /* SA_OPS_TENSORCPP_HPP */
