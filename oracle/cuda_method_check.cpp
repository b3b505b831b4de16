// cuda_method_check.cpp -- test infrastructure: runs the reference's own C++
// API (compiled from its sources into _ref/libsa_ref.so) and the CUDA method
// of this repository through its C++ host layer side by side, on the same
// inputs, with the reference's types:
//   A. attention.h: streaming_attention_serial / naive_attention_serial
//      (attention/src/attention.h:27-35,123-129) vs streaming_attention_cuda /
//      naive_attention_cuda / streaming_attention_cuda_multi
//      (include/sa_attention_cuda.h), U(-1,1) inputs from std::mt19937(42);
//   B. Qwen3: qwen3::qwen3_forward and qwen3::qwen3_forward_with_cache
//      (tensor_cpp/include/tensor_cpp/qwen3_ops.h:250-332) vs
//      qwen3::cuda::qwen3_forward_cuda[_with_cache]
//      (include/sa_qwen3_tensorcpp.hpp) on random-init bf16-exact weights:
//      all-position logits, a cached prefill + greedy decode, a CPU prefill
//      continued on the GPU (host KVCache adoption), sync_kv_to_host, two
//      caches taking turns on the device cache, the qkv_projs and the split
//      q/k/v_proj weight layouts, and the error behaviour (out-of-vocabulary
//      id, full cache, a displaced GPU-only cache);
//   C. tensor_cpp attention operators: ops::self_attention (no mask, the
//      causal mask, an offset causal mask), self_attention_streaming_blockwise
//      (Sq = Skv and Sq < Skv) and the decode attention (tensor_cpp/include/
//      tensor_cpp/ops.h:133-279) vs ops::cuda::* (include/sa_ops_tensorcpp.hpp),
//      and the head-wise / sequence strategies ops::mpi::cuda::* against the
//      reference's unsplit ops::self_attention after repeat_kv (its MPI
//      versions need an MPI install), at head_dim 128 and 64.
// Bars: attention 1e-4 max-abs (fp32 path); Qwen3 logits 2e-3 of max |logit|
// and identical greedy tokens.  Prints "CUDA METHOD CHECK OK" and exits 0 on
// success.  Built by oracle/Makefile (target `check`) where the reference
// tree exists; run by tests/test_cpp_host_gpu.py on a GPU box.
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <limits>
#include <random>
#include <stdexcept>
#include <string>
#include <vector>

#include "attention.h"
#include "tensor_cpp/ops.h"
#include "tensor_cpp/qwen3_ops.h"

#include "sa_attention_cuda.h"
#include "sa_ops_tensorcpp.hpp"
#include "sa_qwen3_tensorcpp.hpp"

using namespace tensor_cpp;

namespace {

int g_fail = 0;

void expect(bool ok, const std::string& what) {
    std::printf("%s %s\n", ok ? "ok  " : "FAIL", what.c_str());
    if (!ok) ++g_fail;
}

double max_abs_diff(const float* a, const float* b, size_t n, double* scale) {
    double e = 0.0, s = 0.0;
    for (size_t i = 0; i < n; ++i) {
        e = std::max(e, std::fabs((double)a[i] - b[i]));
        s = std::max(s, std::fabs((double)b[i]));
    }
    if (scale) *scale = s;
    return e;
}

float bf16_round(float x) {
    uint32_t u;
    std::memcpy(&u, &x, 4);
    u += 0x7FFFu + ((u >> 16) & 1u);
    u &= 0xFFFF0000u;
    std::memcpy(&x, &u, 4);
    return x;
}

Tensor randn_bf16(const Shape& s, std::mt19937& g, float mean, float stdv) {
    std::normal_distribution<float> nd(mean, stdv);
    Tensor t(s);
    for (size_t i = 0; i < t.size(); ++i) t.data()[i] = bf16_round(nd(g));
    return t;
}

// ---------------------------------------------------------------- A
void check_attention() {
    std::mt19937 gen(42);
    std::uniform_real_distribution<float> u(-1.0f, 1.0f);
    const int d = 128;
    for (int T : {1, 63, 64, 1000, 8192}) {
        std::vector<float> Q(d), K((size_t)T * d), V((size_t)T * d);
        for (auto& x : Q) x = u(gen);
        for (auto& x : K) x = u(gen);
        for (auto& x : V) x = u(gen);
        const std::vector<float> ref = streaming_attention_serial(Q.data(), K.data(), V.data(), T, d, 64);
        const std::vector<float> refn = naive_attention_serial(Q.data(), K.data(), V.data(), T, d);
        const std::vector<float> got = streaming_attention_cuda(Q.data(), K.data(), V.data(), T, d, 64);
        const std::vector<float> gotn = naive_attention_cuda(Q.data(), K.data(), V.data(), T, d);
        expect(max_abs_diff(got.data(), ref.data(), d, nullptr) <= 1e-4,
               "streaming_attention_cuda vs streaming_attention_serial, T=" + std::to_string(T));
        expect(max_abs_diff(gotn.data(), refn.data(), d, nullptr) <= 1e-4,
               "naive_attention_cuda vs naive_attention_serial, T=" + std::to_string(T));
        const int n = attention_cuda_device_count();
        for (int g = 2; g <= n && g <= 4; g *= 2) {
            const std::vector<float> gm = streaming_attention_cuda_multi(Q.data(), K.data(), V.data(), T, d, 64, g);
            expect(max_abs_diff(gm.data(), ref.data(), d, nullptr) <= 1e-4,
                   "streaming_attention_cuda_multi (" + std::to_string(g) + " GPUs), T=" + std::to_string(T));
        }
    }
    bool threw = false;
    try {
        std::vector<float> z(96);
        streaming_attention_cuda(z.data(), z.data(), z.data(), 1, 96, 64);
    } catch (const std::invalid_argument&) {
        threw = true;
    }
    expect(threw, "d = 96 raises std::invalid_argument");
}

// ---------------------------------------------------------------- B
struct Model {
    size_t V = 1000, H = 512, L = 2, hq = 8, hkv = 4, D = 128, I = 1024;
    float eps = 1e-6f;
    Tensor embed, norm, lm_head;
    std::vector<qwen3::Qwen3LayerWeights> layers;
};

Model make_model(unsigned seed, bool split_qkv) {
    Model m;
    std::mt19937 g(seed);
    m.embed = randn_bf16(Shape{m.V, m.H}, g, 0.f, 0.02f);
    m.norm = randn_bf16(Shape{m.H}, g, 1.f, 0.1f);
    m.lm_head = m.embed;   // tied, as Qwen3-0.6B
    const size_t QD = m.hq * m.D, KD = m.hkv * m.D;
    for (size_t l = 0; l < m.L; ++l) {
        qwen3::Qwen3LayerWeights w;
        w.qkv_projs = randn_bf16(Shape{QD + 2 * KD, m.H}, g, 0.f, 0.02f);
        if (split_qkv) {
            const float* p = w.qkv_projs.data();
            w.q_proj = Tensor(std::vector<float>(p, p + QD * m.H), Shape{QD, m.H});
            w.k_proj = Tensor(std::vector<float>(p + QD * m.H, p + (QD + KD) * m.H), Shape{KD, m.H});
            w.v_proj = Tensor(std::vector<float>(p + (QD + KD) * m.H, p + (QD + 2 * KD) * m.H), Shape{KD, m.H});
        }
        w.o_proj = randn_bf16(Shape{m.H, QD}, g, 0.f, 0.02f);
        w.q_norm_weight = randn_bf16(Shape{m.D}, g, 1.f, 0.1f);
        w.k_norm_weight = randn_bf16(Shape{m.D}, g, 1.f, 0.1f);
        w.input_layernorm_weight = randn_bf16(Shape{m.H}, g, 1.f, 0.1f);
        w.post_attention_layernorm_weight = randn_bf16(Shape{m.H}, g, 1.f, 0.1f);
        w.gate_proj = randn_bf16(Shape{m.I, m.H}, g, 0.f, 0.02f);
        w.up_proj = randn_bf16(Shape{m.I, m.H}, g, 0.f, 0.02f);
        w.down_proj = randn_bf16(Shape{m.H, m.I}, g, 0.f, 0.02f);
        m.layers.push_back(std::move(w));
    }
    return m;
}

TensorL ids_of(const std::vector<long>& v) { return TensorL(v, Shape{1, v.size()}); }

long argmax_last(const Tensor& logits) {
    const size_t S = logits.shape()[1], V = logits.shape()[2];
    const float* row = logits.data() + (S - 1) * V;
    size_t best = 0;
    for (size_t i = 1; i < V; ++i)
        if (row[i] > row[best]) best = i;
    return (long)best;
}

bool close_logits(const Tensor& got, const Tensor& ref, const std::string& what) {
    double scale = 0.0;
    const double err = max_abs_diff(got.data(), ref.data(), ref.size(), &scale);
    const bool ok = got.shape() == ref.shape() && err <= 2e-3 * std::max(scale, 1e-3);
    if (!ok) std::printf("     %s: max|err| %.3e vs max|ref| %.3e\n", what.c_str(), err, scale);
    return ok;
}

void check_qwen3(bool split_qkv) {
    const std::string tag = split_qkv ? " [q/k/v_proj]" : " [qkv_projs]";
    Model m = make_model(split_qkv ? 11 : 7, split_qkv);
    std::mt19937 g(42);
    std::uniform_int_distribution<long> tok(0, (long)m.V - 1);
    std::vector<long> prompt(37);
    for (auto& t : prompt) t = tok(g);
    auto cpu = [&](const TensorL& ids, qwen3::KVCache* kv) {
        return kv ? qwen3::qwen3_forward_with_cache(ids, kv, m.embed, m.layers, m.norm, m.lm_head, m.L, m.hq, m.hkv,
                                                    m.D, m.eps)
                  : qwen3::qwen3_forward(ids, m.embed, m.layers, m.norm, m.lm_head, m.L, m.hq, m.hkv, m.D, m.eps);
    };
    auto gpu = [&](const TensorL& ids, qwen3::KVCache* kv) {
        return kv ? qwen3::cuda::qwen3_forward_cuda_with_cache(ids, kv, m.embed, m.layers, m.norm, m.lm_head, m.L,
                                                               m.hq, m.hkv, m.D, m.eps)
                  : qwen3::cuda::qwen3_forward_cuda(ids, m.embed, m.layers, m.norm, m.lm_head, m.L, m.hq, m.hkv,
                                                    m.D, m.eps);
    };
    // all-position logits, no cache
    expect(close_logits(gpu(ids_of(prompt), nullptr), cpu(ids_of(prompt), nullptr), "forward"),
           "qwen3_forward_cuda vs qwen3_forward (37 tokens)" + tag);

    // cached prefill + greedy decode on both sides
    const int steps = 6, max_seq = 64;
    qwen3::KVCache kc(m.L, 1, m.hkv, m.D, max_seq), kg(m.L, 1, m.hkv, m.D, max_seq);
    Tensor rc = cpu(ids_of(prompt), &kc), rg = gpu(ids_of(prompt), &kg);
    bool ok = close_logits(rg, rc, "cached prefill") && kg.current_seq_len == prompt.size();
    std::vector<long> tc, tg;
    for (int s = 0; s < steps && ok; ++s) {
        tc.push_back(argmax_last(rc));
        tg.push_back(argmax_last(rg));
        rc = cpu(ids_of({tc.back()}), &kc);
        rg = gpu(ids_of({tg.back()}), &kg);
        ok = close_logits(rg, rc, "decode step " + std::to_string(s));
    }
    expect(ok && tc == tg && kg.current_seq_len == kc.current_seq_len,
           "forward_with_cache: prefill + " + std::to_string(steps) + " greedy steps, same tokens" + tag);

    // the device cache written back into the host KVCache equals the CPU cache
    qwen3::cuda::sync_kv_to_host(&kg);
    double worst = 0.0, scale = 0.0;
    for (size_t l = 0; l < m.L; ++l) {
        double s1 = 0.0, s2 = 0.0;
        worst = std::max(worst, max_abs_diff(kg.key_cache[l].data(), kc.key_cache[l].data(), kc.key_cache[l].size(), &s1));
        worst = std::max(worst, max_abs_diff(kg.value_cache[l].data(), kc.value_cache[l].data(),
                                             kc.value_cache[l].size(), &s2));
        scale = std::max(scale, std::max(s1, s2));
    }
    expect(worst <= 2e-3 * scale, "sync_kv_to_host: host K/V equal the reference's cache" + tag);

    // a cache filled by the CPU method, continued by the CUDA method
    qwen3::KVCache kx(m.L, 1, m.hkv, m.D, max_seq);
    cpu(ids_of(prompt), &kx);
    qwen3::KVCache ky = kx;   // same host rows and length
    const Tensor a = cpu(ids_of({5}), &kx), b = gpu(ids_of({5}), &ky);
    expect(close_logits(b, a, "adopted cache") && ky.current_seq_len == prompt.size() + 1,
           "CPU-filled KVCache continued on the GPU" + tag);

    // two caches taking turns on the one device cache: a cache that was
    // written back (sync_kv_to_host) resumes from its host rows; one whose
    // rows lived only on the GPU raises instead of resuming from zeros
    {
        qwen3::KVCache ka(m.L, 1, m.hkv, m.D, max_seq), kb(m.L, 1, m.hkv, m.D, max_seq), kr(m.L, 1, m.hkv, m.D, max_seq);
        gpu(ids_of(prompt), &ka);
        cpu(ids_of(prompt), &kr);
        qwen3::cuda::sync_kv_to_host(&ka);
        gpu(ids_of({3, 4}), &kb);                       // kb takes the device cache
        const Tensor ra = cpu(ids_of({9}), &kr), ga = gpu(ids_of({9}), &ka);
        expect(close_logits(ga, ra, "resumed cache"), "synced cache resumes after another cache used the GPU" + tag);
        bool stale = false;
        try {
            gpu(ids_of({1}), &kb);                      // kb was never written back
        } catch (const std::runtime_error&) {
            stale = true;
        }
        expect(stale, "GPU-only cache displaced by another raises std::runtime_error" + tag);
        kb.reset();
        expect(gpu(ids_of({1}), &kb).shape()[1] == 1 && kb.current_seq_len == 1, "reset() cache starts over" + tag);
    }

    // errors keep the reference's exception types
    bool oor = false, full = false;
    try {
        gpu(ids_of({(long)m.V}), nullptr);
    } catch (const std::out_of_range&) {
        oor = true;
    }
    try {
        qwen3::KVCache ks(m.L, 1, m.hkv, m.D, 8);
        gpu(ids_of(std::vector<long>(9, 1)), &ks);
    } catch (const std::runtime_error&) {
        full = true;
    }
    expect(oor, "token id == vocab raises std::out_of_range" + tag);
    expect(full, "prompt longer than the cache raises std::runtime_error" + tag);
}

// ---------------------------------------------------------------- C
Tensor uniform(const Shape& s, std::mt19937& g) {
    std::uniform_real_distribution<float> u(-1.0f, 1.0f);
    Tensor t(s);
    for (size_t i = 0; i < t.size(); ++i) t.data()[i] = u(g);
    return t;
}

bool close_attn(const Tensor& got, const Tensor& ref, const std::string& what) {
    const double err = max_abs_diff(got.data(), ref.data(), ref.size(), nullptr);
    const bool ok = got.shape() == ref.shape() && err <= 1e-4;
    if (!ok) std::printf("     %s: max|err| %.3e\n", what.c_str(), err);
    return ok;
}

// mask [Sq, Sk]: 0 where key j <= query i + off, -inf after
Tensor offset_causal_mask(size_t Sq, size_t Sk, size_t off) {
    Tensor m(Shape{Sq, Sk});
    for (size_t i = 0; i < Sq; ++i)
        for (size_t j = 0; j < Sk; ++j)
            m.data()[i * Sk + j] = j <= i + off ? 0.0f : -std::numeric_limits<float>::infinity();
    return m;
}

void check_ops(size_t D) {
    const std::string tag = " [d=" + std::to_string(D) + "]";
    std::mt19937 g(42 + D);
    const float scale = 1.0f / std::sqrt((float)D);
    const size_t B = 2, H = 8, S = 150;
    const Tensor q = uniform(Shape{B, H, S, D}, g), k = uniform(Shape{B, H, S, D}, g), v = uniform(Shape{B, H, S, D}, g);
    const Tensor causal = qwen3::create_causal_mask(S).view(Shape{1, 1, S, S});
    expect(close_attn(ops::cuda::self_attention(q, k, v, &causal, scale), ops::self_attention(q, k, v, &causal, scale),
                      "causal"),
           "ops::cuda::self_attention, causal mask (create_causal_mask)" + tag);
    expect(close_attn(ops::cuda::self_attention(q, k, v, nullptr, scale), ops::self_attention(q, k, v, nullptr, scale),
                      "no mask"),
           "ops::cuda::self_attention, no mask" + tag);
    expect(close_attn(ops::cuda::self_attention_streaming_blockwise(q, k, v, scale, 32, 64),
                      ops::self_attention_streaming_blockwise(q, k, v, scale, 32, 64), "blockwise"),
           "ops::cuda::self_attention_streaming_blockwise, Sq = Skv" + tag);
    {   // a query block after a cached prefix: offset causal mask, and the
        // block-wise form (queries see keys 0..i)
        const size_t Sq = 40, Sk = 170;
        const Tensor qq = uniform(Shape{1, H, Sq, D}, g), kk = uniform(Shape{1, H, Sk, D}, g),
                     vv = uniform(Shape{1, H, Sk, D}, g);
        const Tensor m = offset_causal_mask(Sq, Sk, Sk - Sq);
        expect(close_attn(ops::cuda::self_attention(qq, kk, vv, &m, scale), ops::self_attention(qq, kk, vv, &m, scale),
                          "offset causal"),
               "ops::cuda::self_attention, causal mask of a query block at offset Sk - Sq" + tag);
        expect(close_attn(ops::cuda::self_attention_streaming_blockwise(qq, kk, vv, scale, 32, 64),
                          ops::self_attention_streaming_blockwise(qq, kk, vv, scale, 32, 64), "blockwise Sq<Skv"),
               "ops::cuda::self_attention_streaming_blockwise, Sq < Skv" + tag);
        Tensor bad = offset_causal_mask(Sq, Sk, 3);
        bad.data()[5] = 0.5f;
        bool rejected = false;
        try {
            ops::cuda::self_attention(qq, kk, vv, &bad, scale);
        } catch (const std::invalid_argument&) {
            rejected = true;
        }
        expect(rejected, "a mask that is not causal raises std::invalid_argument" + tag);
    }
    {   // decode: one query over a long cache (the attention the Qwen3 decode needs)
        const size_t T = 3001;
        const Tensor qd = uniform(Shape{1, 16, 1, D}, g), kd = uniform(Shape{1, 16, T, D}, g),
                     vd = uniform(Shape{1, 16, T, D}, g);
        expect(close_attn(ops::cuda::self_attention_streaming(qd, kd, vd, scale, 64),
                          ops::self_attention(qd, kd, vd, nullptr, scale), "decode"),
               "ops::cuda::self_attention_streaming (decode, scale on the scores) = ops::self_attention" + tag);
    }
    {   // GQA strategies: 16 query heads, 8 KV heads, ground truth after repeat_kv
        const size_t hq = 16, hkv = 8, Sg = 203;
        const Tensor qg = uniform(Shape{1, hq, Sg, D}, g), kg = uniform(Shape{1, hkv, Sg, D}, g),
                     vg = uniform(Shape{1, hkv, Sg, D}, g);
        const Tensor kr = qwen3::repeat_kv(kg, (int)(hq / hkv)), vr = qwen3::repeat_kv(vg, (int)(hq / hkv));
        const Tensor cm = qwen3::create_causal_mask(Sg).view(Shape{1, 1, Sg, Sg});
        const Tensor ref_c = ops::self_attention(qg, kr, vr, &cm, scale);
        const Tensor ref_n = ops::self_attention(qg, kr, vr, nullptr, scale);
        expect(close_attn(ops::mpi::cuda::attention_headwise_standard(qg, kg, vg, &cm, scale, hq, hkv), ref_c, "hw std"),
               "ops::mpi::cuda::attention_headwise_standard (causal mask, heads over the GPUs)" + tag);
        expect(close_attn(ops::mpi::cuda::attention_headwise_standard(qg, kg, vg, nullptr, scale, hq, hkv), ref_n,
                          "hw std nomask"),
               "ops::mpi::cuda::attention_headwise_standard (no mask)" + tag);
        expect(close_attn(ops::mpi::cuda::attention_headwise_online_softmax(qg, kg, vg, nullptr, scale, hq, hkv), ref_c,
                          "hw online"),
               "ops::mpi::cuda::attention_headwise_online_softmax (causal)" + tag);
        expect(close_attn(ops::mpi::cuda::attention_sequence_online_softmax(qg, kg, vg, nullptr, scale, hq, hkv, Sg),
                          ref_c, "sequence"),
               "ops::mpi::cuda::attention_sequence_online_softmax (zig-zag chunks over the GPUs)" + tag);
        expect(close_attn(ops::mpi::cuda::attention_sequence_online_softmax(qg, kg, vg, nullptr, scale, hq, hkv, Sg, 1),
                          ref_c, "sequence 1 gpu"),
               "ops::mpi::cuda::attention_sequence_online_softmax on one GPU" + tag);
    }
}

}  // namespace

int main() {
    std::setvbuf(stdout, nullptr, _IONBF, 0);   // every line out before a possible abort
    try {
        check_attention();
        check_ops(128);
        check_ops(64);
        check_qwen3(false);
        check_qwen3(true);
    } catch (const std::exception& e) {
        std::printf("FAIL unexpected exception: %s\n", e.what());
        ++g_fail;
    }
    qwen3::cuda::release();
    ops::cuda::release();
    attention_cuda_release();
    if (g_fail) {
        std::printf("CUDA METHOD CHECK FAILED (%d)\n", g_fail);
        return 1;
    }
    std::printf("CUDA METHOD CHECK OK\n");
    return 0;
}
