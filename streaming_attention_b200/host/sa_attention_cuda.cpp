// sa_attention_cuda.cpp -- the CUDA method for the attention.h functions
// (include/sa_attention_cuda.h), on top of the C ABI of libsa_cuda.so.
//
// Host buffers go through the C ABI with SA_HOST_PTRS: the library stages
// them in device memory, runs the split-KV decode kernel and copies the d
// outputs back before returning, so each call is synchronous like the
// reference's CPU functions.
#include "sa_attention_cuda.h"

#include <atomic>
#include <memory>
#include <mutex>
#include <stdexcept>
#include <string>
#include <thread>
#include <vector>

#include "sa_cuda.h"

namespace {

[[noreturn]] void fail(int rc, const char* what) {
    const std::string msg = std::string(what) + ": " + sa_last_error();
    if (rc == SA_ERR_ARG) throw std::invalid_argument(msg);
    throw std::runtime_error(msg);
}

inline void check(int rc, const char* what) {
    if (rc != SA_OK) fail(rc, what);
}

// One context per GPU, created on first use; a call holds its GPU's mutex.
struct Device {
    std::mutex mu;
    sa_ctx* ctx = nullptr;
};

struct Registry {
    std::mutex mu;
    std::vector<std::unique_ptr<Device>> devs;
    std::atomic<int> current{0};

    ~Registry() { release(); }

    void release() {
        std::lock_guard<std::mutex> lk(mu);
        for (auto& d : devs) {
            std::lock_guard<std::mutex> dl(d->mu);
            if (d->ctx) sa_ctx_destroy(d->ctx);
            d->ctx = nullptr;
        }
    }

    // The device's slot (its context is created by the first Lease).
    Device& slot(int device) {
        std::lock_guard<std::mutex> lk(mu);
        if (device < 0) throw std::invalid_argument("attention_cuda: negative device");
        while ((int)devs.size() <= device) devs.emplace_back(new Device);
        return *devs[device];
    }
};

Registry& registry() {
    static Registry r;
    return r;
}

// Locked context of one GPU for the duration of a call.
struct Lease {
    Device& dev;
    std::unique_lock<std::mutex> lk;
    sa_ctx* ctx = nullptr;
    explicit Lease(int device) : dev(registry().slot(device)), lk(dev.mu) {
        if (!dev.ctx) check(sa_ctx_create(device, &dev.ctx), "sa_ctx_create");
        ctx = dev.ctx;
    }
};

void check_sizes(int T, int d, int block_size, const char* fn) {
    if (T < 0) throw std::invalid_argument(std::string(fn) + ": T < 0");
    if (d != 64 && d != 128 && d != 256)
        throw std::invalid_argument(std::string(fn) + ": d = " + std::to_string(d) +
                                    " (the GPU path supports 64, 128, 256)");
    if (block_size <= 0) throw std::invalid_argument(std::string(fn) + ": block_size <= 0");
}

// One query row against T keys on `device`: softmax(q K^T) V, scale 1.
std::vector<float> decode_one(int device, const float* Q, const float* K, const float* V, int T, int d, int block,
                              const char* fn) {
    check_sizes(T, d, block, fn);
    std::vector<float> out((size_t)d, 0.f);
    if (T == 0) return out;
    Lease lease(device);
    check(sa_attn_decode(lease.ctx, SA_F32, Q, K, V, (long long)T * d, T, d, 1, 1, block, 1.0f, out.data(),
                         SA_HOST_PTRS),
          fn);
    return out;
}

}  // namespace

std::vector<float> naive_attention_cuda(const float* Q, const float* K, const float* V, int T, int d) {
    return decode_one(registry().current, Q, K, V, T, d, 64, "naive_attention_cuda");
}

std::vector<float> streaming_attention_cuda(const float* Q, const float* K, const float* V, int T, int d,
                                            int block_size) {
    return decode_one(registry().current, Q, K, V, T, d, block_size, "streaming_attention_cuda");
}

std::vector<float> streaming_attention_cuda_multi(const float* Q, const float* K, const float* V, int T, int d,
                                                  int block_size, int num_gpus) {
    const char* fn = "streaming_attention_cuda_multi";
    check_sizes(T, d, block_size, fn);
    const int avail = attention_cuda_device_count();
    if (num_gpus < 1 || num_gpus > avail)
        throw std::invalid_argument(std::string(fn) + ": num_gpus = " + std::to_string(num_gpus) + " of " +
                                    std::to_string(avail) + " visible");
    // contiguous slices, the first T % n slices one row longer (the rank
    // partition of the reference's MPI drivers)
    std::vector<float> m(num_gpus), l(num_gpus), o((size_t)num_gpus * d);
    std::vector<std::string> errors(num_gpus);
    std::vector<int> codes(num_gpus, SA_OK);
    auto work = [&](int i) {
        const int base = T / num_gpus, rem = T % num_gpus;
        const int t0 = i * base + (i < rem ? i : rem);
        const int n = base + (i < rem ? 1 : 0);
        try {
            Lease lease(i);
            const int rc = sa_attn_decode_partial(lease.ctx, SA_F32, Q, K + (size_t)t0 * d, V + (size_t)t0 * d,
                                                  (long long)n * d, n, d, 1, 1, block_size, 1.0f, &m[i], &l[i],
                                                  &o[(size_t)i * d], SA_HOST_PTRS);
            if (rc != SA_OK) {
                codes[i] = rc;
                errors[i] = sa_last_error();
            }
        } catch (const std::exception& e) {
            codes[i] = SA_ERR_CUDA;
            errors[i] = e.what();
        }
    };
    std::vector<std::thread> threads;
    for (int i = 1; i < num_gpus; ++i) threads.emplace_back(work, i);
    work(0);
    for (auto& t : threads) t.join();
    for (int i = 0; i < num_gpus; ++i)
        if (codes[i] != SA_OK) {
            const std::string msg = std::string(fn) + ": GPU " + std::to_string(i) + ": " + errors[i];
            if (codes[i] == SA_ERR_ARG) throw std::invalid_argument(msg);
            throw std::runtime_error(msg);
        }
    std::vector<float> out((size_t)d, 0.f);
    Lease lease(0);
    check(sa_attn_merge(lease.ctx, num_gpus, 1, d, m.data(), l.data(), o.data(), out.data(), nullptr, nullptr,
                        SA_HOST_PTRS),
          fn);
    return out;
}

void attention_cuda_set_device(int device) {
    if (device < 0 || device >= attention_cuda_device_count())
        throw std::invalid_argument("attention_cuda_set_device: no GPU " + std::to_string(device));
    registry().current = device;
}

int attention_cuda_device_count() {
    int n = 0;
    return sa_device_count(&n) == SA_OK ? n : 0;
}

void attention_cuda_release() { registry().release(); }
