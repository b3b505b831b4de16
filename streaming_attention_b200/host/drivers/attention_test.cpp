// attention_test.cpp -- command-line drivers for the CUDA method of the
// attention.h functions, with the argument order and the "Time: <ms> ms"
// output line of the reference's test drivers (whose scripts read the
// second token of that line as milliseconds: run_mpi_tests.sh:91-92,
// compare_attention_full.py:210-228).
//
// Built four times (SA_DRIVER_MODE):
//   0 test_naive_cuda            <T> <d> [block]
//   1 test_streaming_cuda        <T> <d> <block>
//   2 test_streaming_cuda_multi  <T> <d> <block> <num_gpus>
//   3 test_mpi_cuda              --T <T> --d <d> --block <b> [--gpus N]
// Common options after the positional ones: --iters N (timed calls, default
// 10), --seed S (default 42).
//
// Inputs: Q, K, V uniform in [-1, 1) from std::mt19937(seed), as the
// reference's attention tests draw them.  The reported time is the mean wall
// time of one call, host buffers in and the d outputs back on the host
// (the reference API's contract).  The driver also prints the max |error|
// against an fp64 three-pass softmax computed here.
#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <random>
#include <stdexcept>
#include <string>
#include <vector>

#include "sa_attention_cuda.h"

#ifndef SA_DRIVER_MODE
#define SA_DRIVER_MODE 1
#endif

namespace {

std::vector<double> softmax_attention_f64(const float* q, const float* k, const float* v, int T, int d) {
    std::vector<double> s(T), out(d, 0.0);
    double mx = -INFINITY;
    for (int t = 0; t < T; ++t) {
        double acc = 0.0;
        for (int i = 0; i < d; ++i) acc += (double)q[i] * k[(size_t)t * d + i];
        s[t] = acc;
        mx = std::max(mx, acc);
    }
    double sum = 0.0;
    for (int t = 0; t < T; ++t) sum += (s[t] = std::exp(s[t] - mx));
    for (int t = 0; t < T; ++t)
        for (int i = 0; i < d; ++i) out[i] += s[t] / sum * v[(size_t)t * d + i];
    return out;
}

int usage(const char* prog) {
    const char* forms[] = {"<T> <d> [block]", "<T> <d> <block>", "<T> <d> <block> <num_gpus>",
                           "--T <T> --d <d> --block <b> [--gpus N]"};
    std::fprintf(stderr, "usage: %s %s [--iters N] [--seed S]\n", prog, forms[SA_DRIVER_MODE]);
    return 2;
}

}  // namespace

int main(int argc, char** argv) {
    int T = 8192, d = 128, block = 64, gpus = 1, iters = 10;
    unsigned seed = 42;
    std::vector<std::string> pos;
    for (int i = 1; i < argc; ++i) {
        const std::string a = argv[i];
        auto next = [&](int& dst) {
            if (i + 1 >= argc) throw std::invalid_argument("missing value after " + a);
            dst = std::atoi(argv[++i]);
        };
        if (a == "--iters") next(iters);
        else if (a == "--seed") { int s; next(s); seed = (unsigned)s; }
        else if (a == "--T") next(T);
        else if (a == "--d") next(d);
        else if (a == "--block") next(block);
        else if (a == "--gpus") next(gpus);
        else if (a == "-h" || a == "--help") return usage(argv[0]);
        else pos.push_back(a);
    }
    const int need_min[] = {2, 3, 4, 0};
    if ((int)pos.size() < need_min[SA_DRIVER_MODE] || (SA_DRIVER_MODE == 3 && !pos.empty())) return usage(argv[0]);
    if (pos.size() > 0) T = std::atoi(pos[0].c_str());
    if (pos.size() > 1) d = std::atoi(pos[1].c_str());
    if (pos.size() > 2) block = std::atoi(pos[2].c_str());
    if (pos.size() > 3) gpus = std::atoi(pos[3].c_str());
    if (T <= 0 || d <= 0 || block <= 0 || gpus <= 0 || iters <= 0) return usage(argv[0]);

    std::mt19937 gen(seed);
    std::uniform_real_distribution<float> dist(-1.0f, 1.0f);
    std::vector<float> Q(d), K((size_t)T * d), V((size_t)T * d);
    for (auto& x : Q) x = dist(gen);
    for (auto& x : K) x = dist(gen);
    for (auto& x : V) x = dist(gen);

    const char* names[] = {"naive (cuda)", "streaming (cuda)", "streaming, KV split over GPUs (cuda)",
                           "streaming, KV split over GPUs (cuda)"};
    auto run = [&]() -> std::vector<float> {
        switch (SA_DRIVER_MODE) {
            case 0: return naive_attention_cuda(Q.data(), K.data(), V.data(), T, d);
            case 1: return streaming_attention_cuda(Q.data(), K.data(), V.data(), T, d, block);
            default: return streaming_attention_cuda_multi(Q.data(), K.data(), V.data(), T, d, block, gpus);
        }
    };
    try {
        std::vector<float> out = run();   // warm-up: contexts, staging buffers
        const auto t0 = std::chrono::steady_clock::now();
        for (int it = 0; it < iters; ++it) out = run();
        const auto t1 = std::chrono::steady_clock::now();
        const double ms = std::chrono::duration<double, std::milli>(t1 - t0).count() / iters;
        const std::vector<double> ref = softmax_attention_f64(Q.data(), K.data(), V.data(), T, d);
        double err = 0.0, sum = 0.0;
        for (int i = 0; i < d; ++i) {
            err = std::max(err, std::fabs((double)out[i] - ref[i]));
            sum += out[i];
        }
        std::printf("Method: %s  T=%d d=%d block=%d%s\n", names[SA_DRIVER_MODE], T, d, block,
                    SA_DRIVER_MODE >= 2 ? (" gpus=" + std::to_string(gpus)).c_str() : "");
        std::printf("Time: %.4f ms\n", ms);
        std::printf("Bandwidth: %.2f GB/s (K and V read once)\n", 2.0 * T * d * 4 / (ms * 1e6));
        std::printf("Output checksum: %.6f\n", sum);
        std::printf("Max error vs fp64 softmax: %.3e\n", err);
        attention_cuda_release();
        return err <= 1e-4 ? 0 : 1;
    } catch (const std::exception& e) {
        std::fprintf(stderr, "error: %s\n", e.what());
        return 1;
    }
}
