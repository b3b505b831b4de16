// benchmark_qwen3_cuda -- the CUDA method of tensor_cpp's Qwen3 benchmark
// driver (tensor_cpp/tests/benchmark/benchmark_qwen3.cpp), over the C ABI of
// libsa_cuda.so.
//
// It takes that driver's options (--model, --phase prefill|decode, --method,
// --parallel-strategy headwise|sequence, --attention-algo, the legacy
// --attention, --prompt-len, --gen-len, --iters, --warmup, --batch-size, ...)
// plus --gpus N, and prints the same "Benchmark Results" block (total time,
// tokens processed, time per token, throughput).  Unlike the reference's
// parser (benchmark_qwen3.cpp:199-217), the legacy --attention does not
// override an explicit --parallel-strategy / --attention-algo, so head-wise
// and sequence parallelism can both be selected:
//   headwise -> sa_qwen3_load_safetensors_tp (KV heads split over the GPUs)
//   sequence -> sa_qwen3_load_safetensors_sp (prompt tokens split over the GPUs)
// Both attention algorithms (standard, online_softmax) compute the same
// softmax attention on the GPU.
//
// With --gpus N > 1 the driver forks one process per GPU before touching
// CUDA; the ranks swap their exchange handles through shared memory.  Timing
// is wall clock around blocking calls, as the reference times; the reported
// time is the slowest rank's.
//
//   prefill: --warmup then --iters cache-free forwards of --prompt-len random
//            tokens (mt19937(42), as generate_random_tokens) with the logits of
//            every position; tokens = prompt_len * iters.
//   decode:  greedy decode of --gen-len tokens after a --prompt-len prompt
//            with the KV cache; the time of generate(prompt, gen_len + 1)
//            minus that of generate(prompt, 1), i.e. the gen_len decode steps.
//            The generated tokens are printed (the same for every strategy).
#include <sys/mman.h>
#include <sys/wait.h>
#include <unistd.h>

#include <algorithm>
#include <atomic>
#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <random>
#include <string>
#include <thread>
#include <vector>

#include "sa_cuda.h"

namespace {

struct Config {
    std::string model, phase = "prefill", method = "cuda", strategy, algo, attention;
    int batch = 1, prompt_len = 128, gen_len = 100, iters = 5, warmup = 2, gpus = 1;
    bool use_cache = true, verbose = false;
};

int usage(const char* prog) {
    std::fprintf(stderr,
                 "usage: %s --model PATH [--phase prefill|decode] [--method cuda]\n"
                 "       [--parallel-strategy headwise|sequence] [--attention-algo standard|online_softmax]\n"
                 "       [--attention standard|streaming] [--gpus N] [--prompt-len N] [--gen-len N]\n"
                 "       [--iters N] [--warmup N] [--batch-size 1] [--use-kv-cache] [--verbose]\n"
                 "  (--mode, --threads, --q-block-size, --kv-block-size are accepted and ignored)\n",
                 prog);
    return 2;
}

bool parse(int argc, char** argv, Config& c) {
    for (int i = 1; i < argc; ++i) {
        const std::string a = argv[i];
        auto val = [&]() -> const char* { return i + 1 < argc ? argv[++i] : nullptr; };
        const char* v = nullptr;
        if (a == "--model" && (v = val())) c.model = v;
        else if (a == "--phase" && (v = val())) c.phase = v;
        else if (a == "--method" && (v = val())) c.method = v;
        else if (a == "--parallel-strategy" && (v = val())) c.strategy = v;
        else if (a == "--attention-algo" && (v = val())) c.algo = v;
        else if (a == "--attention" && (v = val())) c.attention = v;
        else if (a == "--batch-size" && (v = val())) c.batch = std::atoi(v);
        else if (a == "--prompt-len" && (v = val())) c.prompt_len = std::atoi(v);
        else if (a == "--gen-len" && (v = val())) c.gen_len = std::atoi(v);
        else if (a == "--iters" && (v = val())) c.iters = std::atoi(v);
        else if (a == "--warmup" && (v = val())) c.warmup = std::atoi(v);
        else if (a == "--gpus" && (v = val())) c.gpus = std::atoi(v);
        else if ((a == "--mode" || a == "--threads" || a == "--q-block-size" || a == "--kv-block-size") && val()) continue;
        else if (a == "--use-kv-cache") c.use_cache = true;
        else if (a == "--no-kv-cache") c.use_cache = false;
        else if (a == "--verbose") c.verbose = true;
        else return false;
    }
    // the legacy option only fills in what was not given explicitly
    if (c.attention == "streaming") {
        if (c.strategy.empty()) c.strategy = "headwise";
        if (c.algo.empty()) c.algo = "online_softmax";
    } else if (c.attention == "standard") {
        if (c.strategy.empty()) c.strategy = "headwise";
        if (c.algo.empty()) c.algo = "standard";
    } else if (!c.attention.empty()) {
        return false;
    }
    if (c.strategy.empty()) c.strategy = "headwise";
    if (c.algo.empty()) c.algo = "standard";
    return !c.model.empty() && (c.phase == "prefill" || c.phase == "decode") &&
           (c.strategy == "headwise" || c.strategy == "sequence") &&
           (c.algo == "standard" || c.algo == "online_softmax") && c.prompt_len >= 1 && c.gen_len >= 1 &&
           c.iters >= 1 && c.warmup >= 0 && c.gpus >= 1 && c.gpus <= 8;
}

// What the ranks share (an anonymous shared mapping made before fork).
struct Shared {
    std::atomic<int> arrived;
    std::atomic<int> failed;
    char handles[8][SA_QWEN3_SP_HANDLE_BYTES];
    double ms[8];
    long long tokens[8][128];
};

bool barrier(Shared* sh, int world, int& gen) {
    ++gen;
    sh->arrived.fetch_add(1);
    for (int i = 0; i < 600000; ++i) {            // bounded: 60 s
        if (sh->failed.load()) return false;
        if (sh->arrived.load() >= world * gen) return true;
        std::this_thread::sleep_for(std::chrono::microseconds(100));
    }
    return false;
}

std::vector<int64_t> random_tokens(int n, int vocab) {   // generate_random_tokens (benchmark_qwen3.cpp:223-234)
    std::mt19937 gen(42);
    std::uniform_int_distribution<long> dist(0, vocab - 1);
    std::vector<int64_t> t(n);
    for (auto& x : t) x = dist(gen);
    return t;
}

double now_ms() {
    return std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now().time_since_epoch()).count();
}

int fail(Shared* sh, int rank, const char* what) {
    std::fprintf(stderr, "rank %d: %s: %s\n", rank, what, sa_last_error());
    if (sh) sh->failed.store(1);
    return 1;
}

// One rank's run; returns the process exit code.
int run_rank(const Config& c, int rank, int world, Shared* sh) {
    int gen = 0;
    sa_ctx* ctx = nullptr;
    if (sa_ctx_create(rank, &ctx)) return fail(sh, rank, "sa_ctx_create");
    const int max_seq = c.prompt_len + (c.phase == "decode" ? c.gen_len + 8 : 8);
    sa_qwen3* m = nullptr;
    int rc;
    if (world == 1)
        rc = sa_qwen3_load_safetensors(ctx, c.model.c_str(), max_seq, 0.f, 0.f, &m);
    else if (c.strategy == "sequence")
        rc = sa_qwen3_load_safetensors_sp(ctx, c.model.c_str(), max_seq, 0.f, 0.f, rank, world, &m);
    else
        rc = sa_qwen3_load_safetensors_tp(ctx, c.model.c_str(), max_seq, 0.f, 0.f, rank, world, &m);
    if (rc) return fail(sh, rank, "loading the checkpoint");
    sa_qwen3_config cfg;
    if (sa_safetensors_inspect(c.model.c_str(), &cfg)) return fail(sh, rank, "sa_safetensors_inspect");
    if (world > 1) {
        const bool seq = c.strategy == "sequence";
        const int hb = seq ? SA_QWEN3_SP_HANDLE_BYTES : SA_TP_HANDLE_BYTES;
        if ((seq ? sa_qwen3_sp_handle(m, sh->handles[rank]) : sa_qwen3_tp_handle(m, sh->handles[rank])))
            return fail(sh, rank, "handle");
        if (!barrier(sh, world, gen)) return fail(sh, rank, "waiting for the other ranks' handles");
        std::vector<char> all((size_t)world * hb);
        for (int r = 0; r < world; ++r) std::memcpy(all.data() + (size_t)r * hb, sh->handles[r], hb);
        if ((seq ? sa_qwen3_sp_connect(m, all.data()) : sa_qwen3_tp_connect(m, all.data())))
            return fail(sh, rank, "connect");
    }
    const std::vector<int64_t> ids = random_tokens(c.prompt_len, cfg.vocab);
    double ms = 0.0;
    std::vector<int64_t> toks;
    if (c.phase == "prefill") {
        std::vector<float> logits((size_t)c.prompt_len * cfg.vocab);
        for (int i = 0; i < c.warmup; ++i)
            if (sa_qwen3_forward(m, ids.data(), c.prompt_len, 0, logits.data(), 0, SA_HOST_PTRS))
                return fail(sh, rank, "forward");
        if (world > 1 && !barrier(sh, world, gen)) return fail(sh, rank, "barrier");
        const double t0 = now_ms();
        for (int i = 0; i < c.iters; ++i)
            if (sa_qwen3_forward(m, ids.data(), c.prompt_len, 0, logits.data(), 0, SA_HOST_PTRS))
                return fail(sh, rank, "forward");
        ms = now_ms() - t0;
    } else {
        toks.resize((size_t)c.gen_len + 1);
        auto gen_time = [&](int n) -> double {
            if (sa_qwen3_reset(m)) return -1.0;
            if (world > 1 && !barrier(sh, world, gen)) return -1.0;
            const double t0 = now_ms();
            if (sa_qwen3_generate(m, ids.data(), c.prompt_len, n, toks.data(), SA_HOST_PTRS)) return -1.0;
            return now_ms() - t0;
        };
        for (int i = 0; i < std::max(1, c.warmup); ++i)
            if (gen_time(c.gen_len + 1) < 0) return fail(sh, rank, "generate");
        double best_long = 1e30, best_short = 1e30;
        for (int i = 0; i < c.iters; ++i) {
            const double tl = gen_time(c.gen_len + 1);
            if (tl < 0) return fail(sh, rank, "generate");
            best_long = std::min(best_long, tl);
        }
        for (int i = 0; i < c.iters; ++i) {
            const double ts = gen_time(1);
            if (ts < 0) return fail(sh, rank, "generate");
            best_short = std::min(best_short, ts);
        }
        if (gen_time(c.gen_len + 1) < 0) return fail(sh, rank, "generate");   // the tokens to print
        ms = std::max(best_long - best_short, 1e-6);
    }
    if (sh) {
        sh->ms[rank] = ms;
        for (size_t i = 0; i < toks.size() && i < 128; ++i) sh->tokens[rank][i] = toks[i];
        if (!barrier(sh, world, gen)) return fail(sh, rank, "barrier");
    }
    if (rank == 0) {
        double worst = ms;
        if (sh)
            for (int r = 0; r < world; ++r) worst = std::max(worst, sh->ms[r]);
        const long long ntok = c.phase == "prefill" ? (long long)c.prompt_len * c.iters : c.gen_len;
        std::printf("==================================================\n");
        std::printf("         Qwen3 Performance Benchmark\n");
        std::printf("==================================================\n");
        std::printf("模型路径:       %s\n", c.model.c_str());
        std::printf("测试阶段:       %s\n", c.phase.c_str());
        std::printf("优化方法:       CUDA (%s)\n", sa_version());
        std::printf("并行策略:       %s\n", c.strategy.c_str());
        std::printf("Attention算法:  %s\n", c.algo.c_str());
        std::printf("GPU数:          %d\n", world);
        std::printf("Prompt长度:     %d\n", c.prompt_len);
        if (c.phase == "decode") std::printf("生成长度:       %d\n", c.gen_len);
        std::printf("迭代次数:       %d\n", c.iters);
        std::printf("==================================================\n\n");
        std::printf("==================================================\n");
        std::printf("              Benchmark Results\n");
        std::printf("==================================================\n");
        std::printf("总时间:         %.2f ms\n", worst);
        std::printf("处理token数:    %lld\n", ntok);
        std::printf("平均时间/token: %.4f ms\n", worst / (double)ntok);
        std::printf("吞吐量:         %.2f tokens/sec\n", (double)ntok / (worst / 1e3));
        std::printf("==================================================\n");
        if (c.phase == "decode") {
            std::printf("生成tokens:    ");
            for (int i = 0; i < c.gen_len && i < 128; ++i) std::printf(" %lld", (long long)toks[i]);
            std::printf("\n");
            if (sh)
                for (int r = 1; r < world; ++r)
                    for (int i = 0; i < c.gen_len && i < 128; ++i)
                        if (sh->tokens[r][i] != toks[i]) {
                            std::fprintf(stderr, "rank %d generated other tokens than rank 0\n", r);
                            return 1;
                        }
        }
    }
    sa_qwen3_destroy(m);
    sa_ctx_destroy(ctx);
    return 0;
}

}  // namespace

int main(int argc, char** argv) {
    Config c;
    if (!parse(argc, argv, c)) return usage(argv[0]);
    std::fflush(stdout);   // nothing buffered is duplicated into the forked ranks
    if (c.method != "cuda") {
        std::fprintf(stderr, "this driver runs --method cuda (got %s)\n", c.method.c_str());
        return 2;
    }
    if (c.batch != 1 || !c.use_cache) {
        std::fprintf(stderr, "the CUDA method benchmarks batch 1 with the KV cache\n");
        return 2;
    }
    if (c.gpus == 1) return run_rank(c, 0, 1, nullptr);
    // one process per GPU, forked before any CUDA call
    void* mem = mmap(nullptr, sizeof(Shared), PROT_READ | PROT_WRITE, MAP_SHARED | MAP_ANONYMOUS, -1, 0);
    if (mem == MAP_FAILED) return 1;
    Shared* sh = new (mem) Shared();
    std::vector<pid_t> kids;
    for (int r = 0; r < c.gpus; ++r) {
        const pid_t p = fork();
        if (p == 0) {
            const int code = run_rank(c, r, c.gpus, sh);
            std::fflush(stdout);   // _exit does not flush stdio
            std::fflush(stderr);
            _exit(code);
        }
        if (p < 0) {
            sh->failed.store(1);
            break;
        }
        kids.push_back(p);
    }
    int code = (int)kids.size() == c.gpus ? 0 : 1;
    for (pid_t p : kids) {
        int st = 0;
        waitpid(p, &st, 0);
        if (!WIFEXITED(st) || WEXITSTATUS(st) != 0) code = 1;
    }
    return code;
}
