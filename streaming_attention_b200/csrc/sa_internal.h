// sa_internal.h -- context object and error plumbing shared by the C-ABI
// translation units of libsa_cuda.so.
#pragma once
#include <cuda_runtime.h>
#include <cstdarg>
#include <cstddef>
#include <cstdio>
#include <cstdlib>
#include <string>

#include "../../include/sa_cuda.h"

#define SA_API extern "C" __attribute__((visibility("default")))

// Largest number of KV heads a decode call may use (size of the per-head
// completion counters the last-CTA merge uses).
#define SA_MAX_KV_HEADS 1024

struct sa_ctx {
    int device = 0;
    int num_sms = 0;
    cudaStream_t own_stream = nullptr;
    cudaStream_t stream = nullptr;
    // grow-only device scratch (split partials etc.)
    void* ws = nullptr;
    size_t ws_bytes = 0;
    // per-KV-head arrival counters for the decode kernel's last-CTA merge;
    // zero between launches (the last CTA resets its counter)
    unsigned* counters = nullptr;
    // device status word: 0 ok, else a SA_STATUS_* code set by a kernel
    int* status = nullptr;
    // grow-only device staging for SA_HOST_PTRS calls
    void* stage = nullptr;
    size_t stage_bytes = 0;
};

namespace sa {

int set_error(int code, const char* fmt, ...);
void clear_error();

// Switch to the context's device for the duration of a call.
struct DeviceGuard {
    int prev = -1;
    explicit DeviceGuard(int dev) {
        cudaGetDevice(&prev);
        if (prev != dev) cudaSetDevice(dev);
    }
    ~DeviceGuard() {
        int cur = -1;
        cudaGetDevice(&cur);
        if (prev >= 0 && cur != prev) cudaSetDevice(prev);
    }
};

// Ensure ctx->ws holds at least `bytes` (grow-only; synchronises on growth).
int ensure_ws(sa_ctx* ctx, size_t bytes);
// Ensure ctx->stage holds at least `bytes`.
int ensure_stage(sa_ctx* ctx, size_t bytes);
// Synchronise the stream and translate CUDA / device-status errors.
int sync_and_check(sa_ctx* ctx);

inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

}  // namespace sa

namespace sa {
// Launch `k` with programmatic stream serialization (PDL): the kernel may start
// while the previous kernel in the stream drains; it must call pdl_wait()
// before reading that kernel's outputs.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*k)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                              Args... args);
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl_k(int kind, void (*k)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                                Args... args) {
    static const int mask = std::getenv("SA_PDL_MASK") ? std::atoi(std::getenv("SA_PDL_MASK")) : -1;
    if (!(mask & (1 << kind))) {
        k<<<grid, block, smem, st>>>(static_cast<KArgs>(args)...);
        return cudaGetLastError();
    }
    return launch_pdl(k, grid, block, smem, st, args...);
}
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*k)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                              Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    static const bool disabled = std::getenv("SA_NO_PDL") != nullptr;   // ordinary launches if set
    cfg.numAttrs = disabled ? 0 : 1;
    return cudaLaunchKernelEx(&cfg, k, static_cast<KArgs>(args)...);
}
}  // namespace sa

#define SA_CUDA_TRY(expr)                                                          \
    do {                                                                           \
        cudaError_t e_ = (expr);                                                   \
        if (e_ != cudaSuccess)                                                     \
            return sa::set_error(SA_ERR_CUDA, "%s failed: %s (%s:%d)", #expr,      \
                                 cudaGetErrorString(e_), __FILE__, __LINE__);      \
    } while (0)

#define SA_RC_TRY(expr)                                                            \
    do {                                                                           \
        int rc_ = (expr);                                                          \
        if (rc_) return rc_;                                                       \
    } while (0)

#define SA_CHECK_ARG(cond, ...)                                                    \
    do {                                                                           \
        if (!(cond)) return sa::set_error(SA_ERR_ARG, __VA_ARGS__);                \
    } while (0)
