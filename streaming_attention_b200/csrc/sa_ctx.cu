// sa_ctx.cu -- context lifetime, error reporting and scratch management for
// libsa_cuda.so.
#include "sa_internal.h"
#include "sa_ptx.cuh"

namespace sa {

// A plain array, not a std::string: it has no destructor, so a call made
// while the process exits (a static object's destructor destroying its
// context after the thread's thread_local objects are gone) still writes
// into live memory.
static thread_local char g_last_error[1024];

int set_error(int code, const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
    va_end(ap);
    return code;
}

void clear_error() { g_last_error[0] = '\0'; }

int ensure_ws(sa_ctx* ctx, size_t bytes) {
    if (bytes <= ctx->ws_bytes) return SA_OK;
    size_t nb = align_up(bytes > 2 * ctx->ws_bytes ? bytes : 2 * ctx->ws_bytes, 1 << 20);
    if (ctx->ws) {
        SA_CUDA_TRY(cudaStreamSynchronize(ctx->stream));
        SA_CUDA_TRY(cudaFree(ctx->ws));
        ctx->ws = nullptr;
        ctx->ws_bytes = 0;
    }
    if (cudaMalloc(&ctx->ws, nb) != cudaSuccess) {
        cudaGetLastError();
        return set_error(SA_ERR_OOM, "cudaMalloc of %zu scratch bytes failed", nb);
    }
    ctx->ws_bytes = nb;
    return SA_OK;
}

int ensure_stage(sa_ctx* ctx, size_t bytes) {
    if (bytes <= ctx->stage_bytes) return SA_OK;
    size_t nb = align_up(bytes, 1 << 20);
    if (ctx->stage) {
        SA_CUDA_TRY(cudaStreamSynchronize(ctx->stream));
        SA_CUDA_TRY(cudaFree(ctx->stage));
        ctx->stage = nullptr;
        ctx->stage_bytes = 0;
    }
    if (cudaMalloc(&ctx->stage, nb) != cudaSuccess) {
        cudaGetLastError();
        return set_error(SA_ERR_OOM, "cudaMalloc of %zu staging bytes failed", nb);
    }
    ctx->stage_bytes = nb;
    return SA_OK;
}

int sync_and_check(sa_ctx* ctx) {
    SA_CUDA_TRY(cudaStreamSynchronize(ctx->stream));
    int st = 0;
    SA_CUDA_TRY(cudaMemcpy(&st, ctx->status, sizeof(int), cudaMemcpyDeviceToHost));
    if (st != SA_STATUS_OK) {
        int zero = 0;
        cudaMemcpy(ctx->status, &zero, sizeof(int), cudaMemcpyHostToDevice);
        if (st == SA_STATUS_TIMEOUT)
            return set_error(SA_ERR_TIMEOUT, "a device-side wait exceeded its limit");
        return set_error(SA_ERR_RANGE, "a kernel reported an out-of-range index (status %d)", st);
    }
    return SA_OK;
}

}  // namespace sa

SA_API const char* sa_last_error(void) { return sa::g_last_error; }

SA_API const char* sa_version(void) { return "sa_cuda 0.1 (sm_100a)"; }

SA_API int sa_device_count(int* out) {
    sa::clear_error();
    SA_CHECK_ARG(out != nullptr, "sa_device_count: out is NULL");
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) {
        cudaGetLastError();
        n = 0;
    }
    *out = n;
    return SA_OK;
}

SA_API int sa_ctx_create(int device, sa_ctx** out) {
    sa::clear_error();
    SA_CHECK_ARG(out != nullptr, "sa_ctx_create: out is NULL");
    *out = nullptr;
    int n = 0;
    SA_CUDA_TRY(cudaGetDeviceCount(&n));
    SA_CHECK_ARG(device >= 0 && device < n, "sa_ctx_create: device %d of %d", device, n);
    sa::DeviceGuard g(device);
    SA_CUDA_TRY(cudaSetDevice(device));
    cudaDeviceProp prop;
    SA_CUDA_TRY(cudaGetDeviceProperties(&prop, device));
    if (prop.major != 10)
        return sa::set_error(SA_ERR_ARG, "sa_ctx_create: device %d is sm_%d%d; this library is built "
                             "for sm_100a (B200) only", device, prop.major, prop.minor);
    sa_ctx* c = new sa_ctx();
    c->device = device;
    c->num_sms = prop.multiProcessorCount;
    if (cudaStreamCreateWithFlags(&c->own_stream, cudaStreamNonBlocking) != cudaSuccess ||
        cudaMalloc(&c->counters, SA_MAX_KV_HEADS * sizeof(unsigned)) != cudaSuccess ||
        cudaMalloc(&c->status, sizeof(int)) != cudaSuccess) {
        cudaError_t e = cudaGetLastError();
        if (c->counters) cudaFree(c->counters);
        if (c->own_stream) cudaStreamDestroy(c->own_stream);
        delete c;
        return sa::set_error(SA_ERR_CUDA, "sa_ctx_create: %s", cudaGetErrorString(e));
    }
    c->stream = c->own_stream;
    SA_CUDA_TRY(cudaMemset(c->counters, 0, SA_MAX_KV_HEADS * sizeof(unsigned)));
    SA_CUDA_TRY(cudaMemset(c->status, 0, sizeof(int)));
    *out = c;
    return SA_OK;
}

SA_API int sa_ctx_destroy(sa_ctx* ctx) {
    sa::clear_error();
    if (!ctx) return SA_OK;
    sa::DeviceGuard g(ctx->device);
    cudaStreamSynchronize(ctx->stream);
    cudaFree(ctx->ws);
    cudaFree(ctx->stage);
    cudaFree(ctx->counters);
    cudaFree(ctx->status);
    cudaStreamDestroy(ctx->own_stream);
    delete ctx;
    return SA_OK;
}

SA_API int sa_ctx_set_stream(sa_ctx* ctx, void* stream) {
    sa::clear_error();
    SA_CHECK_ARG(ctx != nullptr, "sa_ctx_set_stream: ctx is NULL");
    // NULL is CUDA's legacy default stream (the one torch's default stream
    // handle 0 denotes), never the context's own non-blocking stream: work
    // issued by the caller on stream 0 must stay ordered with this library's.
    ctx->stream = stream ? static_cast<cudaStream_t>(stream) : cudaStreamLegacy;
    return SA_OK;
}

SA_API void* sa_ctx_stream(sa_ctx* ctx) { return ctx ? (void*)ctx->stream : nullptr; }

SA_API int sa_ctx_num_sms(sa_ctx* ctx) { return ctx ? ctx->num_sms : 0; }

SA_API int sa_ctx_synchronize(sa_ctx* ctx) {
    sa::clear_error();
    SA_CHECK_ARG(ctx != nullptr, "sa_ctx_synchronize: ctx is NULL");
    sa::DeviceGuard g(ctx->device);
    return sa::sync_and_check(ctx);
}
