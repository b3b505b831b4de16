// sa_tmap.cu -- host-side TMA tensor-map encoding.  cuTensorMapEncodeTiled is
// a driver API; it is fetched through the runtime's driver entry point so the
// library does not link libcuda directly.
#include <cudaTypedefs.h>
#include <map>
#include <mutex>
#include <set>
#include <tuple>

#include "sa_internal.h"
#include "sa_tc.cuh"

namespace sa {

static PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
static std::once_flag g_encode_once;

static int get_encode() {
    std::call_once(g_encode_once, [] {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fn, 12000, cudaEnableDefault, &q) ==
                cudaSuccess && q == cudaDriverEntryPointSuccess)
            g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    });
    if (!g_encode) return set_error(SA_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
    return SA_OK;
}

int make_tmap_2d_bf16(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols,
                      uint64_t row_stride_elems, uint32_t box_rows, uint32_t box_cols) {
    int rc = get_encode();
    if (rc) return rc;
    SA_CHECK_ARG(((uintptr_t)base & 15) == 0, "tensor map base not 16-byte aligned");
    SA_CHECK_ARG((row_stride_elems * 2) % 16 == 0, "tensor map row stride not a multiple of 16 bytes");
    cuuint64_t dims[2] = {cols, rows};
    cuuint64_t strides[1] = {row_stride_elems * 2};
    cuuint32_t box[2] = {box_cols, box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides,
                          box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
        return set_error(SA_ERR_ARG, "cuTensorMapEncodeTiled failed (%d): rows=%llu cols=%llu stride=%llu box=%ux%u",
                         (int)r, (unsigned long long)rows, (unsigned long long)cols,
                         (unsigned long long)row_stride_elems, box_rows, box_cols);
    return SA_OK;
}

// 2-D fp32 tensor map over a row-major [rows, cols] block (row stride
// row_stride_elems), box [box_rows, 32 columns], 128-byte swizzle: KV-cache
// rows for the prompt attention (16-byte chunk q of row r lands at chunk
// q ^ (r % 8) of the row's 128 bytes in shared memory).
int make_tmap_2d_f32_sw128(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols,
                           uint64_t row_stride_elems, uint32_t box_rows) {
    int rc = get_encode();
    if (rc) return rc;
    SA_CHECK_ARG(((uintptr_t)base & 15) == 0 && (row_stride_elems * 4) % 16 == 0 && cols % 32 == 0,
                 "fp32 tensor map alignment");
    cuuint64_t dims[2] = {cols, rows};
    cuuint64_t strides[1] = {row_stride_elems * 4};
    cuuint32_t box[2] = {32, box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void*>(base), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
        return set_error(SA_ERR_ARG, "cuTensorMapEncodeTiled failed (%d): fp32 rows=%llu cols=%llu", (int)r,
                         (unsigned long long)rows, (unsigned long long)cols);
    return SA_OK;
}

int cached_tmap_2d_f32_sw128(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols,
                             uint64_t row_stride_elems, uint32_t box_rows) {
    using Key = std::tuple<const void*, uint64_t, uint64_t, uint64_t, uint32_t>;
    static std::mutex mu;
    static std::map<Key, CUtensorMap> cache;
    const Key key{base, rows, cols, row_stride_elems, box_rows};
    {
        std::lock_guard<std::mutex> lk(mu);
        auto it = cache.find(key);
        if (it != cache.end()) {
            *map = it->second;
            return SA_OK;
        }
    }
    int rc = make_tmap_2d_f32_sw128(map, base, rows, cols, row_stride_elems, box_rows);
    if (rc) return rc;
    std::lock_guard<std::mutex> lk(mu);
    if (cache.size() > 8192) cache.clear();
    cache.emplace(key, *map);
    return SA_OK;
}

// 3-D fp32 tensor map over `splits` stacked row-major [rows, cols] planes
// (split partial sums), box 128 rows x 32 columns x 1 plane, 128-byte swizzle:
// the tensor-store destination of the prompt GEMM's split partials.
int make_tmap_3d_f32_planes(CUtensorMap* map, void* base, uint64_t rows, uint64_t cols, uint64_t splits) {
    int rc = get_encode();
    if (rc) return rc;
    SA_CHECK_ARG(((uintptr_t)base & 15) == 0 && (cols * 4) % 16 == 0, "partial-plane tensor map alignment");
    cuuint64_t dims[3] = {cols, rows, splits};
    cuuint64_t strides[2] = {cols * 4, rows * cols * 4};
    cuuint32_t box[3] = {32, 128, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, base, dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
        return set_error(SA_ERR_ARG, "cuTensorMapEncodeTiled failed (%d): planes %llu x %llu x %llu", (int)r,
                         (unsigned long long)splits, (unsigned long long)rows, (unsigned long long)cols);
    return SA_OK;
}

int cached_tmap_3d_f32_planes(CUtensorMap* map, void* base, uint64_t rows, uint64_t cols, uint64_t splits) {
    using Key = std::tuple<const void*, uint64_t, uint64_t, uint64_t>;
    static std::mutex mu;
    static std::map<Key, CUtensorMap> cache;
    const Key key{base, rows, cols, splits};
    {
        std::lock_guard<std::mutex> lk(mu);
        auto it = cache.find(key);
        if (it != cache.end()) {
            *map = it->second;
            return SA_OK;
        }
    }
    int rc = make_tmap_3d_f32_planes(map, base, rows, cols, splits);
    if (rc) return rc;
    std::lock_guard<std::mutex> lk(mu);
    if (cache.size() > 8192) cache.clear();
    cache.emplace(key, *map);
    return SA_OK;
}

// Tensor maps depend only on (address, shape, stride, box); the Qwen3 forward
// reuses the same few hundred for its fixed buffers, so encode each once.
int cached_tmap_2d_bf16(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols,
                        uint64_t row_stride_elems, uint32_t box_rows, uint32_t box_cols) {
    using Key = std::tuple<const void*, uint64_t, uint64_t, uint64_t, uint32_t, uint32_t>;
    static std::mutex mu;
    static std::map<Key, CUtensorMap> cache;
    const Key key{base, rows, cols, row_stride_elems, box_rows, box_cols};
    {
        std::lock_guard<std::mutex> lk(mu);
        auto it = cache.find(key);
        if (it != cache.end()) {
            *map = it->second;
            return SA_OK;
        }
    }
    int rc = make_tmap_2d_bf16(map, base, rows, cols, row_stride_elems, box_rows, box_cols);
    if (rc) return rc;
    std::lock_guard<std::mutex> lk(mu);
    if (cache.size() > 8192) cache.clear();
    cache.emplace(key, *map);
    return SA_OK;
}

// cudaFuncSetAttribute(MaxDynamicSharedMemorySize) once per (function, device).
int set_smem_attr_once(const void* fn, int bytes) {
    static std::mutex mu;
    static std::set<std::pair<int, const void*>> done;
    int dev = 0;
    SA_CUDA_TRY(cudaGetDevice(&dev));
    std::lock_guard<std::mutex> lk(mu);
    if (done.count({dev, fn})) return SA_OK;
    SA_CUDA_TRY(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
    done.insert({dev, fn});
    return SA_OK;
}

}  // namespace sa
