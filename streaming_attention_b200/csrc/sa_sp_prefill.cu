// sa_sp_prefill.cu -- sequence-parallel causal prefill over the GPUs of one
// node (configs[2]: S = 8192, 16 / 8 heads of 128, bf16), one rank per GPU.
//
// Replaces the reference's sequence-parallel attention
// (attention_sequence_online_softmax, tensor_cpp/src/ops_mpi.cpp:1000-1212,
// whose statistics all-reduce mixes positions) with the causal prefill the
// strategy stands for: the sequence is cut into 2P chunks of C = S / 2P
// tokens and rank r holds chunks r and 2P-1-r (zig-zag), which gives every
// rank the same causal work.
//
// One call, all on the context's stream:
//   1. spp_scatter_kernel: the rank's K and V chunks go straight into slot
//      (instance & 1) of EVERY rank's K/V buffer (its own and the peers',
//      mapped over CUDA IPC or peer access) at their sequence rows, with
//      16-byte stores; after a system-scope fence and an arrival count, the
//      last CTA stores the instance's epoch into flag [slot][rank] of every
//      rank (release, system scope).
//   2. spp_wait_kernel: one thread per rank waits (bounded by %globaltimer)
//      until this rank's flag [slot][r] carries the epoch: all K/V rows of
//      the sequence are then in the local buffer.
//   3. prefill_pieces_launch: ONE launch of the tcgen05 prefill over a table
//      of pieces.  Each chunk's key range [0, end of chunk) is cut into blocks
//      of max(C, 1024) keys: the blocks before the chunk are fully visible (no
//      mask), the last one is the causal diagonal of C keys.  So no CTA
//      streams more than a block (the heavy chunk's CTAs would otherwise
//      carry the whole prefix), and a rank's pieces fill the SMs.  Pieces
//      write bf16 partial outputs and their rows' log-sum-exp.
//   4. spp_merge_kernel: out = sum_p 2^(lse_p - lse) O_p over the pieces of
//      each chunk (lse = log2 sum_p 2^lse_p), in the caller's dtype.
// The host counts the calls (the instance: slot = instance & 1, epoch =
// instance + 1); an instance is spent as soon as its exchange is issued.
// Slots alternate between calls, so a rank writing call i+1's rows never
// overwrites rows a slower peer still reads for call i: a rank can only
// start call i+2 after every peer published call i+1, which each does only
// after finishing call i.
#include <cuda_bf16.h>
#include <cstring>

#include "sa_internal.h"
#include "sa_ptx.cuh"
#include "sa_qwen3.h"
#include "sa_spp_plan.h"

constexpr int SPP_MAX = 8;

struct sa_spp {
    sa_ctx* ctx = nullptr;
    int device = 0, rank = 0, world = 1;
    int max_seq = 0, hkv = 0;
    size_t slot_bytes = 0;                     // one slot: K then V, [max_seq][hkv][128] bf16 each
    size_t buf_bytes = 0;
    unsigned char* buf = nullptr;              // own buffer: flags, then 2 slots
    unsigned* ctl = nullptr;                   // [0] arrivals of the scatter's CTAs
    unsigned inst = 0;                         // calls issued (slot = inst & 1, epoch = inst + 1)
    unsigned char* peer[SPP_MAX] = {};
    bool opened[SPP_MAX] = {};
    bool connected = false;
    unsigned char uuid[16] = {};
    float* part = nullptr;                     // piece outputs and their lse
    size_t part_floats = 0;
};

namespace sa {
namespace spp {

constexpr int D = 128;
constexpr int MIN_PIECE_KEYS = 1024;           // shorter key blocks cost more in per-CTA set-up than they balance
constexpr size_t FLAG_BYTES = 4096;            // [2 slots][SPP_MAX] u32 flags, then the K/V slots
constexpr uint32_t MAGIC = 0x50505341u;        // "ASPP"

struct Handle {                                // the SA_SPP_HANDLE_BYTES blob
    cudaIpcMemHandle_t ipc;
    unsigned char uuid[16];
    int32_t rank, world, max_seq, hkv;
    uint64_t buf_bytes;
    uint32_t magic;
};
static_assert(sizeof(Handle) <= SA_SPP_HANDLE_BYTES, "handle size");

struct ScatterArgs {
    const uint4* k;                // this rank's [2C][hkv * 128] bf16 rows as 16-byte vectors
    const uint4* v;
    unsigned char* dst[SPP_MAX];   // every rank's buffer
    int world, rank, C, row_vecs;  // row_vecs = hkv * 128 * 2 / 16
    int chunk[2];                  // the sequence chunks of local rows [0, C) and [C, 2C)
    size_t slot_bytes, tensor_bytes;
    unsigned inst;
    unsigned* cnt;
};

__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// One warp per local row (hkv * 128 bf16 of K and of V): lane l loads
// vectors l, l + 32, ... of both rows (all loads in flight before any store),
// then stores them to the row's sequence position in every rank's buffer.
constexpr int SC_VPL = 4;                      // vectors per lane per tensor (row_vecs <= 128: hkv <= 8)
__global__ void __launch_bounds__(512, 2) spp_scatter_kernel(const ScatterArgs a) {
    const unsigned inst = a.inst;
    const int slot = (int)(inst & 1u);
    const int lane = threadIdx.x & 31;
    const int warps = (gridDim.x * blockDim.x) >> 5;
    unsigned char* base[SPP_MAX];
#pragma unroll
    for (int r = 0; r < SPP_MAX; ++r)
        base[r] = r < a.world ? a.dst[r] + FLAG_BYTES + (size_t)slot * a.slot_bytes : nullptr;
    for (int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; row < 2 * a.C; row += warps) {
        const int half = row >= a.C ? 1 : 0;
        const size_t seq_row = (size_t)(half ? a.chunk[1] : a.chunk[0]) * a.C + (row - half * a.C);
        const uint4* ks = a.k + (size_t)row * a.row_vecs;
        const uint4* vs = a.v + (size_t)row * a.row_vecs;
        uint4 kv[SC_VPL], vv[SC_VPL];
#pragma unroll
        for (int j = 0; j < SC_VPL; ++j) {
            const int c = lane + 32 * j;
            if (c < a.row_vecs) {
                kv[j] = __ldg(ks + c);
                vv[j] = __ldg(vs + c);
            }
        }
        const size_t off = seq_row * a.row_vecs * 16;
#pragma unroll
        for (int r = 0; r < SPP_MAX; ++r) {
            if (r >= a.world) break;
#pragma unroll
            for (int j = 0; j < SC_VPL; ++j) {
                const int c = lane + 32 * j;
                if (c < a.row_vecs) {
                    reinterpret_cast<uint4*>(base[r] + off)[c] = kv[j];
                    reinterpret_cast<uint4*>(base[r] + a.tensor_bytes + off)[c] = vv[j];
                }
            }
        }
    }
    // publish: the CTA barrier orders every thread's stores before thread 0's
    // system-scope fence (fences are cumulative), which orders them before
    // the CTA's arrival; the last CTA to arrive stores the epoch into flag
    // [slot][rank] of every rank
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence_system();
        const unsigned prev = atomicAdd(a.cnt, 1u);
        if (prev == gridDim.x - 1) {
            __threadfence_system();
            *a.cnt = 0u;
            for (int r = 0; r < a.world; ++r)
                st_release_sys(reinterpret_cast<unsigned*>(a.dst[r]) + slot * SPP_MAX + a.rank, inst + 1u);
        }
    }
}

__global__ void spp_wait_kernel(const unsigned* flags, int world, unsigned inst, int* status) {
    const int slot = (int)(inst & 1u);
    const int r = threadIdx.x;
    if (r >= world) return;
    const unsigned* f = flags + slot * SPP_MAX + r;
    if (ld_acquire_sys(f) == inst + 1u) return;
    const unsigned long long t0 = globaltimer();
    while (ld_acquire_sys(f) != inst + 1u) {
        if (*reinterpret_cast<volatile int*>(status) != 0) return;   // another wait already gave up
        if (globaltimer() - t0 > kWaitLimitNs) {
            atomicExch(status, SA_STATUS_TIMEOUT);
            return;
        }
    }
}

constexpr int MAX_CHUNK_PIECES = 16;          // pieces of one chunk (the call checks)

struct MergeArgs {
    const __nv_bfloat16* part;     // piece p's output at part + p * piece_elems, [C][hq][128] bf16
    const float* lse;              // piece p's lse at lse + p * C * hq
    long long piece_elems;
    int C, hq;
    int first[2], count[2];        // pieces of local chunk 0 / 1
    void* out;                     // [2C][hq][128], bf16 or fp32
    int out_bf16;
    const int* status;
};

// Sixteen threads per (local row, head): thread j owns dims 8j..8j+7 (one
// 16-byte load per piece).  Pieces are taken four at a time, their loads
// issued together, and folded in with a running maximum, so a thread holds
// few registers and many (row, head) pairs are in flight per SM.  Rows whose
// pieces were cut short by an expired wait come out NaN.
constexpr int MG = 4;                          // pieces per load group
__global__ void __launch_bounds__(512) spp_merge_kernel(const MergeArgs a) {
    // the status word once per block (a read per warp would queue tens of
    // thousands of requests on one L2 line)
    __shared__ int s_failed;
    if (threadIdx.x == 0) s_failed = *reinterpret_cast<const volatile int*>(a.status) != 0;
    __syncthreads();
    const int j = threadIdx.x & 15;
    const long long w = (blockIdx.x * (long long)blockDim.x + threadIdx.x) >> 4;
    const long long n = 2LL * a.C * a.hq;
    if (w >= n) return;
    const int row = (int)(w / a.hq), h = (int)(w - (long long)row * a.hq);
    const int half = row >= a.C ? 1 : 0, lr = row - half * a.C;
    const int p0 = half ? a.first[1] : a.first[0], np = half ? a.count[1] : a.count[0];
    const size_t lse_off = (size_t)lr * a.hq + h, o_off = lse_off * D + 8 * j;
    const size_t lse_stride = (size_t)a.C * a.hq;
    float mx = -INFINITY, den = 0.f, acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int g = 0; g < np; g += MG) {
        float ls[MG];
        uint4 ov[MG];
#pragma unroll
        for (int i = 0; i < MG; ++i) {
            ls[i] = -INFINITY;
            ov[i] = make_uint4(0u, 0u, 0u, 0u);
            if (g + i < np) {
                ls[i] = __ldg(a.lse + (size_t)(p0 + g + i) * lse_stride + lse_off);
                ov[i] = __ldg(reinterpret_cast<const uint4*>(a.part + (size_t)(p0 + g + i) * a.piece_elems + o_off));
            }
        }
        float gm = mx;
#pragma unroll
        for (int i = 0; i < MG; ++i) gm = fmaxf(gm, ls[i]);
        const float r = ex2(mx - gm);              // rescale what is folded in so far (0 at the start)
        den *= r;
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[e] *= r;
#pragma unroll
        for (int i = 0; i < MG; ++i) {
            const float wt = ex2(ls[i] - gm);      // absent pieces: 2^-inf = 0
            const uint32_t u[4] = {ov[i].x, ov[i].y, ov[i].z, ov[i].w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                acc[2 * e] = fmaf(wt, __uint_as_float(u[e] << 16), acc[2 * e]);
                acc[2 * e + 1] = fmaf(wt, __uint_as_float(u[e] & 0xffff0000u), acc[2 * e + 1]);
            }
            den += wt;
        }
        mx = gm;
    }
    const float inv = s_failed ? __int_as_float(0x7fffffff) : 1.f / den;
    const size_t off = ((size_t)row * a.hq + h) * D + 8 * j;
    if (a.out_bf16) {
        uint4 u;
        uint32_t* up = reinterpret_cast<uint32_t*>(&u);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const __nv_bfloat162 b2 = __floats2bfloat162_rn(acc[2 * e] * inv, acc[2 * e + 1] * inv);
            up[e] = *reinterpret_cast<const uint32_t*>(&b2);
        }
        *reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(a.out) + off) = u;
    } else {
        float4* o = reinterpret_cast<float4*>(static_cast<float*>(a.out) + off);
        o[0] = make_float4(acc[0] * inv, acc[1] * inv, acc[2] * inv, acc[3] * inv);
        o[1] = make_float4(acc[4] * inv, acc[5] * inv, acc[6] * inv, acc[7] * inv);
    }
}

void close_peers(sa_spp* sp) {
    for (int r = 0; r < SPP_MAX; ++r) {
        if (sp->opened[r] && sp->peer[r]) cudaIpcCloseMemHandle(sp->peer[r]);
        sp->opened[r] = false;
        sp->peer[r] = nullptr;
    }
    sp->connected = false;
}

}  // namespace spp
}  // namespace sa

SA_API int sa_spp_create(sa_ctx* ctx, int rank, int world, int max_seq, int hkv, int d, sa_spp** out) {
    using namespace sa;
    clear_error();
    SA_CHECK_ARG(ctx && out, "sa_spp_create: null argument");
    *out = nullptr;
    SA_CHECK_ARG(world >= 1 && world <= SPP_MAX, "sa_spp_create: world = %d (1..%d)", world, SPP_MAX);
    SA_CHECK_ARG(rank >= 0 && rank < world, "sa_spp_create: rank %d of %d", rank, world);
    SA_CHECK_ARG(d == spp::D, "sa_spp_create: d = %d (the tensor-core prefill is built for d = 128)", d);
    SA_CHECK_ARG(hkv >= 1 && hkv <= 8 && max_seq >= 2 * world && max_seq <= (1 << 22),
                 "sa_spp_create: hkv = %d, max_seq = %d", hkv, max_seq);
    DeviceGuard guard(ctx->device);
    sa_spp* sp = new sa_spp();
    sp->ctx = ctx;
    sp->device = ctx->device;
    sp->rank = rank;
    sp->world = world;
    sp->max_seq = max_seq;
    sp->hkv = hkv;
    const size_t tensor_bytes = (size_t)max_seq * hkv * spp::D * 2;
    sp->slot_bytes = 2 * tensor_bytes;
    sp->buf_bytes = spp::FLAG_BYTES + 2 * sp->slot_bytes;
    cudaDeviceProp prop;
    if (cudaGetDeviceProperties(&prop, ctx->device) != cudaSuccess ||
        cudaMalloc(&sp->buf, sp->buf_bytes) != cudaSuccess ||
        cudaMalloc(&sp->ctl, sizeof(unsigned)) != cudaSuccess ||
        cudaMemset(sp->buf, 0, spp::FLAG_BYTES) != cudaSuccess ||
        cudaMemset(sp->ctl, 0, sizeof(unsigned)) != cudaSuccess) {
        const cudaError_t e = cudaGetLastError();
        cudaFree(sp->buf);
        cudaFree(sp->ctl);
        delete sp;
        return set_error(SA_ERR_OOM, "sa_spp_create: %s", cudaGetErrorString(e));
    }
    std::memcpy(sp->uuid, &prop.uuid, sizeof(sp->uuid));
    sp->peer[rank] = sp->buf;
    sp->connected = world == 1;
    *out = sp;
    return SA_OK;
}

SA_API int sa_spp_handle(sa_spp* sp, void* handle) {
    using namespace sa;
    clear_error();
    SA_CHECK_ARG(sp && handle, "sa_spp_handle: null argument");
    DeviceGuard guard(sp->device);
    spp::Handle h;
    std::memset(&h, 0, sizeof(h));
    SA_CUDA_TRY(cudaIpcGetMemHandle(&h.ipc, sp->buf));
    std::memcpy(h.uuid, sp->uuid, sizeof(h.uuid));
    h.rank = sp->rank;
    h.world = sp->world;
    h.max_seq = sp->max_seq;
    h.hkv = sp->hkv;
    h.buf_bytes = sp->buf_bytes;
    h.magic = spp::MAGIC;
    std::memset(handle, 0, SA_SPP_HANDLE_BYTES);
    std::memcpy(handle, &h, sizeof(h));
    return SA_OK;
}

SA_API int sa_spp_connect(sa_spp* sp, const void* handles) {
    using namespace sa;
    clear_error();
    SA_CHECK_ARG(sp && handles, "sa_spp_connect: null argument");
    if (sp->world == 1) return SA_OK;
    SA_CHECK_ARG(!sp->connected, "sa_spp_connect: already connected");
    DeviceGuard guard(sp->device);
    const unsigned char* hb = static_cast<const unsigned char*>(handles);
    for (int r = 0; r < sp->world; ++r) {
        spp::Handle h;
        std::memcpy(&h, hb + (size_t)r * SA_SPP_HANDLE_BYTES, sizeof(h));
        const char* bad = nullptr;
        if (h.magic != spp::MAGIC) bad = "is not an sa_spp handle";
        else if (h.rank != r || h.world != sp->world) bad = "names another rank or world size";
        else if (h.max_seq != sp->max_seq || h.hkv != sp->hkv || h.buf_bytes != sp->buf_bytes)
            bad = "was created with other max_seq / hkv";
        else if (r != sp->rank && std::memcmp(h.uuid, sp->uuid, sizeof(h.uuid)) == 0)
            bad = "is on this rank's GPU (the ranks wait for one another: one GPU per rank)";
        if (bad) {
            spp::close_peers(sp);
            sp->peer[sp->rank] = sp->buf;
            return set_error(SA_ERR_ARG, "sa_spp_connect: handle %d %s", r, bad);
        }
        if (r == sp->rank) continue;
        void* p = nullptr;
        const cudaError_t e = cudaIpcOpenMemHandle(&p, h.ipc, cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess) {
            cudaGetLastError();
            spp::close_peers(sp);
            sp->peer[sp->rank] = sp->buf;
            return set_error(SA_ERR_CUDA, "sa_spp_connect: opening rank %d's buffer failed: %s", r,
                             cudaGetErrorString(e));
        }
        sp->peer[r] = static_cast<unsigned char*>(p);
        sp->opened[r] = true;
    }
    sp->peer[sp->rank] = sp->buf;
    sp->connected = true;
    return SA_OK;
}

SA_API int sa_spp_connect_local(sa_spp* const* sps, int n) {
    using namespace sa;
    clear_error();
    SA_CHECK_ARG(sps && n >= 1 && n <= SPP_MAX, "sa_spp_connect_local: n = %d", n);
    for (int i = 0; i < n; ++i) {
        SA_CHECK_ARG(sps[i] && sps[i]->rank == i && sps[i]->world == n,
                     "sa_spp_connect_local: entry %d is not rank %d of %d", i, i, n);
        SA_CHECK_ARG(!sps[i]->connected || n == 1, "sa_spp_connect_local: rank %d already connected", i);
        SA_CHECK_ARG(sps[i]->buf_bytes == sps[0]->buf_bytes,
                     "sa_spp_connect_local: rank %d was created with other max_seq / hkv", i);
        for (int j = 0; j < i; ++j)
            SA_CHECK_ARG(sps[j]->device != sps[i]->device,
                         "sa_spp_connect_local: ranks %d and %d share GPU %d (one GPU per rank)", j, i,
                         sps[i]->device);
    }
    for (int i = 0; i < n; ++i) {
        DeviceGuard guard(sps[i]->device);
        for (int j = 0; j < n; ++j) {
            if (j == i) continue;
            int can = 0;
            SA_CUDA_TRY(cudaDeviceCanAccessPeer(&can, sps[i]->device, sps[j]->device));
            SA_CHECK_ARG(can, "sa_spp_connect_local: GPU %d cannot access GPU %d", sps[i]->device,
                         sps[j]->device);
            const cudaError_t e = cudaDeviceEnablePeerAccess(sps[j]->device, 0);
            if (e != cudaSuccess && e != cudaErrorPeerAccessAlreadyEnabled)
                return set_error(SA_ERR_CUDA, "sa_spp_connect_local: peer access %d -> %d: %s", sps[i]->device,
                                 sps[j]->device, cudaGetErrorString(e));
            cudaGetLastError();
        }
    }
    for (int i = 0; i < n; ++i) {
        for (int j = 0; j < n; ++j) sps[i]->peer[j] = sps[j]->buf;
        sps[i]->connected = true;
    }
    return SA_OK;
}

SA_API int sa_spp_destroy(sa_spp* sp) {
    using namespace sa;
    clear_error();
    if (!sp) return SA_OK;
    DeviceGuard guard(sp->device);
    cudaDeviceSynchronize();
    spp::close_peers(sp);
    cudaFree(sp->buf);
    cudaFree(sp->ctl);
    cudaFree(sp->part);
    delete sp;
    return SA_OK;
}

SA_API int sa_spp_prefill(sa_spp* sp, const void* q_local, const void* k_local, const void* v_local, int S, int hq,
                          int hkv, int d, float scale, void* out_local, int out_dtype, unsigned flags) {
    using namespace sa;
    clear_error();
    SA_CHECK_ARG(sp != nullptr, "sa_spp_prefill: sp is NULL");
    SA_CHECK_ARG(sp->connected, "sa_spp_prefill: rank %d of %d is not connected (sa_spp_connect)", sp->rank,
                 sp->world);
    SA_CHECK_ARG(q_local && k_local && v_local && out_local, "sa_spp_prefill: null pointer");
    SA_CHECK_ARG(!(flags & SA_HOST_PTRS), "sa_spp_prefill: host pointers are not supported (pass device memory)");
    SA_CHECK_ARG(d == spp::D && hkv == sp->hkv && hkv <= 8 && hq >= hkv && hq % hkv == 0 && hq <= 256,
                 "sa_spp_prefill: d = %d, hq = %d, hkv = %d (created for hkv = %d, d = 128)", d, hq, hkv, sp->hkv);
    const int P = sp->world;
    SA_CHECK_ARG(S >= 2 * P && S % (2 * P) == 0 && S <= sp->max_seq,
                 "sa_spp_prefill: S = %d must be a multiple of 2 x %d ranks, at most max_seq = %d", S, P, sp->max_seq);
    SA_CHECK_ARG(out_dtype == SA_F32 || out_dtype == SA_BF16, "sa_spp_prefill: out_dtype %d", out_dtype);
    SA_CHECK_ARG(((((uintptr_t)q_local) | ((uintptr_t)k_local) | ((uintptr_t)v_local) | ((uintptr_t)out_local)) & 15) == 0,
                 "sa_spp_prefill: pointers must be 16-byte aligned");
    DeviceGuard guard(sp->device);
    cudaStream_t st = sp->ctx->stream;
    const int C = S / (2 * P);
    const int chunk[2] = {sp->rank, 2 * P - 1 - sp->rank};

    // the pieces (sa_spp_plan.h): per chunk, unmasked key blocks before it,
    // then its diagonal block
    spp::PieceSpec spec[kPrefillMaxPieces];
    PrefillPiece pcs[kPrefillMaxPieces];
    int first[2], count[2];
    const int n = spp::plan_pieces(sp->rank, P, C, spp::MIN_PIECE_KEYS, spp::MAX_CHUNK_PIECES, spec,
                                   kPrefillMaxPieces, first, count);
    SA_CHECK_ARG(n >= 1, "sa_spp_prefill: S = %d over %d ranks needs too many key blocks", S, P);
    for (int i = 0; i < n; ++i) {
        pcs[i].q_row0 = spec[i].q_row0;
        pcs[i].kv_row0 = spec[i].kv_row0;
        pcs[i].Sq = C;
        pcs[i].Skv = spec[i].Skv;
        pcs[i].q_pos0 = spec[i].q_pos0;
    }
    SA_CHECK_ARG(n <= kPrefillMaxPieces, "sa_spp_prefill: %d pieces", n);
    const long long piece_elems = (long long)C * hq * spp::D;
    // bf16 piece outputs (half floats each) and fp32 lse, in floats
    const size_t need = (size_t)n * (piece_elems / 2 + (size_t)C * hq) + 64;
    if (need > sp->part_floats) {
        SA_CUDA_TRY(cudaStreamSynchronize(st));
        cudaFree(sp->part);
        sp->part = nullptr;
        sp->part_floats = 0;
        if (cudaMalloc(&sp->part, need * sizeof(float)) != cudaSuccess) {
            cudaGetLastError();
            return set_error(SA_ERR_OOM, "sa_spp_prefill: %zu bytes of piece outputs", need * sizeof(float));
        }
        sp->part_floats = need;
    }
    __nv_bfloat16* parts = reinterpret_cast<__nv_bfloat16*>(sp->part);
    float* lse = sp->part + (size_t)n * piece_elems / 2;
    for (int i = 0; i < n; ++i) {
        pcs[i].out = parts + (size_t)i * piece_elems;
        pcs[i].lse = lse + (size_t)i * C * hq;
    }

    spp::ScatterArgs sa_{};
    sa_.k = static_cast<const uint4*>(k_local);
    sa_.v = static_cast<const uint4*>(v_local);
    for (int r = 0; r < P; ++r) sa_.dst[r] = sp->peer[r];
    sa_.world = P;
    sa_.rank = sp->rank;
    sa_.C = C;
    sa_.row_vecs = hkv * spp::D * 2 / 16;
    sa_.chunk[0] = chunk[0];
    sa_.chunk[1] = chunk[1];
    sa_.slot_bytes = sp->slot_bytes;
    sa_.tensor_bytes = sp->slot_bytes / 2;
    sa_.inst = sp->inst;
    sa_.cnt = sp->ctl;
    spp::spp_scatter_kernel<<<2 * sp->ctx->num_sms, 512, 0, st>>>(sa_);
    SA_CUDA_TRY(cudaGetLastError());
    spp::spp_wait_kernel<<<1, 32, 0, st>>>(reinterpret_cast<const unsigned*>(sp->buf), P, sp->inst,
                                           sp->ctx->status);
    // the instance is spent once its exchange is issued, whatever follows, so
    // the ranks' slots and epochs stay in step
    const unsigned inst = sp->inst++;
    SA_CUDA_TRY(cudaGetLastError());
    const unsigned char* kv = sp->buf + spp::FLAG_BYTES + (size_t)(inst & 1u) * sp->slot_bytes;
    const long long tok = (long long)hkv * spp::D;
    SA_RC_TRY(prefill_pieces_launch(st, sp->ctx->status, q_local, 2 * C, (long long)hq * spp::D, kv,
                                    kv + sp->slot_bytes / 2, S, tok, hq, hkv, scale, SA_BF16, (long long)hq * spp::D,
                                    pcs, n));
    spp::MergeArgs ma{};
    ma.part = parts;
    ma.lse = lse;
    ma.piece_elems = piece_elems;
    ma.C = C;
    ma.hq = hq;
    ma.first[0] = first[0]; ma.first[1] = first[1];
    ma.count[0] = count[0]; ma.count[1] = count[1];
    ma.out = out_local;
    ma.out_bf16 = out_dtype == SA_BF16;
    ma.status = sp->ctx->status;
    const long long threads = 16LL * 2 * C * hq;
    spp::spp_merge_kernel<<<(unsigned)((threads + 511) / 512), 512, 0, st>>>(ma);
    SA_CUDA_TRY(cudaGetLastError());
    return SA_OK;
}
