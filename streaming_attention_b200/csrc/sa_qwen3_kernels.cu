// sa_qwen3_kernels.cu -- the Qwen3 layer kernels other than the tensor-core
// GEMM and the attention: embedding, RMSNorm, QK-norm + RoPE + KV-cache
// append, the decode GEMVs with fused prologue/epilogues, and argmax.
//
// Numerics follow the reference's fp32 arithmetic (tensor_cpp/src/ops.cpp,
// qwen3_ops.cpp): fp32 activations and residual stream, weights in bf16
// (exact for bf16-representable weights), RMSNorm eps inside the sqrt,
// rotate-half RoPE with the reference's fp32 inverse-frequency table.
#include <cuda_bf16.h>
#include <cmath>

#include "sa_internal.h"
#include "sa_ptx.cuh"
#include "sa_qwen3.h"
#include "sa_qwen3_dev.cuh"
#include <algorithm>

namespace sa {
namespace qk {

constexpr int QK_MAX_PLANES = 8;   // split-K planes a consumer adds (the GEMM's largest split)

using qd::warp_sum;
using qd::head_norm_rope;

// Block-wide sum for blockDim.x <= 1024; `red` holds 32 floats.
__device__ __forceinline__ float block_sum(float v, float* red) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    v = warp_sum(v);
    __syncthreads();
    if (lane == 0) red[w] = v;
    __syncthreads();
    float t = (threadIdx.x < (blockDim.x + 31) / 32) ? red[threadIdx.x] : 0.f;
    if (w == 0) t = warp_sum(t);
    if (threadIdx.x == 0) red[0] = t;
    __syncthreads();
    return red[0];
}

// ---- embedding (ops.cpp:278-309): x[m, :] = E[id_m, :] ---------------------
__global__ void embedding_kernel(const int64_t* ids, int M, const __nv_bfloat16* E, int V, int H, float* x,
                                 int* status) {
    pdl_trigger();
    pdl_wait();
    const int m = blockIdx.x;
    const int64_t id = ids[m];
    const bool ok = id >= 0 && id < V;
    if (!ok && threadIdx.x == 0) atomicExch(status, SA_STATUS_BAD_INDEX);
    for (int i = threadIdx.x; i < H; i += blockDim.x)
        x[(size_t)m * H + i] = ok ? __bfloat162float(E[(size_t)id * H + i]) : 0.f;
}

// ---- RMSNorm (ops.cpp:375-418) to the two bf16 GEMM operand terms ---------
// With splits > 0, x first gets the `splits` partial planes of the previous
// GEMM added (plane order; row m of plane z at part + z * plane + m * H) and
// is written back: the residual add of a split o_proj / down_proj.
constexpr int RN_THREADS = 256, RN_MAX4 = 4;   // rows of up to 4096 floats, one register float4 per 256
__global__ void __launch_bounds__(RN_THREADS)
rmsnorm_hilo_kernel(float* x, const float* part, int splits, size_t plane, const float* w, int H, float eps,
                    __nv_bfloat16* hi, __nv_bfloat16* lo) {
    __shared__ float red[32];
    const int m = blockIdx.x, t = threadIdx.x, n4 = H / 4;
    // launched programmatically: the next kernel (a GEMM) may start streaming
    // its weights now; the gains do not depend on the previous kernel, x does
    pdl_trigger();
    float4 wv[RN_MAX4], v[RN_MAX4];
#pragma unroll
    for (int k = 0; k < RN_MAX4; ++k)
        if (t + k * RN_THREADS < n4) wv[k] = __ldg(reinterpret_cast<const float4*>(w) + t + k * RN_THREADS);
    pdl_wait();
    float4* xr = reinterpret_cast<float4*>(x + (size_t)m * H);
    const float* pr = part ? part + (size_t)m * H : nullptr;
    float ss = 0.f;
#pragma unroll
    for (int k = 0; k < RN_MAX4; ++k) {
        const int i4 = t + k * RN_THREADS;
        if (i4 >= n4) break;
        // every plane's load issued before any is added
        float4 pv[QK_MAX_PLANES];
#pragma unroll
        for (int z = 0; z < QK_MAX_PLANES; ++z)
            if (z < splits) pv[z] = __ldcg(reinterpret_cast<const float4*>(pr + z * plane) + i4);
        float4 a = xr[i4];
#pragma unroll
        for (int z = 0; z < QK_MAX_PLANES; ++z)
            if (z < splits) { a.x += pv[z].x; a.y += pv[z].y; a.z += pv[z].z; a.w += pv[z].w; }
        if (splits > 0) xr[i4] = a;
        v[k] = a;
        ss += a.x * a.x + a.y * a.y + a.z * a.z + a.w * a.w;
    }
    ss = block_sum(ss, red);
    const float rms = sqrtf(ss / (float)H + eps);
#pragma unroll
    for (int k = 0; k < RN_MAX4; ++k) {
        const int i4 = t + k * RN_THREADS;
        if (i4 >= n4) break;
        const float y[4] = {(v[k].x / rms) * wv[k].x, (v[k].y / rms) * wv[k].y, (v[k].z / rms) * wv[k].z,
                            (v[k].w / rms) * wv[k].w};
        __nv_bfloat162 h2[2], l2[2];
#pragma unroll
        for (int q = 0; q < 2; ++q) {
            h2[q] = __floats2bfloat162_rn(y[2 * q], y[2 * q + 1]);
            const float2 f = __bfloat1622float2(h2[q]);
            l2[q] = __floats2bfloat162_rn(y[2 * q] - f.x, y[2 * q + 1] - f.y);
        }
        *reinterpret_cast<uint2*>(hi + (size_t)m * H + 4 * i4) =
            make_uint2(*reinterpret_cast<uint32_t*>(&h2[0]), *reinterpret_cast<uint32_t*>(&h2[1]));
        *reinterpret_cast<uint2*>(lo + (size_t)m * H + 4 * i4) =
            make_uint2(*reinterpret_cast<uint32_t*>(&l2[0]), *reinterpret_cast<uint32_t*>(&l2[1]));
    }
}


// fp32 -> (hi, lo) bf16 split of an activation for the tensor-core GEMM.
// x += the sum, in plane order, of `splits` partial planes (a split GEMM's
// residual add when no RMSNorm follows).
__global__ void resid_add_kernel(float* x, const float* part, int splits, size_t n4) {
    pdl_trigger();
    pdl_wait();
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n4; i += (size_t)gridDim.x * blockDim.x) {
        float4 pv[QK_MAX_PLANES];
#pragma unroll
        for (int z = 0; z < QK_MAX_PLANES; ++z)
            if (z < splits) pv[z] = __ldcg(reinterpret_cast<const float4*>(part) + z * n4 + i);
        float4 v = reinterpret_cast<float4*>(x)[i];
#pragma unroll
        for (int z = 0; z < QK_MAX_PLANES; ++z)
            if (z < splits) { v.x += pv[z].x; v.y += pv[z].y; v.z += pv[z].z; v.w += pv[z].w; }
        reinterpret_cast<float4*>(x)[i] = v;
    }
}

// SwiGLU of a split gate/up GEMM (qwen3_mlp, qwen3_ops.cpp:265-296): the
// planes hold [M, 2I] partial sums in [gate(32); up(32)] column blocks;
// out[m, i] = silu(g) * u with g, u the plane sums (plane order) of columns
// 64 (i / 32) + i % 32 and that + 32, written as bf16 hi / lo terms.
__global__ void swiglu_hilo_kernel(const float* part, int splits, int M, int I, __nv_bfloat16* hi,
                                   __nv_bfloat16* lo, long long ldo) {
    pdl_trigger();
    pdl_wait();
    const size_t plane = (size_t)M * 2 * I;
    const size_t n4 = (size_t)M * I / 4;
    for (size_t e = blockIdx.x * (size_t)blockDim.x + threadIdx.x; e < n4; e += (size_t)gridDim.x * blockDim.x) {
        const int m = (int)(e / (I / 4)), i = (int)(e % (I / 4)) * 4;
        const size_t gc = (size_t)m * 2 * I + (i / 32) * 64 + (i % 32);
        float4 pg[QK_MAX_PLANES], pu[QK_MAX_PLANES];
#pragma unroll
        for (int z = 0; z < QK_MAX_PLANES; ++z)
            if (z < splits) {
                pg[z] = __ldcg(reinterpret_cast<const float4*>(part + z * plane + gc));
                pu[z] = __ldcg(reinterpret_cast<const float4*>(part + z * plane + gc + 32));
            }
        float4 g = pg[0], u = pu[0];
#pragma unroll
        for (int z = 1; z < QK_MAX_PLANES; ++z)
            if (z < splits) {
                g.x += pg[z].x; g.y += pg[z].y; g.z += pg[z].z; g.w += pg[z].w;
                u.x += pu[z].x; u.y += pu[z].y; u.z += pu[z].z; u.w += pu[z].w;
            }
        const float v[4] = {(g.x / (1.f + expf(-g.x))) * u.x, (g.y / (1.f + expf(-g.y))) * u.y,
                            (g.z / (1.f + expf(-g.z))) * u.z, (g.w / (1.f + expf(-g.w))) * u.w};
        __nv_bfloat16* ho = hi + (size_t)m * ldo + i;
        __nv_bfloat16* lw = lo + (size_t)m * ldo + i;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const __nv_bfloat16 h = __float2bfloat16_rn(v[k]);
            ho[k] = h;
            lw[k] = __float2bfloat16_rn(v[k] - __bfloat162float(h));
        }
    }
}


// ---- RoPE tables (qwen3_ops.cpp:70-104): cos/sin[pos, i], i < D/2 ----------
__global__ void rope_table_kernel(int n_pos, int D, float theta, float* cos_t, float* sin_t) {
    const int half = D / 2;
    const size_t n = (size_t)n_pos * half;
    for (size_t idx = blockIdx.x * (size_t)blockDim.x + threadIdx.x; idx < n; idx += (size_t)gridDim.x * blockDim.x) {
        const int p = (int)(idx / half), i = (int)(idx % half);
        const float inv = 1.0f / powf(theta, (float)i / (float)D);
        const float ang = (float)p * inv;
        cos_t[idx] = cosf(ang);
        sin_t[idx] = sinf(ang);
    }
}

// ---- QK-norm + RoPE + cache append ----------------------------------------
// qkv [M, (hq + 2 hkv) * 128] fp32 from the QKV projection (rows = tokens).
// One warp per (token, head); lane l holds elements 4l..4l+3 of the head.
// Q heads: RMS over the head (eps 1e-6 inside the sqrt, qwen3_ops.cpp:355-369)
// times q_norm, then rotate-half RoPE at position pos0 + m
// (qwen3_ops.cpp:110-188) -> q_out [M, hq, 128].  K heads: the same with
// k_norm -> K cache row pos0 + m.  V heads: copied to the V cache.
// qkv holds `splits` planes of `plane` floats (split-K partial sums of the
// QKV GEMM, added here in plane order) or the finished projection (splits 1).
__global__ void qknorm_rope_append_kernel(const float* qkv, int splits, size_t plane, int M, int hq, int hkv,
                                          const float* qn, const float* kn, const float* cos_t, const float* sin_t,
                                          int pos0, const int* pos_dev, int row_shift, float* q_out, float* kc,
                                          float* vc, int max_seq) {
    constexpr int D = 128;
    pdl_trigger();
    pdl_wait();
    const int lane = threadIdx.x & 31;
    const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int nh = hq + 2 * hkv;
    if (gw >= M * nh) return;
    const int m = gw / nh, h = gw % nh;
    const int pos = (pos_dev ? *pos_dev : pos0) + m;      // RoPE position
    const int row = pos + row_shift;                       // cache row written
    if (row >= max_seq) return;       // the host checks capacity; never write past the cache
    const float* src = qkv + (size_t)m * nh * D + (size_t)h * D;
    // produced by the previous kernel; every plane's load is issued before
    // any is added (an in-order add would wait on each load in turn)
    float4 pv[QK_MAX_PLANES];
#pragma unroll
    for (int z = 0; z < QK_MAX_PLANES; ++z)
        if (z < splits) pv[z] = __ldcg(reinterpret_cast<const float4*>(src + z * plane + 4 * lane));
    float4 v4 = pv[0];
#pragma unroll
    for (int z = 1; z < QK_MAX_PLANES; ++z)
        if (z < splits) { v4.x += pv[z].x; v4.y += pv[z].y; v4.z += pv[z].z; v4.w += pv[z].w; }
    float e[4] = {v4.x, v4.y, v4.z, v4.w};
    if (h >= hq + hkv) {  // V head
        float* dst = vc + ((size_t)(h - hq - hkv) * max_seq + row) * D;
        *reinterpret_cast<float4*>(dst + 4 * lane) = v4;
        return;
    }
    const float4 r4 = head_norm_rope(e, h < hq ? qn : kn, cos_t + (size_t)pos * (D / 2),
                                     sin_t + (size_t)pos * (D / 2), lane);
    if (h < hq) {
        *reinterpret_cast<float4*>(q_out + ((size_t)m * hq + h) * D + 4 * lane) = r4;
    } else {
        float* dst = kc + ((size_t)(h - hq) * max_seq + row) * D;
        *reinterpret_cast<float4*>(dst + 4 * lane) = r4;
    }
}


// ---- decode GEMV v2: one 16-byte chunk column per thread, R rows per CTA ----
// blockDim = K/8: thread t owns K-chunk t (8 bf16) of each of the CTA's R
// rows and the matching 8 activations, so all R weight loads of a thread are
// in flight at once and every weight byte is read exactly once.  NORM folds
// RMSNorm in as a scalar: dot(W, (x / rms) * g) = (1/rms) * dot(W, x * g),
// with sum(x^2) reduced from the same activation loads.  SWIGLU: the CTA's
// rows are (gate, up) pairs of R/2 outputs ([gate 32; up 32] row blocks).
// ARGMAX additionally folds the CTA's maxima into *amax as a 64-bit key
// (ordered value << 32 | ~index): the largest value, first index on ties.
__device__ __forceinline__ uint32_t ordered_f32(float f) {
    const uint32_t u = __float_as_uint(f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// ---- head-parallel exchange primitives --------------------------------------
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Slot and epoch of this launch's exchange instance (read after pdl_wait:
// the sequence word is advanced by an earlier kernel of the stream).
__device__ __forceinline__ void tp_instance(const TpArgs& t, int& slot, unsigned& epoch) {
    const unsigned i = __ldcg(t.seq) + (unsigned)t.k;
    slot = (int)(i & 1u);
    epoch = i + 1u;
}

// Wait until source `src` has published `epoch` into this rank's flag of
// `slot`.  Bounded: after the limit (or when an earlier wait already failed)
// the status word is set and the caller continues with whatever is there.
__device__ __forceinline__ void tp_wait(const TpArgs& t, int slot, unsigned epoch, int src) {
    const unsigned* f = t.flags[t.rank] + slot * t.world + src;
    if ((int)(ld_acquire_sys(f) - epoch) >= 0) return;
    if (*reinterpret_cast<volatile int*>(t.status) != 0) return;
    const unsigned long long t0 = globaltimer();
    while ((int)(ld_acquire_sys(f) - epoch) < 0) {
        if (globaltimer() - t0 > kWaitLimitNs) {
            atomicExch(t.status, SA_STATUS_TIMEOUT);
            return;
        }
    }
}

__device__ __forceinline__ void st_word_sys(unsigned long long* p, unsigned long long v) {
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_word_sys(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ unsigned long long ll_word(unsigned epoch, uint32_t bits) {
    return ((unsigned long long)epoch << 32) | bits;
}
__device__ __forceinline__ ulonglong2 ld_words2_sys(const unsigned long long* p) {
    ulonglong2 v;
    asm volatile("ld.volatile.global.v2.u64 {%0, %1}, [%2];" : "=l"(v.x), "=l"(v.y) : "l"(p) : "memory");
    return v;
}
// Word area [slot][src] of rank `dst`.
__device__ __forceinline__ unsigned long long* tp_words(const TpArgs& t, int dst, int slot, int src) {
    return t.ll[dst] + ((long long)slot * t.world + src) * t.ll_stride;
}
// Wait for a self-validating word of `epoch` (bounded as tp_wait) and return its value bits.
__device__ __forceinline__ uint32_t ll_wait(const TpArgs& t, const unsigned long long* p, unsigned epoch) {
    unsigned long long w = ld_word_sys(p);
    if ((unsigned)(w >> 32) == epoch) return (uint32_t)w;
    if (*reinterpret_cast<volatile int*>(t.status) != 0) return (uint32_t)w;
    const unsigned long long t0 = globaltimer();
    while ((unsigned)((w = ld_word_sys(p)) >> 32) != epoch) {
        if (globaltimer() - t0 > kWaitLimitNs) {
            atomicExch(t.status, SA_STATUS_TIMEOUT);
            break;
        }
    }
    return (uint32_t)w;
}

// Receive block [slot][src] of rank `dst`.
__device__ __forceinline__ float* tp_block(const TpArgs& t, int dst, int slot, int src) {
    return t.recv[dst] + ((long long)slot * t.world + src) * t.slot_floats;
}

// Called by one warp of every CTA of a producing grid after its stores to
// the receive blocks: the last CTA to arrive publishes the instance on every
// rank (lane r sets this rank's flag on rank r) and re-arms the counter.
__device__ __forceinline__ void tp_arrive_publish(const TpArgs& t, int slot, unsigned epoch, int lane) {
    __threadfence_system();
    __syncwarp();
    unsigned last = 0;
    if (lane == 0) last = atomicAdd(t.cnt, 1u) == gridDim.x - 1;
    last = __shfl_sync(0xffffffffu, last, 0);
    if (!last) return;
    __threadfence_system();
    if (lane < t.world) st_release_sys(t.flags[lane] + slot * t.world + t.rank, epoch);
    if (lane == 0) *t.cnt = 0u;
}

// Activations (x, and y in RESID mode) come from the previous kernel, which may
// still be draining when this one starts (programmatic launch): they are read
// through L2 (ld.global.cg) after pdl_wait, never through the read-only path.
// blockDim = K/8 rounded up to whole warps; threads past K/8 contribute zero.
//
// QW_EPI_QKV (the decode step's fused QKV projection): rows are the
// [q heads; k heads; v heads] x 128 outputs, R rows per CTA, so 128 / R CTAs
// make one head.  V outputs go straight to the V cache row.  Q and K outputs
// go to y; the last CTA of a head to arrive (per-head counter) reads the
// head back, applies QK-norm and RoPE (as qknorm_rope_append_kernel) and
// writes the query (e.q_out) or the K cache row, then re-arms the counter.
//
// Head-parallel ranks: QW_EPI_XCHG sends the outputs (this rank's partial
// sums of o_proj / down_proj) as self-validating words to word area
// [slot][rank] of every rank: no fence, counter or flag.  CONSUME adds the
// exchanged sums of the previous instance to the residual before anything
// else: x + the sum over ranks r, in rank order, of word area [slot][r]
// (tp.use_ll; each thread waits for its own 8 words per rank) or of block
// [slot][r] row tp.row after the flags (after a prompt-path exchange); CTA 0
// stores the result at tp.x_out (the other CTAs still read x).
template <int MODE, bool NORM, int R, bool ARGMAX, bool CONSUME>
__global__ void gemv2_kernel(const __nv_bfloat16* __restrict__ W, int N_out, int K,
                             const float* x, const float* __restrict__ nw, float eps,
                             float* y, unsigned long long* amax, const QkvEpi e, const TpArgs tp) {
    constexpr int NV = R + 1;                      // R dot products + sum of squares
    __shared__ float red[32][NV];
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5, nwarp = blockDim.x >> 5;
    const bool act = t < K / 8;                    // thread owns a K-chunk
    const int OUT_PER_CTA = MODE == QW_EPI_SWIGLU ? R / 2 : R;
    const int o0 = blockIdx.x * OUT_PER_CTA;
    // rows of this CTA
    int rows[R];
#pragma unroll
    for (int r = 0; r < R; ++r) {
        if (MODE == QW_EPI_SWIGLU) {
            const int n = min(o0 + r / 2, N_out - 1);
            const int g = (n / 32) * 64 + (n % 32);
            rows[r] = (r & 1) ? g + 32 : g;
        } else {
            rows[r] = min(o0 + r, N_out - 1);
        }
    }
    static_assert(MODE != QW_EPI_QKV || (128 % R == 0 && !ARGMAX), "QKV epilogue: whole heads of R rows");
    pdl_trigger();
    uint4 w[R];
#pragma unroll
    for (int r = 0; r < R; ++r)
        w[r] = act ? __ldg(reinterpret_cast<const uint4*>(W + (size_t)rows[r] * K) + t) : make_uint4(0, 0, 0, 0);
    // weights do not depend on the previous kernel; the activations do
    pdl_wait();
    int q_pos = 0, q_row = 0;      // QKV epilogue: RoPE position and cache row
    if (MODE == QW_EPI_QKV) {
        q_pos = e.pos_dev ? __ldcg(e.pos_dev) : e.pos0;
        q_row = q_pos + e.row_shift;
    }
    float xv[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (act) {
        const float4 xa = __ldcg(reinterpret_cast<const float4*>(x) + 2 * t);
        const float4 xb = __ldcg(reinterpret_cast<const float4*>(x) + 2 * t + 1);
        xv[0] = xa.x; xv[1] = xa.y; xv[2] = xa.z; xv[3] = xa.w;
        xv[4] = xb.x; xv[5] = xb.y; xv[6] = xb.z; xv[7] = xb.w;
    }
    if (CONSUME) {
        __shared__ int s_slot;
        __shared__ unsigned s_epoch;
        if (t == 0) {
            int slot;
            unsigned epoch;
            tp_instance(tp, slot, epoch);
            s_slot = slot;
            s_epoch = epoch;
            if (!tp.use_ll)
                for (int r = 0; r < tp.world; ++r) tp_wait(tp, slot, epoch, r);
        }
        __syncthreads();
        if (act && tp.use_ll) {
            // this thread's 8 words from each source, loaded two sources at a
            // time before any is checked (one round trip per pair when the
            // words are there); words that are not yet there are waited for
            float sum[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
            for (int r0 = 0; r0 < tp.world; r0 += 2) {
                ulonglong2 wv[2][4];
#pragma unroll
                for (int g = 0; g < 2; ++g)
                    if (r0 + g < tp.world) {
                        const unsigned long long* wd = tp_words(tp, tp.rank, s_slot, r0 + g) + 8 * t;
#pragma unroll
                        for (int i = 0; i < 4; ++i) wv[g][i] = ld_words2_sys(wd + 2 * i);
                    }
#pragma unroll
                for (int g = 0; g < 2; ++g)
                    if (r0 + g < tp.world) {
                        const unsigned long long* wd = tp_words(tp, tp.rank, s_slot, r0 + g) + 8 * t;
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            unsigned long long a = wv[g][i].x, b = wv[g][i].y;
                            if ((unsigned)(a >> 32) != s_epoch) a = ll_wait(tp, wd + 2 * i, s_epoch);
                            if ((unsigned)(b >> 32) != s_epoch) b = ll_wait(tp, wd + 2 * i + 1, s_epoch);
                            const float va = __uint_as_float((uint32_t)a), vb = __uint_as_float((uint32_t)b);
                            sum[2 * i] = r0 + g == 0 ? va : sum[2 * i] + va;
                            sum[2 * i + 1] = r0 + g == 0 ? vb : sum[2 * i + 1] + vb;
                        }
                    }
            }
#pragma unroll
            for (int i = 0; i < 8; ++i) xv[i] += sum[i];
            if (blockIdx.x == 0) {
                reinterpret_cast<float4*>(tp.x_out)[2 * t] = make_float4(xv[0], xv[1], xv[2], xv[3]);
                reinterpret_cast<float4*>(tp.x_out)[2 * t + 1] = make_float4(xv[4], xv[5], xv[6], xv[7]);
            }
        } else if (act) {
            float sum[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
            for (int r = 0; r < tp.world; ++r) {
                float pv[8];
                {
                    const float* b = tp_block(tp, tp.rank, s_slot, r) + (size_t)tp.row * K;
                    const float4 pa = __ldcg(reinterpret_cast<const float4*>(b) + 2 * t);
                    const float4 pb = __ldcg(reinterpret_cast<const float4*>(b) + 2 * t + 1);
                    pv[0] = pa.x; pv[1] = pa.y; pv[2] = pa.z; pv[3] = pa.w;
                    pv[4] = pb.x; pv[5] = pb.y; pv[6] = pb.z; pv[7] = pb.w;
                }
#pragma unroll
                for (int i = 0; i < 8; ++i) sum[i] = r == 0 ? pv[i] : sum[i] + pv[i];
            }
#pragma unroll
            for (int i = 0; i < 8; ++i) xv[i] += sum[i];
            if (blockIdx.x == 0) {
                reinterpret_cast<float4*>(tp.x_out)[2 * t] = make_float4(xv[0], xv[1], xv[2], xv[3]);
                reinterpret_cast<float4*>(tp.x_out)[2 * t + 1] = make_float4(xv[4], xv[5], xv[6], xv[7]);
            }
        }
    }
    float v[NV];
    v[R] = 0.f;
    if (NORM) {
#pragma unroll
        for (int i = 0; i < 8; ++i) v[R] = fmaf(xv[i], xv[i], v[R]);
        if (act) {
            const float4 ga = __ldg(reinterpret_cast<const float4*>(nw) + 2 * t);
            const float4 gb = __ldg(reinterpret_cast<const float4*>(nw) + 2 * t + 1);
            const float gv[8] = {ga.x, ga.y, ga.z, ga.w, gb.x, gb.y, gb.z, gb.w};
#pragma unroll
            for (int i = 0; i < 8; ++i) xv[i] *= gv[i];
        }
    }
#pragma unroll
    for (int r = 0; r < R; ++r) {
        const uint32_t wr[4] = {w[r].x, w[r].y, w[r].z, w[r].w};
        float acc = 0.f;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            acc = fmaf(__uint_as_float(wr[j] << 16), xv[2 * j], acc);
            acc = fmaf(__uint_as_float(wr[j] & 0xffff0000u), xv[2 * j + 1], acc);
        }
        v[r] = acc;
    }
#pragma unroll
    for (int i = 0; i < NV; ++i) v[i] = warp_sum(v[i]);
    if (lane == 0)
#pragma unroll
        for (int i = 0; i < NV; ++i) red[warp][i] = v[i];
    __syncthreads();
    if (warp == 0) {
#pragma unroll
        for (int i = 0; i < NV; ++i) {
            float a = lane < nwarp ? red[lane][i] : 0.f;
            a = warp_sum(a);
            v[i] = a;
        }
        float scale = 1.f;
        if (NORM) scale = 1.f / sqrtf(v[R] / (float)K + eps);
        int x_slot = 0;
        unsigned x_epoch = 0;
        if (MODE == QW_EPI_XCHG) tp_instance(tp, x_slot, x_epoch);
        unsigned long long best = 0ull;
        if (lane < OUT_PER_CTA) {
            const int n = o0 + lane;
            float out = 0.f;
#pragma unroll
            for (int r = 0; r < OUT_PER_CTA; ++r) {
                if (r == lane) {
                    if (MODE == QW_EPI_SWIGLU) {
                        const float g = v[2 * r] * scale, u = v[2 * r + 1] * scale;
                        out = (g / (1.f + expf(-g))) * u;
                    } else {
                        out = v[r] * scale;
                    }
                }
            }
            if (MODE == QW_EPI_QKV) {
                if (n < N_out) {
                    const int h = n / 128, vh = h - e.hq - e.hkv;
                    if (vh >= 0) {
                        if (q_row < e.max_seq) e.vc[((size_t)vh * e.max_seq + q_row) * 128 + n % 128] = out;
                    } else {
                        y[n] = out;
                    }
                }
            } else if (MODE == QW_EPI_XCHG) {
                // one self-validating word per output to every rank
                if (n < N_out)
                    for (int r = 0; r < tp.world; ++r)
                        st_word_sys(tp_words(tp, r, x_slot, tp.rank) + n, ll_word(x_epoch, __float_as_uint(out)));
            } else if (n < N_out) {
                if (MODE == QW_EPI_RESID) y[n] = __ldcg(y + n) + out;
                else y[n] = out;
                if (ARGMAX)
                    best = ((unsigned long long)ordered_f32(out) << 32) |
                           (unsigned long long)(0xffffffffu - (uint32_t)(n + tp.n_base));
            }
        }
        if (ARGMAX) {
#pragma unroll
            for (int off = 16; off; off >>= 1) {
                const unsigned long long o = __shfl_xor_sync(0xffffffffu, best, off);
                best = o > best ? o : best;
            }
            if (lane == 0) atomicMax(amax, best);
        }
        if (MODE == QW_EPI_QKV) {
            const int h = o0 / 128;
            if (h < e.hq + e.hkv) {
                // publish this CTA's outputs, then count it in
                __threadfence();
                __syncwarp();
                unsigned last = 0;
                if (lane == 0) last = atomicAdd(e.cnt + h, 1u) == (unsigned)(128 / R - 1);
                last = __shfl_sync(0xffffffffu, last, 0);
                if (last && q_row < e.max_seq) {
                    __threadfence();
                    const float4 v4 = __ldcg(reinterpret_cast<const float4*>(y + (size_t)h * 128) + lane);
                    const float ev[4] = {v4.x, v4.y, v4.z, v4.w};
                    const float* cr = e.cos_t + (size_t)q_pos * 64;
                    const float* sr = e.sin_t + (size_t)q_pos * 64;
                    const float4 r4 = head_norm_rope(ev, h < e.hq ? e.qn : e.kn, cr, sr, lane);
                    float* dst = h < e.hq ? e.q_out + (size_t)h * 128
                                          : e.kc + ((size_t)(h - e.hq) * e.max_seq + q_row) * 128;
                    reinterpret_cast<float4*>(dst)[lane] = r4;
                }
                if (last && lane == 0) e.cnt[h] = 0u;
            }
        }
    }
}

// ---- head-parallel: prompt-path exchange ------------------------------------
// Producer: rows [0, M) x H of `part` (this rank's o_proj / down_proj partial
// sums from the tensor-core GEMM) go to block [slot][rank] of every rank.
__global__ void tp_scatter_kernel(const float* part, size_t n4, const TpArgs tp) {
    pdl_trigger();
    pdl_wait();
    int slot;
    unsigned epoch;
    tp_instance(tp, slot, epoch);
    const float4* src = reinterpret_cast<const float4*>(part);
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n4; i += (size_t)gridDim.x * blockDim.x) {
        const float4 v = __ldcg(src + i);
        for (int r = 0; r < tp.world; ++r) reinterpret_cast<float4*>(tp_block(tp, r, slot, tp.rank))[i] = v;
    }
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x < 32) tp_arrive_publish(tp, slot, epoch, threadIdx.x);
}

// Consumer: x[m] += sum over ranks of block row (tp.row + m), then RMSNorm of
// the row split into bf16 hi/lo terms (as rmsnorm_hilo_kernel).  One CTA per
// row; each updates only its own row of x.
__global__ void rmsnorm_hilo_tp_kernel(float* x, const float* w, int H, float eps, __nv_bfloat16* hi,
                                       __nv_bfloat16* lo, const TpArgs tp) {
    __shared__ float red[32];
    __shared__ int s_slot;
    pdl_trigger();
    pdl_wait();
    const int m = blockIdx.x;
    if (threadIdx.x == 0) {
        int slot;
        unsigned epoch;
        tp_instance(tp, slot, epoch);
        s_slot = slot;
        for (int r = 0; r < tp.world; ++r) tp_wait(tp, slot, epoch, r);
    }
    __syncthreads();
    float* xr = x + (size_t)m * H;
    float ss = 0.f;
    for (int i = threadIdx.x; i < H; i += blockDim.x) {
        float sum = 0.f;
        for (int r = 0; r < tp.world; ++r) {
            const float p = __ldcg(tp_block(tp, tp.rank, s_slot, r) + (size_t)(tp.row + m) * H + i);
            sum = r == 0 ? p : sum + p;
        }
        const float v = xr[i] + sum;
        xr[i] = v;
        ss += v * v;
    }
    ss = block_sum(ss, red);
    const float rms = sqrtf(ss / (float)H + eps);
    for (int i = threadIdx.x; i < H; i += blockDim.x) {
        const float y = (xr[i] / rms) * w[i];
        const __nv_bfloat16 h = __float2bfloat16_rn(y);
        hi[(size_t)m * H + i] = h;
        lo[(size_t)m * H + i] = __float2bfloat16_rn(y - __bfloat162float(h));
    }
}

// Greedy token across the ranks' vocabulary slices: every rank sends its
// argmax key (largest value, first index; indices are global) to every rank
// as self-validating words,
// takes the maximum of the `world` keys and decodes it; then the segment's
// instance count is added to the sequence word.  One warp.
__global__ void tp_amax_token_kernel(unsigned long long* amax, int64_t* tok, const TpArgs tp, int seg) {
    pdl_trigger();
    pdl_wait();
    const int lane = threadIdx.x;
    int slot;
    unsigned epoch;
    tp_instance(tp, slot, epoch);
    const unsigned long long mine = __ldcg(amax);            // folded in by the lm_head GEMV
    if (lane < tp.world) {   // the key as two self-validating words (high, low half)
        unsigned long long* w = tp_words(tp, lane, slot, tp.rank);
        st_word_sys(w, ll_word(epoch, (uint32_t)(mine >> 32)));
        st_word_sys(w + 1, ll_word(epoch, (uint32_t)mine));
    }
    unsigned long long best = 0ull;
    if (lane < tp.world) {
        const unsigned long long* w = tp_words(tp, tp.rank, slot, lane);
        const uint32_t hi = ll_wait(tp, w, epoch), lo = ll_wait(tp, w + 1, epoch);
        best = ((unsigned long long)hi << 32) | lo;
    }
#pragma unroll
    for (int off = 16; off; off >>= 1) {
        const unsigned long long o = __shfl_xor_sync(0xffffffffu, best, off);
        best = o > best ? o : best;
    }
    if (lane == 0) {
        *tok = (int64_t)(0xffffffffu - (uint32_t)(best & 0xffffffffull));
        *amax = 0ull;
        *const_cast<unsigned*>(tp.seq) = __ldcg(tp.seq) + (unsigned)seg;
    }
}

// ---- sequence-parallel prompt: row exchange --------------------------------
// Blocks of rows this rank produced (one layer's K and V cache rows of its
// tokens; the final residual rows) are copied to the same place in every
// other rank's memory (CUDA IPC mappings), then the instance is published on
// every rank as in tp_scatter_kernel.
__global__ void sp_rows_scatter_kernel(const SpCopy c, const TpArgs tp) {
    pdl_trigger();
    pdl_wait();
    int slot;
    unsigned epoch;
    tp_instance(tp, slot, epoch);
    const long long per4 = c.blk_floats / 4;
    const long long n4 = (long long)c.nreg * c.nblk * per4;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n4; i += (long long)gridDim.x * blockDim.x) {
        const int reg = (int)(i / ((long long)c.nblk * per4));
        const long long rem = i - (long long)reg * c.nblk * per4;
        const long long b = rem / per4, e = rem - b * per4;
        const long long off = b * c.stride + e * 4;
        const float4 v = __ldcg(reinterpret_cast<const float4*>(c.src[reg] + off));
        for (int r = 0; r < tp.world; ++r)
            if (c.dst[reg][r])   // null: this rank's own copy, already in place
                *reinterpret_cast<float4*>(c.dst[reg][r] + (long long)slot * c.slot_floats + off) = v;
    }
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x < 32) tp_arrive_publish(tp, slot, epoch, threadIdx.x);
}

// ---- long prompts: operands of the tensor-core attention --------------------
__device__ __forceinline__ uint4 pack8_bf16(float4 a, float4 b) {
    uint4 r;
    __nv_bfloat162 t;
    t = __floats2bfloat162_rn(a.x, a.y); r.x = *reinterpret_cast<uint32_t*>(&t);
    t = __floats2bfloat162_rn(a.z, a.w); r.y = *reinterpret_cast<uint32_t*>(&t);
    t = __floats2bfloat162_rn(b.x, b.y); r.z = *reinterpret_cast<uint32_t*>(&t);
    t = __floats2bfloat162_rn(b.z, b.w); r.w = *reinterpret_cast<uint32_t*>(&t);
    return r;
}

// Groups of 8 values: [0, nq8) of q (same layout), then K and V rows t of
// head h (source row h * max_seq + t, destination row t * hkv + h).
__global__ void tc_pack_kernel(const float* __restrict__ q, long long nq8, const float* __restrict__ kc,
                               const float* __restrict__ vc, int max_seq, int hkv, int T, __nv_bfloat16* qb,
                               __nv_bfloat16* kb, __nv_bfloat16* vb) {
    pdl_trigger();
    pdl_wait();
    const long long nkv8 = (long long)T * hkv * 16;
    const long long n = nq8 + 2 * nkv8;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
        const float* src;
        __nv_bfloat16* dst;
        if (i < nq8) {
            src = q + i * 8;
            dst = qb + i * 8;
        } else {
            long long j = i - nq8;
            const bool is_v = j >= nkv8;
            if (is_v) j -= nkv8;
            const long long c = j & 15, th = j >> 4;          // 16 groups of 8 per 128-wide row
            const long long t = th / hkv, h = th - t * hkv;
            src = (is_v ? vc : kc) + ((size_t)h * max_seq + t) * 128 + c * 8;
            dst = (is_v ? vb : kb) + ((size_t)t * hkv + h) * 128 + c * 8;
        }
        const float4 a = __ldcg(reinterpret_cast<const float4*>(src));
        const float4 b = __ldcg(reinterpret_cast<const float4*>(src) + 1);
        *reinterpret_cast<uint4*>(dst) = pack8_bf16(a, b);
    }
}

// Wait (bounded) until every rank published this instance.
__global__ void sp_wait_kernel(const TpArgs tp) {
    pdl_trigger();
    pdl_wait();
    if ((int)threadIdx.x < tp.world) {
        int slot;
        unsigned epoch;
        tp_instance(tp, slot, epoch);
        tp_wait(tp, slot, epoch, threadIdx.x);
    }
}

__global__ void tp_seq_add_kernel(unsigned* seq, int n) {
    pdl_trigger();
    pdl_wait();
    *seq = __ldcg(seq) + (unsigned)n;
}

// Decode the argmax key into a token id and clear the key for the next step.
__global__ void amax_to_token_kernel(unsigned long long* amax, int64_t* tok) {
    pdl_trigger();
    pdl_wait();
    const unsigned long long k = __ldcg(amax);      // folded in by the previous kernel's atomics
    *tok = (int64_t)(0xffffffffu - (uint32_t)(k & 0xffffffffull));
    *amax = 0ull;
}


// Decode-loop bookkeeping after a token was chosen: record it and advance the
// step counter; with inc_len the token just processed is now in the cache.
// state[0] = cache length, state[1] = tokens recorded.
__global__ void advance_kernel(int* state, const int64_t* tok, int64_t* toks, int cap, int inc_len) {
    pdl_trigger();
    pdl_wait();
    volatile int* vs = state;                       // written by earlier steps
    const int s = vs[1];
    if (s < cap) toks[s] = __ldcg(reinterpret_cast<const long long*>(tok));
    vs[1] = s + 1;
    if (inc_len) vs[0] = vs[0] + 1;
}

}  // namespace qk

// ---- launchers --------------------------------------------------------------
int launch_advance(cudaStream_t st, int* state, const int64_t* tok, int64_t* toks, int cap, int inc_len,
                   bool after_kernel) {
    // programmatic launch only directly after another kernel: after a copy
    // (the decode state) the ordinary stream order is needed
    if (after_kernel)
        SA_CUDA_TRY(launch_pdl_k(3, qk::advance_kernel, dim3(1), dim3(1), 0, st, state, tok, toks, cap, inc_len));
    else
        qk::advance_kernel<<<1, 1, 0, st>>>(state, tok, toks, cap, inc_len);
    SA_CUDA_TRY(cudaGetLastError());
    return SA_OK;
}
int launch_embedding(cudaStream_t st, const int64_t* ids, int M, const __nv_bfloat16* E, int V, int H, float* x,
                     int* status) {
    // the first kernel of a forward follows the copy of the token ids, a
    // non-kernel stream operation, so it is launched the ordinary way
    qk::embedding_kernel<<<M, 256, 0, st>>>(ids, M, E, V, H, x, status);
    SA_CUDA_TRY(cudaGetLastError());
    SA_CUDA_TRY(cudaGetLastError());
    return SA_OK;
}
int launch_rmsnorm_hilo(cudaStream_t st, float* x, const float* w, int M, int H, float eps,
                        __nv_bfloat16* hi, __nv_bfloat16* lo, const float* part, int splits) {
    SA_CHECK_ARG(splits == 0 || (part && splits <= qk::QK_MAX_PLANES), "rmsnorm_hilo: partial planes");
    SA_CHECK_ARG(H % 4 == 0 && H <= 4 * qk::RN_THREADS * qk::RN_MAX4, "rmsnorm_hilo: H=%d", H);
    SA_CUDA_TRY(launch_pdl_k(1, qk::rmsnorm_hilo_kernel, dim3(M), dim3(qk::RN_THREADS), 0, st, x, part, splits,
                             (size_t)M * H, w, H, eps, hi, lo));
    return SA_OK;
}
int launch_resid_add(cudaStream_t st, float* x, const float* part, int splits, int M, int H, int num_sms) {
    SA_CHECK_ARG(splits >= 1 && splits <= qk::QK_MAX_PLANES && part && H % 4 == 0, "resid_add: splits %d H %d", splits, H);
    const size_t n4 = (size_t)M * H / 4;
    const int grid = (int)std::min<size_t>((n4 + 255) / 256, (size_t)num_sms * 4);
    SA_CUDA_TRY(launch_pdl_k(1, qk::resid_add_kernel, dim3(grid), dim3(256), 0, st, x, part, splits, n4));
    return SA_OK;
}
int launch_swiglu_hilo(cudaStream_t st, const float* part, int splits, int M, int I, __nv_bfloat16* hi,
                       __nv_bfloat16* lo, long long ldo, int num_sms) {
    SA_CHECK_ARG(splits >= 1 && splits <= qk::QK_MAX_PLANES && part && I % 32 == 0, "swiglu_hilo: splits %d I %d", splits, I);
    const size_t n4 = (size_t)M * I / 4;
    const int grid = (int)std::min<size_t>((n4 + 255) / 256, (size_t)num_sms * 4);
    SA_CUDA_TRY(launch_pdl_k(1, qk::swiglu_hilo_kernel, dim3(grid), dim3(256), 0, st, part, splits, M, I, hi, lo, ldo));
    return SA_OK;
}
int launch_rope_table(cudaStream_t st, int n_pos, int D, float theta, float* cos_t, float* sin_t) {
    const size_t n = (size_t)n_pos * (D / 2);
    const int grid = (int)std::min<size_t>((n + 255) / 256, 4096);
    qk::rope_table_kernel<<<grid, 256, 0, st>>>(n_pos, D, theta, cos_t, sin_t);
    SA_CUDA_TRY(cudaGetLastError());
    return SA_OK;
}
int launch_qknorm_rope_append(cudaStream_t st, const float* qkv, int splits, int M, int hq, int hkv, const float* qn,
                              const float* kn, const float* cos_t, const float* sin_t, int pos0, const int* pos_dev,
                              int row_shift, float* q_out, float* kc, float* vc, int max_seq) {
    const int warps = M * (hq + 2 * hkv);
    SA_CHECK_ARG(splits >= 1 && splits <= qk::QK_MAX_PLANES, "qknorm_rope_append: splits %d", splits);
    SA_CUDA_TRY(launch_pdl_k(1, qk::qknorm_rope_append_kernel, dim3((warps + 7) / 8), dim3(256), 0, st, qkv, splits,
                             (size_t)M * (hq + 2 * hkv) * 128, M, hq, hkv, qn, kn, cos_t, sin_t, pos0, pos_dev,
                             row_shift, q_out, kc, vc, max_seq));
    SA_CUDA_TRY(cudaGetLastError());
    return SA_OK;
}
int launch_gemv2_tp(cudaStream_t st, int mode, bool norm, const __nv_bfloat16* W, int N_out, int K,
                    const float* x, const float* nw, float eps, float* y, unsigned long long* amax,
                    const QkvEpi* qkv, const TpArgs& tp, bool consume) {
    SA_CHECK_ARG(K % 64 == 0 && K / 8 <= 1024, "gemv2: K=%d (multiple of 64, <= 8192)", K);
    const int threads = (K / 8 + 31) / 32 * 32;
    // rows per CTA: enough CTAs to cover the SMs several times over
    const int rows = mode == QW_EPI_SWIGLU ? 2 * N_out : N_out;
    const int R = rows >= 8 * 1024 ? 8 : (rows >= 4 * 512 ? 4 : 2);
    const int outs = mode == QW_EPI_SWIGLU ? R / 2 : R;
    const int grid = (N_out + outs - 1) / outs;
    const QkvEpi e = qkv ? *qkv : QkvEpi{};
    const bool xchg = tp.world > 1 && (mode == QW_EPI_XCHG || consume);
    SA_CHECK_ARG(!xchg || (tp.seq && tp.status && tp.world <= TP_MAX), "gemv2: exchange operands missing");
    SA_CHECK_ARG(!consume || (tp.x_out && K % 256 == 0 && K / 8 == threads),
                 "gemv2: the consuming GEMV needs x_out and whole warps of K-chunks");
    SA_CHECK_ARG(mode != QW_EPI_XCHG || (tp.ll_stride >= N_out && tp.row == 0 && !norm && !amax),
                 "gemv2: exchange epilogue operands");
    SA_CHECK_ARG(!consume || !tp.use_ll || tp.ll_stride >= K, "gemv2: word area smaller than the residual");
#define SA_G2(M, N, RR, A, C) SA_CUDA_TRY(launch_pdl_k(0, qk::gemv2_kernel<M, N, RR, A, C>, dim3(grid), dim3(threads), \
                                                     0, st, W, N_out, K, x, nw, eps, y, amax, e, tp))
#define SA_G2R(M, N, A, C) do { if (R == 8) SA_G2(M, N, 8, A, C); else if (R == 4) SA_G2(M, N, 4, A, C); \
                                else SA_G2(M, N, 2, A, C); } while (0)
    if (consume) {
        SA_CHECK_ARG(norm, "gemv2: the consuming GEMV applies the norm");
        if (mode == QW_EPI_QKV) {
            SA_CHECK_ARG(qkv && !amax && qkv->cnt && N_out == 128 * (qkv->hq + 2 * qkv->hkv), "gemv2: QKV operands");
            SA_G2R(QW_EPI_QKV, true, false, true);
        } else if (mode == QW_EPI_SWIGLU) {
            SA_G2R(QW_EPI_SWIGLU, true, false, true);
        } else if (mode == QW_EPI_STORE) {
            if (amax) SA_G2R(QW_EPI_STORE, true, true, true); else SA_G2R(QW_EPI_STORE, true, false, true);
        } else {
            return set_error(SA_ERR_ARG, "gemv2: mode %d cannot consume an exchange", mode);
        }
    } else if (mode == QW_EPI_XCHG) {
        SA_G2R(QW_EPI_XCHG, false, false, false);
    } else if (mode == QW_EPI_QKV) {
        SA_CHECK_ARG(qkv && norm && !amax && qkv->cnt && N_out == 128 * (qkv->hq + 2 * qkv->hkv),
                     "gemv2: QKV epilogue needs its operands, the input norm and N_out = 128 (hq + 2 hkv)");
        SA_G2R(QW_EPI_QKV, true, false, false);
    } else if (amax) {
        SA_CHECK_ARG(mode == QW_EPI_STORE && norm, "gemv2: argmax only with the normed STORE head");
        SA_G2R(QW_EPI_STORE, true, true, false);
    } else if (mode == QW_EPI_STORE) {
        if (norm) SA_G2R(QW_EPI_STORE, true, false, false); else SA_G2R(QW_EPI_STORE, false, false, false);
    } else if (mode == QW_EPI_RESID) {
        if (norm) SA_G2R(QW_EPI_RESID, true, false, false); else SA_G2R(QW_EPI_RESID, false, false, false);
    } else {
        if (norm) SA_G2R(QW_EPI_SWIGLU, true, false, false); else SA_G2R(QW_EPI_SWIGLU, false, false, false);
    }
#undef SA_G2R
#undef SA_G2
    SA_CUDA_TRY(cudaGetLastError());
    return SA_OK;
}
int launch_gemv2(cudaStream_t st, int mode, bool norm, const __nv_bfloat16* W, int N_out, int K, const float* x,
                 const float* nw, float eps, float* y, unsigned long long* amax, const QkvEpi* qkv) {
    SA_CHECK_ARG(mode != QW_EPI_XCHG, "gemv2: the exchange epilogue needs launch_gemv2_tp");
    return launch_gemv2_tp(st, mode, norm, W, N_out, K, x, nw, eps, y, amax, qkv, TpArgs{}, false);
}
int launch_tp_scatter(cudaStream_t st, const float* part, int M, int H, const TpArgs& tp, int grid) {
    SA_CHECK_ARG(tp.world > 1 && tp.seq && tp.cnt && (size_t)M * H <= (size_t)tp.slot_floats && H % 4 == 0,
                 "tp_scatter: M=%d H=%d", M, H);
    qk::tp_scatter_kernel<<<grid, 256, 0, st>>>(part, (size_t)M * H / 4, tp);
    SA_CUDA_TRY(cudaGetLastError());
    return SA_OK;
}
int launch_rmsnorm_hilo_tp(cudaStream_t st, float* x, const float* w, int M, int H, float eps,
                           __nv_bfloat16* hi, __nv_bfloat16* lo, const TpArgs& tp) {
    SA_CHECK_ARG(tp.world > 1 && tp.seq && tp.status && (size_t)(tp.row + M) * H <= (size_t)tp.slot_floats,
                 "rmsnorm_hilo_tp: rows %d..%d", tp.row, tp.row + M);
    qk::rmsnorm_hilo_tp_kernel<<<M, 256, 0, st>>>(x, w, H, eps, hi, lo, tp);
    SA_CUDA_TRY(cudaGetLastError());
    return SA_OK;
}
int launch_tp_amax_token(cudaStream_t st, unsigned long long* amax, int64_t* tok, const TpArgs& tp, int seg) {
    SA_CHECK_ARG(tp.world > 1 && tp.seq && tp.status, "tp_amax_token: exchange operands missing");
    SA_CUDA_TRY(launch_pdl_k(3, qk::tp_amax_token_kernel, dim3(1), dim3(32), 0, st, amax, tok, tp, seg));
    SA_CUDA_TRY(cudaGetLastError());
    return SA_OK;
}
int launch_sp_rows_scatter(cudaStream_t st, const SpCopy& c, const TpArgs& tp, int grid) {
    SA_CHECK_ARG(tp.world > 1 && tp.seq && tp.cnt && c.nreg >= 1 && c.nreg <= 2 && c.blk_floats % 4 == 0 &&
                     c.stride % 4 == 0 && c.slot_floats % 4 == 0,
                 "sp_rows_scatter: regions %d, block %lld, stride %lld", c.nreg, c.blk_floats, c.stride);
    if (c.nblk == 0 || c.blk_floats == 0) grid = 1;     // nothing to copy: publish only
    qk::sp_rows_scatter_kernel<<<grid, 256, 0, st>>>(c, tp);
    SA_CUDA_TRY(cudaGetLastError());
    return SA_OK;
}
int launch_tc_pack(cudaStream_t st, const float* q, int M, int QD, const float* kc, const float* vc, int max_seq,
                   int hkv, int T, __nv_bfloat16* qb, __nv_bfloat16* kb, __nv_bfloat16* vb, int num_sms) {
    SA_CHECK_ARG(M >= 0 && (M == 0 || q) && QD % 8 == 0 && T >= 1 && T <= max_seq && hkv >= 1,
                 "tc_pack: M=%d QD=%d T=%d", M, QD, T);
    SA_CUDA_TRY(launch_pdl_k(4, qk::tc_pack_kernel, dim3(4 * num_sms), dim3(256), 0, st, q, (long long)M * QD / 8, kc,
                             vc, max_seq, hkv, T, qb, kb, vb));
    return SA_OK;
}
int launch_sp_wait(cudaStream_t st, const TpArgs& tp) {
    SA_CHECK_ARG(tp.world > 1 && tp.world <= 32 && tp.seq && tp.status, "sp_wait: world %d", tp.world);
    qk::sp_wait_kernel<<<1, 32, 0, st>>>(tp);
    SA_CUDA_TRY(cudaGetLastError());
    return SA_OK;
}
int launch_tp_seq_add(cudaStream_t st, unsigned* seq, int n) {
    SA_CUDA_TRY(launch_pdl_k(3, qk::tp_seq_add_kernel, dim3(1), dim3(1), 0, st, seq, n));
    SA_CUDA_TRY(cudaGetLastError());
    return SA_OK;
}
int launch_amax_to_token(cudaStream_t st, unsigned long long* amax, int64_t* tok) {
    SA_CUDA_TRY(launch_pdl_k(3, qk::amax_to_token_kernel, dim3(1), dim3(1), 0, st, amax, tok));
    SA_CUDA_TRY(cudaGetLastError());
    return SA_OK;
}

}  // namespace sa
