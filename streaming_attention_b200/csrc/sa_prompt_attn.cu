// sa_prompt_attn.cu -- causal attention of a prompt's queries over the fp32
// KV cache (the attention of qwen3_attention, tensor_cpp/src/qwen3_ops.cpp:
// 302-431, with the scale on the scores and the causal mask of
// create_causal_mask, :240-259; GQA by head index as repeat_kv, :194-234).
//
// Query m of the prompt (RoPE position pos0 + m) attends cache rows
// [0, T0 + m) with T0 = pos0 + 1.  One CTA serves QV = 8 query vectors that
// read the same KV head: 8 / G consecutive prompt rows x the G = hq / hkv
// query heads of that KV head (two vectors per warp, four warps).  The CTA streams the KV head's rows once, in
// 32-row tiles (cp.async, double-buffered), for all 16 vectors:
//   * scores: warp w owns vectors 2w, 2w+1, lane = key of the tile; q rows are
//     shared-memory broadcasts, K rows are padded to 132 floats so the 32
//     lanes' float4 reads hit distinct banks;
//   * online softmax in the exp2 domain (scale * log2 e folded into q), per
//     vector, reduced across the warp with shuffles;
//   * P.V: lane owns 4 consecutive output dims of the warp's 2 vectors; each
//     key is one float4 of V and one broadcast float2 of the 2 vectors' p.
// fp32 throughout (CUDA cores), like the reference.  The output is written as
// fp32 and/or as the bf16 hi/lo planes the o_proj GEMM reads.
#include <cuda_bf16.h>
#include <cmath>

#include "sa_internal.h"
#include "sa_ptx.cuh"
#include "sa_qwen3.h"
#include "sa_tc.cuh"

namespace sa {
namespace pa {

constexpr int D = 128, VPW = 2, NWARP = 4, QV = VPW * NWARP, KT = 32, KP = D + 4, THREADS = 32 * NWARP;
constexpr float LOG2E = 1.4426950408889634f;
constexpr int SMEM_FLOATS = QV * D + 2 * KT * KP + 2 * KT * D + NWARP * KT * VPW;
constexpr int SMEM_BYTES = SMEM_FLOATS * 4;

struct Args {
    const float* q;
    long long q_stride;       // floats between prompt rows of q
    const float* k;
    const float* v;
    long long kv_head_stride; // floats between KV heads of the cache
    int T0, M, hq, hkv, G, qb;  // qb = prompt rows per CTA = QV / G
    float qscale;             // scale * log2 e
    float* out;               // [M, o_stride] fp32 or null
    long long o_stride;
    __nv_bfloat16* out_hi;    // [M, o_stride] bf16 planes or null
    __nv_bfloat16* out_lo;
};

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_1() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_0() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

__global__ void __launch_bounds__(THREADS)
prompt_attn_kernel(const Args a) {
    extern __shared__ float4 smem4[];
    float* Qs = reinterpret_cast<float*>(smem4);     // [QV][D]
    float* Ks = Qs + QV * D;                          // [2][KT][KP]
    float* Vs = Ks + 2 * KT * KP;                     // [2][KT][D]
    float* Ps = Vs + 2 * KT * D;                      // [NWARP][KT][VPW]
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int h = blockIdx.y;
    // heaviest (latest) query blocks first
    const int blk = gridDim.x - 1 - blockIdx.x;
    const int m0 = blk * a.qb;
    const int m_end = min(m0 + a.qb, a.M);            // rows [m0, m_end)
    const int n_keys = a.T0 + m_end - 1;              // rows the last query attends
    const float* kh = a.k + (size_t)h * a.kv_head_stride;
    const float* vh = a.v + (size_t)h * a.kv_head_stride;

    pdl_wait();
    pdl_trigger();
    // queries (pre-scaled); vector j = prompt row m0 + j / G, head h * G + j % G
    for (int e = tid; e < QV * (D / 4); e += THREADS) {
        const int j = e / (D / 4), c = (e % (D / 4)) * 4;
        const int m = m0 + j / a.G, head = h * a.G + j % a.G;
        float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
        if (m < m_end) {
            x = __ldg(reinterpret_cast<const float4*>(a.q + (size_t)m * a.q_stride + (size_t)head * D + c));
            x.x *= a.qscale; x.y *= a.qscale; x.z *= a.qscale; x.w *= a.qscale;
        }
        *reinterpret_cast<float4*>(Qs + j * D + c) = x;
    }
    const int n_tiles = (n_keys + KT - 1) / KT;
    auto load_tile = [&](int t, int buf) {
        float* kd = Ks + buf * KT * KP;
        float* vd = Vs + buf * KT * D;
        for (int e = tid; e < KT * (D / 4); e += THREADS) {
            const int r = e / (D / 4), c = (e % (D / 4)) * 4, row = t * KT + r;
            if (row < n_keys) {
                cp_async16(kd + r * KP + c, kh + (size_t)row * D + c);
                cp_async16(vd + r * D + c, vh + (size_t)row * D + c);
            } else {
                *reinterpret_cast<float4*>(kd + r * KP + c) = make_float4(0.f, 0.f, 0.f, 0.f);
                *reinterpret_cast<float4*>(vd + r * D + c) = make_float4(0.f, 0.f, 0.f, 0.f);
            }
        }
        cp_async_commit();
    };
    load_tile(0, 0);

    // per warp: vectors VPW w + i; per lane: output dims 4 lane .. 4 lane + 3
    float mrun[VPW], lrun[VPW];
    float4 o[VPW];
    int lim[VPW];   // keys vector i may attend
#pragma unroll
    for (int i = 0; i < VPW; ++i) {
        mrun[i] = -INFINITY;
        lrun[i] = 0.f;
        o[i] = make_float4(0.f, 0.f, 0.f, 0.f);
        const int j = warp * VPW + i, m = m0 + j / a.G;
        lim[i] = m < m_end ? a.T0 + m : 0;
    }
    for (int t = 0; t < n_tiles; ++t) {
        if (t + 1 < n_tiles) {
            load_tile(t + 1, (t + 1) & 1);
            cp_async_wait_1();
        } else {
            cp_async_wait_0();
        }
        __syncthreads();
        const float* kt = Ks + (t & 1) * KT * KP;
        const float* vt = Vs + (t & 1) * KT * D;
        // scores s[i] = q_i . k_lane
        float s[VPW];
#pragma unroll
        for (int i = 0; i < VPW; ++i) s[i] = 0.f;
        const float* qw = Qs + warp * VPW * D;
#pragma unroll 8
        for (int d = 0; d < D; d += 4) {
            const float4 kv = *reinterpret_cast<const float4*>(kt + lane * KP + d);
#pragma unroll
            for (int i = 0; i < VPW; ++i) {
                const float4 qv = *reinterpret_cast<const float4*>(qw + i * D + d);
                s[i] = fmaf(qv.x, kv.x, s[i]);
                s[i] = fmaf(qv.y, kv.y, s[i]);
                s[i] = fmaf(qv.z, kv.z, s[i]);
                s[i] = fmaf(qv.w, kv.w, s[i]);
            }
        }
        const int key = t * KT + lane;
        float p[VPW];
#pragma unroll
        for (int i = 0; i < VPW; ++i) {
            const float si = key < lim[i] ? s[i] : -INFINITY;
            float mx = si;
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
            const float mnew = fmaxf(mrun[i], mx);
            // rows with no valid key yet keep m = -inf: nothing to rescale
            const float alpha = mnew == -INFINITY ? 1.f : ex2(mrun[i] - mnew);
            p[i] = mnew == -INFINITY ? 0.f : ex2(si - mnew);
            float sum = p[i];
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
            lrun[i] = lrun[i] * alpha + sum;
            mrun[i] = mnew;
            o[i].x *= alpha; o[i].y *= alpha; o[i].z *= alpha; o[i].w *= alpha;
        }
        float* pw = Ps + warp * KT * VPW;
        static_assert(VPW == 2, "p is stored as float2");
        *reinterpret_cast<float2*>(pw + lane * VPW) = make_float2(p[0], p[1]);
        __syncwarp();
#pragma unroll 8
        for (int kk = 0; kk < KT; ++kk) {
            const float2 pk = *reinterpret_cast<const float2*>(pw + kk * VPW);
            const float4 vv = *reinterpret_cast<const float4*>(vt + kk * D + lane * 4);
            o[0].x = fmaf(pk.x, vv.x, o[0].x); o[0].y = fmaf(pk.x, vv.y, o[0].y);
            o[0].z = fmaf(pk.x, vv.z, o[0].z); o[0].w = fmaf(pk.x, vv.w, o[0].w);
            o[1].x = fmaf(pk.y, vv.x, o[1].x); o[1].y = fmaf(pk.y, vv.y, o[1].y);
            o[1].z = fmaf(pk.y, vv.z, o[1].z); o[1].w = fmaf(pk.y, vv.w, o[1].w);
        }
        __syncthreads();   // the buffer of tile t is refilled at t + 2
    }
#pragma unroll
    for (int i = 0; i < VPW; ++i) {
        const int j = warp * VPW + i, m = m0 + j / a.G, head = h * a.G + j % a.G;
        if (m >= m_end) continue;
        const float inv = lrun[i] > 0.f ? 1.f / lrun[i] : 0.f;
        const float4 r = make_float4(o[i].x * inv, o[i].y * inv, o[i].z * inv, o[i].w * inv);
        const size_t off = (size_t)m * a.o_stride + (size_t)head * D + lane * 4;
        if (a.out) *reinterpret_cast<float4*>(a.out + off) = r;
        if (a.out_hi) {
            const __nv_bfloat162 h01 = __floats2bfloat162_rn(r.x, r.y), h23 = __floats2bfloat162_rn(r.z, r.w);
            const float2 f01 = __bfloat1622float2(h01), f23 = __bfloat1622float2(h23);
            const __nv_bfloat162 l01 = __floats2bfloat162_rn(r.x - f01.x, r.y - f01.y);
            const __nv_bfloat162 l23 = __floats2bfloat162_rn(r.z - f23.x, r.w - f23.y);
            uint2 uh, ul;
            uh.x = *reinterpret_cast<const uint32_t*>(&h01); uh.y = *reinterpret_cast<const uint32_t*>(&h23);
            ul.x = *reinterpret_cast<const uint32_t*>(&l01); ul.y = *reinterpret_cast<const uint32_t*>(&l23);
            *reinterpret_cast<uint2*>(a.out_hi + off) = uh;
            *reinterpret_cast<uint2*>(a.out_lo + off) = ul;
        }
    }
}

}  // namespace pa

int prompt_attn_launch(cudaStream_t st, const float* q, long long q_stride, const float* k, const float* v,
                       long long kv_head_stride, int T0, int M, int d, int hq, int hkv, float scale, float* out,
                       long long o_stride, __nv_bfloat16* out_hi, __nv_bfloat16* out_lo) {
    SA_CHECK_ARG(d == pa::D, "prompt attention: head_dim %d (128 supported)", d);
    SA_CHECK_ARG(M >= 1 && T0 >= 1 && hkv >= 1 && hq % hkv == 0, "prompt attention: M=%d T0=%d hq=%d hkv=%d", M, T0,
                 hq, hkv);
    const int G = hq / hkv;
    SA_CHECK_ARG(G == 1 || G == 2 || G == 4 || G == 8, "prompt attention: hq/hkv=%d", G);
    SA_CHECK_ARG(q_stride % 4 == 0 && kv_head_stride % 4 == 0 && o_stride % 4 == 0 && ((uintptr_t)q & 15) == 0 &&
                     ((uintptr_t)k & 15) == 0 && ((uintptr_t)v & 15) == 0 && ((uintptr_t)out & 15) == 0 &&
                     ((uintptr_t)out_hi & 7) == 0 && ((uintptr_t)out_lo & 7) == 0,
                 "prompt attention: alignment");
    SA_CHECK_ARG(out || (out_hi && out_lo), "prompt attention: no output");
    pa::Args a;
    a.q = q; a.q_stride = q_stride; a.k = k; a.v = v; a.kv_head_stride = kv_head_stride;
    a.T0 = T0; a.M = M; a.hq = hq; a.hkv = hkv; a.G = G; a.qb = pa::QV / G;
    a.qscale = scale * pa::LOG2E;
    a.out = out; a.o_stride = o_stride; a.out_hi = out_hi; a.out_lo = out_lo;
    const int nblk = (M + a.qb - 1) / a.qb;
    SA_CHECK_ARG(nblk <= 2147483647 && hkv <= 65535, "prompt attention: grid");
    SA_RC_TRY(set_smem_attr_once((const void*)pa::prompt_attn_kernel, pa::SMEM_BYTES));
    SA_CUDA_TRY(launch_pdl(pa::prompt_attn_kernel, dim3(nblk, hkv), dim3(pa::THREADS), pa::SMEM_BYTES, st, a));
    return SA_OK;
}

}  // namespace sa
