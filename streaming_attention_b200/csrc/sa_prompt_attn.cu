// sa_prompt_attn.cu -- causal attention of a prompt's queries over the fp32
// KV cache (the attention of qwen3_attention, tensor_cpp/src/qwen3_ops.cpp:
// 302-431, with the scale on the scores and the causal mask of
// create_causal_mask, :240-259; GQA by head index as repeat_kv, :194-234).
//
// Query m of the prompt (RoPE position pos0 + m) attends cache rows
// [0, T0 + m) with T0 = pos0 + 1.  One CTA serves QV = 16 query vectors that
// read the same KV head: 16 / G consecutive prompt rows x the G = hq / hkv
// query heads of that KV head.  The CTA streams the head's rows in rounds of
// 128 (cp.async into shared memory, K before V) and its four warps split each
// round's keys, 32 each, for all 16 vectors.  Every thread works on a
// register tile so that shared memory is not the limit:
//   * scores: lane = (vector quad vq, key group kg) computes the 4 x 4 tile
//     of vectors vq + 4i and keys kg + 8j: 8 float4 reads per 64 FMAs (rows
//     padded to 132 floats, so the 8 key rows / 4 query rows a read touches
//     sit in distinct banks);
//   * online softmax in the exp2 domain (scale * log2 e folded into q), per
//     warp and vector, reduced over the 8 key-group lanes with shuffles;
//   * P.V: lane owns 4 consecutive output dims of all 16 vectors; each key
//     is one float4 of V and four broadcast float4 of the 16 vectors' p;
//   * the four warps' (m, l, O) states are merged at the end (the merge of
//     streaming_omp.cpp:27-48), in warp order.
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

constexpr int D = 128, QV = 16, NWARP = 4, KW = 32, KR = NWARP * KW, KP = D + 4, THREADS = 32 * NWARP;
constexpr float LOG2E = 1.4426950408889634f;
constexpr int OFF_Q = 0;                           // [QV][KP]
constexpr int OFF_K = OFF_Q + QV * KP;             // [KR][KP]
constexpr int OFF_V = OFF_K + KR * KP;             // [KR][D]
constexpr int OFF_P = OFF_V + KR * D;              // [NWARP][KW][QV]
constexpr int SMEM_FLOATS = OFF_P + NWARP * KW * QV;
constexpr int SMEM_BYTES = SMEM_FLOATS * 4;
static_assert(NWARP * QV * (D + 2) <= KR * KP, "the merge area reuses the K rows");

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

__global__ void __launch_bounds__(THREADS, 1)
prompt_attn_kernel(const Args a) {
    extern __shared__ float4 smem4[];
    float* sm = reinterpret_cast<float*>(smem4);
    float* Qs = sm + OFF_Q;
    float* Ks = sm + OFF_K;
    float* Vs = sm + OFF_V;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    // score phase: lane = (vector quad vq, key group kg); vectors vq + 4 i,
    // keys kg + 8 j of the warp's 32 (i, j < 4)
    const int kg = lane & 7, vq = lane >> 3;
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
        *reinterpret_cast<float4*>(Qs + j * KP + c) = x;
    }
    // keys of this lane's 4 vectors (0 for the unused vectors of a ragged block)
    int lim[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int m = m0 + (vq + 4 * i) / a.G;
        lim[i] = m < m_end ? a.T0 + m : 0;
    }
    // per warp: the state of all 16 vectors; P.V lane = 4 output dims
    float mrun[QV], lrun[QV];
    float4 o[QV];
#pragma unroll
    for (int j = 0; j < QV; ++j) {
        mrun[j] = -INFINITY;
        lrun[j] = 0.f;
        o[j] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    float* Pw = sm + OFF_P + warp * KW * QV;          // [KW][QV]
    const int n_rounds = (n_keys + KR - 1) / KR;
    for (int rd = 0; rd < n_rounds; ++rd) {
        const int base = rd * KR;
        if (rd > 0) __syncthreads();                   // every warp is done with the previous round's rows
        // K rows first (group 0), then V rows (group 1): the scores start
        // while V is still arriving
        for (int e = tid; e < KR * (D / 4); e += THREADS) {
            const int r = e / (D / 4), c = (e % (D / 4)) * 4, row = base + r;
            if (row < n_keys) cp_async16(Ks + r * KP + c, kh + (size_t)row * D + c);
            else *reinterpret_cast<float4*>(Ks + r * KP + c) = make_float4(0.f, 0.f, 0.f, 0.f);
        }
        cp_async_commit();
        for (int e = tid; e < KR * (D / 4); e += THREADS) {
            const int r = e / (D / 4), c = (e % (D / 4)) * 4, row = base + r;
            if (row < n_keys) cp_async16(Vs + r * D + c, vh + (size_t)row * D + c);
            else *reinterpret_cast<float4*>(Vs + r * D + c) = make_float4(0.f, 0.f, 0.f, 0.f);
        }
        cp_async_commit();
        cp_async_wait_1();
        __syncthreads();
        // scores s[i][j] = q_{vq + 4i} . k_{kg + 8j} over this warp's 32 keys
        const float* kw = Ks + (warp * KW + kg) * KP;
        const float* qv = Qs + vq * KP;
        float sc[4][4];
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int j = 0; j < 4; ++j) sc[i][j] = 0.f;
#pragma unroll 4
        for (int d = 0; d < D; d += 4) {
            float4 kk[4], qq[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) kk[j] = *reinterpret_cast<const float4*>(kw + 8 * j * KP + d);
#pragma unroll
            for (int i = 0; i < 4; ++i) qq[i] = *reinterpret_cast<const float4*>(qv + 4 * i * KP + d);
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    sc[i][j] = fmaf(qq[i].x, kk[j].x, sc[i][j]);
                    sc[i][j] = fmaf(qq[i].y, kk[j].y, sc[i][j]);
                    sc[i][j] = fmaf(qq[i].z, kk[j].z, sc[i][j]);
                    sc[i][j] = fmaf(qq[i].w, kk[j].w, sc[i][j]);
                }
        }
        // online softmax of the warp's 32 keys per vector (over j in-thread,
        // then the 8 key-group lanes), P to shared memory [key][vector]
        float alpha[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            float mx = -INFINITY;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int key = base + warp * KW + kg + 8 * j;
                if (key >= lim[i]) sc[i][j] = -INFINITY;
                mx = fmaxf(mx, sc[i][j]);
            }
#pragma unroll
            for (int off = 1; off < 8; off <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
            // every lane holds the state of all 16 vectors; this lane's vector i is vq + 4 i
            float mold = mrun[0];
#pragma unroll
            for (int v = 0; v < 4; ++v) if (vq == v) mold = mrun[v + 4 * i];
            const float mnew = fmaxf(mold, mx);
            alpha[i] = mnew == -INFINITY ? 1.f : ex2(mold - mnew);
            float sum = 0.f;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const float p = mnew == -INFINITY ? 0.f : ex2(sc[i][j] - mnew);
                Pw[(kg + 8 * j) * QV + vq + 4 * i] = p;
                sum += p;
            }
#pragma unroll
            for (int off = 1; off < 8; off <<= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
            // broadcast vector (v + 4 i)'s new state from the lanes of quad v
#pragma unroll
            for (int v = 0; v < 4; ++v) {
                const float a_v = __shfl_sync(0xffffffffu, alpha[i], 8 * v);
                const float m_v = __shfl_sync(0xffffffffu, mnew, 8 * v);
                const float s_v = __shfl_sync(0xffffffffu, sum, 8 * v);
                const int jv = v + 4 * i;
                lrun[jv] = lrun[jv] * a_v + s_v;
                mrun[jv] = m_v;
                o[jv].x *= a_v; o[jv].y *= a_v; o[jv].z *= a_v; o[jv].w *= a_v;
            }
        }
        cp_async_wait_0();
        __syncthreads();                               // V rows landed; P of the warp visible
        // P.V over this warp's 32 keys; lane = output dims 4 lane .. 4 lane + 3
        const float* vw = Vs + warp * KW * D + lane * 4;
#pragma unroll 2
        for (int kk = 0; kk < KW; ++kk) {
            const float4 vv = *reinterpret_cast<const float4*>(vw + kk * D);
            const float* pk = Pw + kk * QV;
#pragma unroll
            for (int q4 = 0; q4 < QV / 4; ++q4) {
                const float4 pp = *reinterpret_cast<const float4*>(pk + 4 * q4);
                const float pj[4] = {pp.x, pp.y, pp.z, pp.w};
#pragma unroll
                for (int t = 0; t < 4; ++t) {
                    float4& acc = o[4 * q4 + t];
                    acc.x = fmaf(pj[t], vv.x, acc.x);
                    acc.y = fmaf(pj[t], vv.y, acc.y);
                    acc.z = fmaf(pj[t], vv.z, acc.z);
                    acc.w = fmaf(pj[t], vv.w, acc.w);
                }
            }
        }
        __syncwarp();
    }
    // merge the warps' states (the K rows are free now): [warp][vector][m, l, O]
    __syncthreads();
    float* Ms = sm + OFF_K;
#pragma unroll
    for (int j = 0; j < QV; ++j) {
        float* st = Ms + (warp * QV + j) * (D + 2);
        if (lane == 0) { st[0] = mrun[j]; st[1] = lrun[j]; }
        *reinterpret_cast<float2*>(st + 2 + lane * 4) = make_float2(o[j].x, o[j].y);
        *reinterpret_cast<float2*>(st + 4 + lane * 4) = make_float2(o[j].z, o[j].w);
    }
    __syncthreads();
    for (int j = warp; j < QV; j += NWARP) {
        const int m = m0 + j / a.G, head = h * a.G + j % a.G;
        if (m >= m_end) continue;
        float mw[NWARP], mx = -INFINITY;
#pragma unroll
        for (int w = 0; w < NWARP; ++w) {
            mw[w] = Ms[(w * QV + j) * (D + 2)];
            mx = fmaxf(mx, mw[w]);
        }
        float l = 0.f;
        float4 r = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int w = 0; w < NWARP; ++w) {
            const float* st = Ms + (w * QV + j) * (D + 2);
            const float f = mw[w] == -INFINITY ? 0.f : ex2(mw[w] - mx);
            l += st[1] * f;
            const float2 a01 = *reinterpret_cast<const float2*>(st + 2 + lane * 4);
            const float2 a23 = *reinterpret_cast<const float2*>(st + 4 + lane * 4);
            r.x += a01.x * f; r.y += a01.y * f; r.z += a23.x * f; r.w += a23.y * f;
        }
        const float inv = l > 0.f ? 1.f / l : 0.f;
        r.x *= inv; r.y *= inv; r.z *= inv; r.w *= inv;
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
    SA_CHECK_ARG(G == 1 || G == 2 || G == 4 || G == 8 || G == 16, "prompt attention: hq/hkv=%d", G);
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
    SA_CHECK_ARG(hkv <= 65535, "prompt attention: grid");
    SA_RC_TRY(set_smem_attr_once((const void*)pa::prompt_attn_kernel, pa::SMEM_BYTES));
    SA_CUDA_TRY(launch_pdl(pa::prompt_attn_kernel, dim3(nblk, hkv), dim3(pa::THREADS), pa::SMEM_BYTES, st, a));
    return SA_OK;
}

}  // namespace sa
