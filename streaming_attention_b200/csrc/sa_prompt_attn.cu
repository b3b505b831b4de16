// sa_prompt_attn.cu -- causal attention of a prompt's queries over the fp32
// KV cache (the attention of qwen3_attention, tensor_cpp/src/qwen3_ops.cpp:
// 302-431, with the scale on the scores and the causal mask of
// create_causal_mask, :240-259; GQA by head index as repeat_kv, :194-234).
//
// Query m of the prompt (RoPE position pos0 + m) attends cache rows
// [0, T0 + m) with T0 = pos0 + 1.  One CTA serves QV = 16 query vectors that
// read the same KV head: 16 / G consecutive prompt rows x the G = hq / hkv
// query heads of that KV head.  The CTA streams the head's rows in rounds of
// 128 -- K as four 32-column TMA tiles with the 128-byte swizzle, V as one
// bulk copy -- and its eight warps split each round's keys, 16 each, for all
// 16 vectors.  Every thread works on a register tile so that shared memory
// is not the limit:
//   * scores: lane = (vector quad vq, key group kg) computes the 4 x 2 tile
//     of vectors vq + 4i and keys kg + 8j: 6 float4 reads per 32 FMAs; the
//     swizzle puts the 8 key rows a read touches (rows kg mod 8) in distinct
//     banks, the query rows are padded to 132 floats;
//   * online softmax in the exp2 domain (scale * log2 e folded into q), per
//     warp and vector, reduced over the 8 key-group lanes with shuffles;
//   * P.V: lane owns 4 consecutive output dims of all 16 vectors; each key
//     is one float4 of V and four broadcast float4 of the 16 vectors' p;
//   * the eight warps' (m, l, O) states are merged at the end (the merge of
//     streaming_omp.cpp:27-48), in warp order.
// fp32 throughout (CUDA cores), like the reference.  The output is written as
// fp32 and/or as the bf16 hi/lo planes the o_proj GEMM reads.  Waits on the
// copies are bounded (status SA_STATUS_TIMEOUT, no output).
#include <cuda_bf16.h>
#include <cmath>

#include "sa_internal.h"
#include "sa_ptx.cuh"
#include "sa_qwen3.h"
#include "sa_tc.cuh"

namespace sa {
namespace pa {

constexpr int D = 128, QV = 16, NWARP = 8, KW = 16, KR = NWARP * KW, KP = D + 4, THREADS = 32 * NWARP;
constexpr int NJ = KW / 8;                         // keys per lane in the score tile
constexpr float LOG2E = 1.4426950408889634f;
constexpr int K_TILE = KR * 32;                    // floats of one 32-column K tile (128 rows x 128 bytes)
constexpr int OFF_K = 0;                           // [4 tiles][KR][32] swizzled (1024-byte aligned)
constexpr int OFF_V = OFF_K + 4 * K_TILE;          // [KR][D]
constexpr int OFF_Q = OFF_V + KR * D;              // [QV][KP]
constexpr int OFF_P = OFF_Q + QV * KP;             // [NWARP][KW][QV]
constexpr int OFF_F = OFF_P + NWARP * KW * QV;     // merge factors [QV][NWARP + 1]
constexpr int OFF_BAR = (OFF_F + QV * (NWARP + 1) + 1) & ~1;   // two mbarriers
constexpr int SMEM_FLOATS = OFF_BAR + 4;
constexpr int SMEM_BYTES = SMEM_FLOATS * 4 + 1024;               // + alignment slack
static_assert(NWARP * QV * (D + 2) <= 4 * K_TILE + KR * D, "the merge area reuses the K and V rows");

struct Args {
    const float* q;
    long long q_stride;       // floats between prompt rows of q
    const float* v;
    long long kv_head_stride; // floats between KV heads of the cache
    int T0, M, hq, hkv, G, qb;  // qb = prompt rows per CTA = QV / G
    float qscale;             // scale * log2 e
    float* out;               // [M, o_stride] fp32 or null
    long long o_stride;
    __nv_bfloat16* out_hi;    // [M, o_stride] bf16 planes or null
    __nv_bfloat16* out_lo;
    int* status;
};

__global__ void __launch_bounds__(THREADS, 1)
prompt_attn_kernel(const __grid_constant__ CUtensorMap tk, const Args a) {
    extern __shared__ unsigned char smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    float* sm = reinterpret_cast<float*>(smem_raw + (((raw + 1023u) & ~1023u) - raw));
    float* Ks = sm + OFF_K;
    float* Vs = sm + OFF_V;
    float* Qs = sm + OFF_Q;
    uint64_t* kbar = reinterpret_cast<uint64_t*>(sm + OFF_BAR);
    uint64_t* vbar = kbar + 1;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    // score phase: lane = (vector quad vq, key group kg); vectors vq + 4 i,
    // keys kg + 8 j of the warp's 16 (i < 4, j < NJ)
    const int kg = lane & 7, vq = lane >> 3;
    const int h = blockIdx.y;
    // heaviest (latest) query blocks first
    const int blk = gridDim.x - 1 - blockIdx.x;
    const int m0 = blk * a.qb;
    const int m_end = min(m0 + a.qb, a.M);            // rows [m0, m_end)
    const int n_keys = a.T0 + m_end - 1;              // rows the last query attends
    const int krow0 = (int)(h * (a.kv_head_stride / D));   // tensor-map row of this head's key 0
    const float* vh = a.v + (size_t)h * a.kv_head_stride;
    if (tid == 0) {
        tc::prefetch_tmap(&tk);
        mbar_init(kbar, 1);
        mbar_init(vbar, 1);
        fence_barrier_init();
    }

    pdl_wait();
    pdl_trigger();
    // queries (pre-scaled); vector j = prompt row m0 + j / G, head h * G + j % G;
    // both loads of a thread are issued before either is stored
    {
        constexpr int PER = QV * (D / 4) / THREADS;
        float4 x[PER];
#pragma unroll
        for (int u = 0; u < PER; ++u) {
            const int e = tid + u * THREADS, j = e / (D / 4), c = (e % (D / 4)) * 4;
            const int m = m0 + j / a.G, head = h * a.G + j % a.G;
            x[u] = m < m_end ? __ldg(reinterpret_cast<const float4*>(a.q + (size_t)m * a.q_stride +
                                                                      (size_t)head * D + c))
                             : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int u = 0; u < PER; ++u) {
            const int e = tid + u * THREADS, j = e / (D / 4), c = (e % (D / 4)) * 4;
            *reinterpret_cast<float4*>(Qs + j * KP + c) =
                make_float4(x[u].x * a.qscale, x[u].y * a.qscale, x[u].z * a.qscale, x[u].w * a.qscale);
        }
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
    bool ok = true;
    for (int rd = 0; rd < n_rounds; ++rd) {
        const int base = rd * KR, nr = min(KR, n_keys - base);
        if (rd > 0) __syncthreads();                   // every warp is done with the previous round's rows
        // K: four 32-column tiles of 128 rows (rows past the keys are masked);
        // V: one bulk copy of the round's rows, the rest zeroed (0 * p must
        // stay 0)
        if (warp == 0) {
            if (lane == 0) {
                fence_proxy_async_smem();              // the previous round's reads before the copies' writes
                mbar_arrive_expect_tx(kbar, (uint32_t)4 * K_TILE * 4);
                for (int t = 0; t < 4; ++t) tc::tma_load_2d(Ks + t * K_TILE, &tk, 32 * t, krow0 + base, kbar);
                mbar_arrive_expect_tx(vbar, (uint32_t)nr * D * 4);
                bulk_g2s(Vs, vh + (size_t)base * D, (uint32_t)nr * D * 4, vbar);
            }
        } else {
            for (int e = tid - 32; e < (KR - nr) * (D / 4); e += THREADS - 32)
                reinterpret_cast<float4*>(Vs + nr * D)[e] = make_float4(0.f, 0.f, 0.f, 0.f);
        }
        ok = ok && mbar_wait(kbar, rd & 1, a.status);
        __syncthreads();
        // scores s[i][j] = q_{vq + 4i} . k_{kg + 8j} over this warp's keys;
        // K float4 c of row r (tile c / 8) sits at chunk (c % 8) ^ (r % 8) of
        // the row, and r % 8 = kg
        const float* kw = Ks + (warp * KW + kg) * 32;
        const float* qv = Qs + vq * KP;
        float sc[4][NJ];
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int j = 0; j < NJ; ++j) sc[i][j] = 0.f;
        if (warp * KW < nr) {                          // warps past the last key skip the scores
#pragma unroll 4
            for (int c = 0; c < D / 4; ++c) {
                const float* kt = kw + (c >> 3) * K_TILE + (((c & 7) ^ kg) << 2);
                float4 kk[NJ], qq[4];
#pragma unroll
                for (int j = 0; j < NJ; ++j) kk[j] = *reinterpret_cast<const float4*>(kt + 8 * j * 32);
#pragma unroll
                for (int i = 0; i < 4; ++i) qq[i] = *reinterpret_cast<const float4*>(qv + 4 * i * KP + 4 * c);
#pragma unroll
                for (int i = 0; i < 4; ++i)
#pragma unroll
                    for (int j = 0; j < NJ; ++j) {
                        sc[i][j] = fmaf(qq[i].x, kk[j].x, sc[i][j]);
                        sc[i][j] = fmaf(qq[i].y, kk[j].y, sc[i][j]);
                        sc[i][j] = fmaf(qq[i].z, kk[j].z, sc[i][j]);
                        sc[i][j] = fmaf(qq[i].w, kk[j].w, sc[i][j]);
                    }
            }
        }
        // online softmax of the warp's keys per vector (over j in-thread, then
        // the 8 key-group lanes), P to shared memory [key][vector]
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            float mx = -INFINITY;
#pragma unroll
            for (int j = 0; j < NJ; ++j) {
                const int key = base + warp * KW + kg + 8 * j;
                if (key >= lim[i]) sc[i][j] = -INFINITY;
                mx = fmaxf(mx, sc[i][j]);
            }
#pragma unroll
            for (int off = 1; off < 8; off <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
            // every lane holds the state of all 16 vectors; this lane's vector i is vq + 4 i
            float mold = mrun[i * 4];
#pragma unroll
            for (int v = 1; v < 4; ++v) if (vq == v) mold = mrun[v + 4 * i];
            const float mnew = fmaxf(mold, mx);
            const float alpha = mnew == -INFINITY ? 1.f : ex2(mold - mnew);
            float sum = 0.f;
#pragma unroll
            for (int j = 0; j < NJ; ++j) {
                const float p = mnew == -INFINITY ? 0.f : ex2(sc[i][j] - mnew);
                Pw[(kg + 8 * j) * QV + vq + 4 * i] = p;
                sum += p;
            }
#pragma unroll
            for (int off = 1; off < 8; off <<= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
            // broadcast vector (v + 4 i)'s new state from the lanes of quad v
#pragma unroll
            for (int v = 0; v < 4; ++v) {
                const float a_v = __shfl_sync(0xffffffffu, alpha, 8 * v);
                const float m_v = __shfl_sync(0xffffffffu, mnew, 8 * v);
                const float s_v = __shfl_sync(0xffffffffu, sum, 8 * v);
                const int jv = v + 4 * i;
                lrun[jv] = lrun[jv] * a_v + s_v;
                mrun[jv] = m_v;
                o[jv].x *= a_v; o[jv].y *= a_v; o[jv].z *= a_v; o[jv].w *= a_v;
            }
        }
        ok = ok && mbar_wait(vbar, rd & 1, a.status);
        __syncwarp();                                  // P of the warp visible to the warp
        // P.V over this warp's keys; lane = output dims 4 lane .. 4 lane + 3
        if (warp * KW < nr) {
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
        }
        __syncwarp();
    }
    // merge the warps' states (the K and V rows are free now): [warp][vector][m, l, O]
    __syncthreads();
    float* Ms = sm + OFF_K;
    float* F = sm + OFF_F;
#pragma unroll
    for (int j = 0; j < QV; ++j) {
        float* st = Ms + (warp * QV + j) * (D + 2);
        if (lane == 0) { st[0] = mrun[j]; st[1] = lrun[j]; }
        *reinterpret_cast<float2*>(st + 2 + lane * 4) = make_float2(o[j].x, o[j].y);
        *reinterpret_cast<float2*>(st + 4 + lane * 4) = make_float2(o[j].z, o[j].w);
    }
    __syncthreads();
    // per vector: each warp's weight e^(m_w - m) / l (warp order), in F
    if (tid < QV) {
        float mx = -INFINITY, mw[NWARP];
#pragma unroll
        for (int w = 0; w < NWARP; ++w) {
            mw[w] = Ms[(w * QV + tid) * (D + 2)];
            mx = fmaxf(mx, mw[w]);
        }
        float l = 0.f;
#pragma unroll
        for (int w = 0; w < NWARP; ++w) {
            mw[w] = mw[w] == -INFINITY ? 0.f : ex2(mw[w] - mx);
            l += Ms[(w * QV + tid) * (D + 2) + 1] * mw[w];
        }
        const float inv = l > 0.f ? 1.f / l : 0.f;
#pragma unroll
        for (int w = 0; w < NWARP; ++w) F[tid * (NWARP + 1) + w] = mw[w] * inv;
    }
    __syncthreads();
    if (!ok) return;
    // outputs: item = (vector, 4 dims)
    for (int e = tid; e < QV * (D / 4); e += THREADS) {
        const int j = e / (D / 4), c = (e % (D / 4)) * 4;
        const int m = m0 + j / a.G, head = h * a.G + j % a.G;
        if (m >= m_end) continue;
        float4 r = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int w = 0; w < NWARP; ++w) {
            const float* st = Ms + (w * QV + j) * (D + 2) + 2 + c;
            const float f = F[j * (NWARP + 1) + w];
            const float2 a01 = *reinterpret_cast<const float2*>(st);
            const float2 a23 = *reinterpret_cast<const float2*>(st + 2);
            r.x += a01.x * f; r.y += a01.y * f; r.z += a23.x * f; r.w += a23.y * f;
        }
        const size_t off = (size_t)m * a.o_stride + (size_t)head * D + c;
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

int prompt_attn_launch(cudaStream_t st, int* status, const float* q, long long q_stride, const float* k,
                       const float* v, long long kv_head_stride, long long kv_rows, int T0, int M, int d, int hq,
                       int hkv, float scale, float* out, long long o_stride, __nv_bfloat16* out_hi,
                       __nv_bfloat16* out_lo) {
    SA_CHECK_ARG(d == pa::D, "prompt attention: head_dim %d (128 supported)", d);
    SA_CHECK_ARG(M >= 1 && T0 >= 1 && hkv >= 1 && hq % hkv == 0, "prompt attention: M=%d T0=%d hq=%d hkv=%d", M, T0,
                 hq, hkv);
    const int G = hq / hkv;
    SA_CHECK_ARG(G == 1 || G == 2 || G == 4 || G == 8 || G == 16, "prompt attention: hq/hkv=%d", G);
    SA_CHECK_ARG(q_stride % 4 == 0 && kv_head_stride % d == 0 && o_stride % 4 == 0 && ((uintptr_t)q & 15) == 0 &&
                     ((uintptr_t)k & 15) == 0 && ((uintptr_t)v & 15) == 0 && ((uintptr_t)out & 15) == 0 &&
                     ((uintptr_t)out_hi & 7) == 0 && ((uintptr_t)out_lo & 7) == 0,
                 "prompt attention: alignment");
    SA_CHECK_ARG(out || (out_hi && out_lo), "prompt attention: no output");
    const long long rows_per_head = kv_head_stride / d;
    SA_CHECK_ARG(kv_rows <= (long long)hkv * rows_per_head && (hkv - 1) * rows_per_head + T0 + M - 1 <= kv_rows &&
                     kv_rows < (1ll << 31),
                 "prompt attention: %d keys of %d heads in %lld rows", T0 + M - 1, hkv, kv_rows);
    // K of every head as one [kv_rows, 128] tensor: the rows addressable from
    // k (a tile reaching past them reads zeros, never memory beyond)
    CUtensorMap tk;
    SA_RC_TRY(cached_tmap_2d_f32_sw128(&tk, k, (uint64_t)kv_rows, (uint64_t)d, (uint64_t)d, pa::KR));
    pa::Args a;
    a.q = q; a.q_stride = q_stride; a.v = v; a.kv_head_stride = kv_head_stride;
    a.T0 = T0; a.M = M; a.hq = hq; a.hkv = hkv; a.G = G; a.qb = pa::QV / G;
    a.qscale = scale * pa::LOG2E;
    a.out = out; a.o_stride = o_stride; a.out_hi = out_hi; a.out_lo = out_lo;
    a.status = status;
    const int nblk = (M + a.qb - 1) / a.qb;
    SA_CHECK_ARG(hkv <= 65535, "prompt attention: grid");
    SA_RC_TRY(set_smem_attr_once((const void*)pa::prompt_attn_kernel, pa::SMEM_BYTES));
    SA_CUDA_TRY(launch_pdl(pa::prompt_attn_kernel, dim3(nblk, hkv), dim3(pa::THREADS), pa::SMEM_BYTES, st, tk, a));
    return SA_OK;
}

}  // namespace sa
