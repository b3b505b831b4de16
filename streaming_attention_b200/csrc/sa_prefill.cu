// sa_prefill.cu -- causal prefill attention on the 5th-generation tensor
// cores (tcgen05 + TMEM + TMA), bf16 in, fp32 accumulation.
//
// Replaces the reference's causal prefill attention:
//   ops::self_attention (tensor_cpp/src/ops.cpp:514-641) with the causal mask
//   of create_causal_mask (qwen3_ops.cpp:240-259), and the block-wise online
//   softmax self_attention_streaming_blockwise (ops.cpp:1027-1112,1383-1450),
//   both after repeat_kv (qwen3_ops.cpp:194-234).
//
// Design (tensor-core bound: 4*hq*d*S(S+1)/2 FLOPs causal).
//  * One CTA per (128-row query tile, pair of query heads sharing a KV head).
//    The two heads' Q tiles share every K/V tile in shared memory, so GQA
//    costs one K/V load per pair, and the two softmax warpgroups alternate
//    with the tensor core (while one head's softmax runs, the MMA warp
//    computes the other head's P.V and next S).
//  * Warp roles (12 warps): warp 0 issues TMA loads (Q once; K and V tiles of
//    64 keys into a 3-stage ring, 128-byte swizzle); warp 1 owns TMEM (512
//    columns: S_A, S_B 64 columns each, O_A, O_B 128 each) and one lane issues
//    every tcgen05.mma; warps 4-7 and 8-11 are the softmax warpgroups of the
//    two heads (one thread per query row = TMEM lane).
//  * S = Q K^T: M=128, N=64, K=128 (8 MMAs of K=16), A and B K-major.
//    O += P V: M=128, N=128, K=64 (4 MMAs), A = P (bf16, written by the softmax
//    threads to shared memory in the K-major 128-byte-swizzled layout), B = V
//    MN-major (the V tile as loaded: keys x d).
//  * Online softmax in the exp2 domain (scale*log2 e folded into the scores)
//    with a lazy rescale: the running max used for the exponent only moves
//    when a row's max grows by more than 8 (2^8 headroom in P), and only then
//    is the row's O accumulator in TMEM loaded, scaled and stored back.
//  * Causal: a tile's KV range stops at the last key its last row may see;
//    only tiles crossing the diagonal are masked.  Heavy (late) query tiles
//    are scheduled first.
//  * Every mbarrier wait is bounded; a timeout sets the status word, stops all
//    roles, lets in-flight copies and MMAs land, frees TMEM and returns.
#include <cuda_bf16.h>
#include <cmath>

#include "sa_internal.h"
#include "sa_tc.cuh"

namespace sa {
namespace pf {

constexpr int BM = 128, BN = 64, D = 128;
constexpr int STAGES = 3;
constexpr int THREADS = 384;
constexpr int Q_BYTES = BM * D * 2;            // 32 KB per head
constexpr int KV_BYTES = BN * D * 2;           // 16 KB per K (or V) tile
constexpr int P_BYTES = BM * BN * 2;           // 16 KB per head
constexpr int OFF_QA = 0;
constexpr int OFF_QB = OFF_QA + Q_BYTES;
constexpr int OFF_K = OFF_QB + Q_BYTES;
constexpr int OFF_V = OFF_K + STAGES * KV_BYTES;
constexpr int OFF_PA = OFF_V + STAGES * KV_BYTES;
constexpr int OFF_PB = OFF_PA + P_BYTES;
constexpr int OFF_BAR = OFF_PB + P_BYTES;      // 196608
constexpr int SMEM_BYTES = OFF_BAR + 256 + 1024;   // + barriers + alignment slack
constexpr uint32_t TMEM_COLS = 512;
// TMEM columns: S of head x at x*64 (64 columns), O of head x at 128 + x*128
__device__ __forceinline__ uint32_t col_s(int x) { return (uint32_t)x * 64u; }
__device__ __forceinline__ uint32_t col_o(int x) { return 128u + (uint32_t)x * 128u; }
constexpr float LOG2E = 1.4426950408889634f;
constexpr float RESCALE_THRESHOLD = 8.0f;      // log2 units

struct Args {
    int Sq, Skv, q_pos0, hq, hkv, G;
    int n_qtiles, upk;          // units (head pairs or singles) per KV head
    float sl2;                  // scale * log2(e)
    void* out;
    long long o_tok, o_head;    // element strides of out
    int out_bf16;
    int* status;
};

struct Bars {
    uint64_t q_full;
    uint64_t k_full[STAGES], v_full[STAGES], kv_empty[STAGES];
    uint64_t s_full[2], p_full[2], o_full[2];
    uint64_t drain;
    uint32_t tmem_base;
    int abort;
};

__device__ __forceinline__ bool wait_ab(uint64_t* bar, uint32_t parity, volatile int* abort, int* status) {
    if (mbar_try_wait(bar, parity)) return true;
    const unsigned long long t0 = globaltimer();
    while (!mbar_try_wait(bar, parity)) {
        if (*abort) return false;
        if (globaltimer() - t0 > kWaitLimitNs) {
            *abort = 1;
            atomicExch(status, SA_STATUS_TIMEOUT);
            return false;
        }
    }
    return true;
}

__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
}

__global__ void __launch_bounds__(THREADS, 1)
prefill_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
               const __grid_constant__ CUtensorMap tv, const Args a) {
    extern __shared__ unsigned char smem_raw[];
    // 1024-byte alignment for the 128-byte-swizzled operand tiles
    const uint32_t raw = smem_u32(smem_raw);
    unsigned char* sm = smem_raw + (((raw + 1023u) & ~1023u) - raw);
    Bars* B = reinterpret_cast<Bars*>(sm + OFF_BAR);
    volatile int* abort = &B->abort;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const bool paired = a.G >= 2;
    const int per_tile = a.hkv * a.upk;
    const int qt = a.n_qtiles - 1 - (int)blockIdx.x / per_tile;     // heavy tiles first
    const int r = (int)blockIdx.x % per_tile;
    const int kvh = r / a.upk, pair = r % a.upk;
    const int hA = paired ? kvh * a.G + 2 * pair : kvh;
    const int q0 = qt * BM;
    const int last_row = min(q0 + BM - 1, a.Sq - 1);
    const int last_key = min(a.Skv - 1, a.q_pos0 + last_row);
    const int n_kv = last_key / BN + 1;

    if (tid == 0) {
        mbar_init(&B->q_full, 1);
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&B->k_full[s], 1);
            mbar_init(&B->v_full[s], 1);
            mbar_init(&B->kv_empty[s], 1);
        }
        for (int x = 0; x < 2; ++x) {
            mbar_init(&B->s_full[x], 1);
            mbar_init(&B->p_full[x], 128);
            mbar_init(&B->o_full[x], 1);
        }
        mbar_init(&B->drain, 1);
        B->abort = 0;
        fence_barrier_init();
    }
    if (warp == 1) tc::tmem_alloc(&B->tmem_base, TMEM_COLS);
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tbase = B->tmem_base;

    if (warp == 0) {
        // ------------------------------------------------ TMA producer
        if (lane == 0) {
            tc::prefetch_tmap(&tq);
            tc::prefetch_tmap(&tk);
            tc::prefetch_tmap(&tv);
            mbar_arrive_expect_tx(&B->q_full, (paired ? 2 : 1) * Q_BYTES);
            for (int kb = 0; kb < 2; ++kb) {
                tc::tma_load_2d(sm + OFF_QA + kb * (Q_BYTES / 2), &tq, hA * D + kb * 64, q0, &B->q_full);
                if (paired)
                    tc::tma_load_2d(sm + OFF_QB + kb * (Q_BYTES / 2), &tq, (hA + 1) * D + kb * 64, q0,
                                    &B->q_full);
            }
            int issued = 0;
            for (int j = 0; j < n_kv; ++j) {
                const int s = j % STAGES;
                if (j >= STAGES && !wait_ab(&B->kv_empty[s], ((j / STAGES) & 1) ^ 1, abort, a.status)) break;
                mbar_arrive_expect_tx(&B->k_full[s], KV_BYTES);
                for (int kb = 0; kb < 2; ++kb)
                    tc::tma_load_2d(sm + OFF_K + s * KV_BYTES + kb * (KV_BYTES / 2), &tk, kvh * D + kb * 64,
                                    j * BN, &B->k_full[s]);
                mbar_arrive_expect_tx(&B->v_full[s], KV_BYTES);
                for (int kb = 0; kb < 2; ++kb)
                    tc::tma_load_2d(sm + OFF_V + s * KV_BYTES + kb * (KV_BYTES / 2), &tv, kvh * D + kb * 64,
                                    j * BN, &B->v_full[s]);
                issued = j + 1;
            }
            if (*abort) {
                // let the loads still in flight land before the CTA exits
                mbar_wait(&B->q_full, 0, nullptr);
                for (int j = max(0, issued - STAGES); j < issued; ++j) {
                    mbar_wait(&B->k_full[j % STAGES], (j / STAGES) & 1, nullptr);
                    mbar_wait(&B->v_full[j % STAGES], (j / STAGES) & 1, nullptr);
                }
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------ MMA issuer
        if (lane == 0) {
            constexpr uint32_t idS = tc::idesc_bf16_f32(BM, BN, false, false);
            constexpr uint32_t idO = tc::idesc_bf16_f32(BM, D, false, true);
            const uint32_t sQ[2] = {smem_u32(sm + OFF_QA), smem_u32(sm + OFF_QB)};
            const uint32_t sP[2] = {smem_u32(sm + OFF_PA), smem_u32(sm + OFF_PB)};
            const uint32_t sK = smem_u32(sm + OFF_K), sV = smem_u32(sm + OFF_V);
            auto issue_S = [&](int x, int s) {
#pragma unroll
                for (int kk = 0; kk < D / 16; ++kk) {
                    const uint64_t ad = tc::sdesc_sw128(sQ[x] + (kk >> 2) * (Q_BYTES / 2) + (kk & 3) * 32, 16, 1024);
                    const uint64_t bd = tc::sdesc_sw128(sK + s * KV_BYTES + (kk >> 2) * (KV_BYTES / 2) + (kk & 3) * 32,
                                                        16, 1024);
                    tc::mma_bf16(tbase + col_s(x), ad, bd, idS, kk > 0);
                }
            };
            auto issue_PV = [&](int x, int s, bool acc) {
#pragma unroll
                for (int kk = 0; kk < BN / 16; ++kk) {
                    const uint64_t ad = tc::sdesc_sw128(sP[x] + kk * 32, 16, 1024);
                    const uint64_t bd = tc::sdesc_sw128(sV + s * KV_BYTES + kk * 2048, KV_BYTES / 2, 1024);
                    tc::mma_bf16(tbase + col_o(x), ad, bd, idO, (acc || kk > 0) ? 1u : 0u);
                }
            };
            bool ok = wait_ab(&B->q_full, 0, abort, a.status);
            tc::fence_after_sync();
            for (int j = 0; ok && j < n_kv; ++j) {
                const int s = j % STAGES;
                const uint32_t ph = (j / STAGES) & 1;
                if (j == 0) {
                    if (!(ok = wait_ab(&B->k_full[s], ph, abort, a.status))) break;
                    tc::fence_after_sync();
                    issue_S(0, s);
                    tc::mma_commit(&B->s_full[0]);
                    if (paired) {
                        issue_S(1, s);
                        tc::mma_commit(&B->s_full[1]);
                    }
                }
                if (!(ok = wait_ab(&B->v_full[s], ph, abort, a.status))) break;
                if (!(ok = wait_ab(&B->p_full[0], j & 1, abort, a.status))) break;
                tc::fence_after_sync();
                issue_PV(0, s, j > 0);
                const int s2 = (j + 1) % STAGES;
                if (j + 1 < n_kv) {
                    if (!(ok = wait_ab(&B->k_full[s2], ((j + 1) / STAGES) & 1, abort, a.status))) break;
                    tc::fence_after_sync();
                    issue_S(0, s2);
                    tc::mma_commit(&B->s_full[0]);
                } else {
                    tc::mma_commit(&B->o_full[0]);
                }
                if (paired) {
                    if (!(ok = wait_ab(&B->p_full[1], j & 1, abort, a.status))) break;
                    tc::fence_after_sync();
                    issue_PV(1, s, j > 0);
                }
                tc::mma_commit(&B->kv_empty[s]);
                if (paired) {
                    if (j + 1 < n_kv) {
                        issue_S(1, s2);
                        tc::mma_commit(&B->s_full[1]);
                    } else {
                        tc::mma_commit(&B->o_full[1]);
                    }
                }
            }
            // all issued MMAs complete before TMEM is released
            tc::mma_commit(&B->drain);
            mbar_wait(&B->drain, 0, nullptr);
        }
    } else if (warp >= 4) {
        // ------------------------------------------------ softmax warpgroups
        const int x = (warp >= 8) ? 1 : 0;
        if (x == 0 || paired) {
            const int h = hA + x;
            const int row = (warp & 3) * 32 + lane;
            const uint32_t lane_addr = tbase + ((uint32_t)((warp & 3) * 32) << 16);
            const int qrow = q0 + row;
            const int limit = a.q_pos0 + qrow;          // last visible key of this row
            unsigned char* P = sm + (x ? OFF_PB : OFF_PA);
            unsigned char* prow = P + (row >> 3) * 1024 + (row & 7) * 128;
            float m = -INFINITY, l = 0.f;
            bool ok = true;
            for (int j = 0; j < n_kv; ++j) {
                if (!(ok = wait_ab(&B->s_full[x], j & 1, abort, a.status))) break;
                tc::fence_after_sync();
                uint32_t r0[32], r1[32];
                tc::tmem_ld32(lane_addr + col_s(x), r0);
                tc::tmem_ld32(lane_addr + col_s(x) + 32, r1);
                tc::tmem_wait_ld();
                float s[BN];
#pragma unroll
                for (int c = 0; c < 32; ++c) {
                    s[c] = __uint_as_float(r0[c]) * a.sl2;
                    s[32 + c] = __uint_as_float(r1[c]) * a.sl2;
                }
                const int k0 = j * BN;
                if (k0 + BN - 1 > a.q_pos0 + q0 || k0 + BN > a.Skv) {
#pragma unroll
                    for (int c = 0; c < BN; ++c)
                        if (k0 + c > limit || k0 + c >= a.Skv) s[c] = -INFINITY;
                }
                float mx = s[0];
#pragma unroll
                for (int c = 1; c < BN; ++c) mx = fmaxf(mx, s[c]);
                float alpha = 1.f;
                if (mx > m + RESCALE_THRESHOLD || (m == -INFINITY && mx != -INFINITY)) {
                    const float mn = fmaxf(mx, m);
                    alpha = (m == -INFINITY) ? 0.f : ex2(m - mn);
                    m = mn;
                }
                const float mref = (m == -INFINITY) ? 0.f : m;
                float ps = 0.f;
#pragma unroll
                for (int c = 0; c < BN; ++c) {
                    s[c] = ex2(s[c] - mref);
                    ps += s[c];
                }
                l = l * alpha + ps;
                // rescale this row's O accumulator (warp-collective TMEM access)
                if (j > 0 && __any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll 1
                    for (int cb = 0; cb < D / 32; ++cb) {
                        uint32_t o[32];
                        tc::tmem_ld32(lane_addr + col_o(x) + cb * 32, o);
                        tc::tmem_wait_ld();
#pragma unroll
                        for (int c = 0; c < 32; ++c) o[c] = __float_as_uint(__uint_as_float(o[c]) * alpha);
                        tc::tmem_st32(lane_addr + col_o(x) + cb * 32, o);
                    }
                    tc::tmem_wait_st();
                }
                // P row (bf16) into the K-major 128-byte-swizzled operand layout
#pragma unroll
                for (int c = 0; c < 8; ++c) {
                    uint4 v;
                    v.x = pack_bf16(s[c * 8 + 0], s[c * 8 + 1]);
                    v.y = pack_bf16(s[c * 8 + 2], s[c * 8 + 3]);
                    v.z = pack_bf16(s[c * 8 + 4], s[c * 8 + 5]);
                    v.w = pack_bf16(s[c * 8 + 6], s[c * 8 + 7]);
                    *reinterpret_cast<uint4*>(prow + ((c ^ (row & 7)) << 4)) = v;
                }
                fence_proxy_async_smem();
                tc::fence_before_sync();
                mbar_arrive(&B->p_full[x]);
            }
            if (ok && wait_ab(&B->o_full[x], 0, abort, a.status)) {
                tc::fence_after_sync();
                const float inv = l > 0.f ? 1.f / l : 0.f;
                const bool store = qrow < a.Sq;
#pragma unroll 1
                for (int cb = 0; cb < D / 32; ++cb) {
                    uint32_t o[32];
                    tc::tmem_ld32(lane_addr + col_o(x) + cb * 32, o);
                    tc::tmem_wait_ld();
                    if (!store) continue;
                    if (a.out_bf16) {
                        __nv_bfloat16* dst = static_cast<__nv_bfloat16*>(a.out) + (size_t)qrow * a.o_tok +
                                             (size_t)h * a.o_head + cb * 32;
#pragma unroll
                        for (int c = 0; c < 32; c += 8) {
                            uint4 v;
                            v.x = pack_bf16(__uint_as_float(o[c]) * inv, __uint_as_float(o[c + 1]) * inv);
                            v.y = pack_bf16(__uint_as_float(o[c + 2]) * inv, __uint_as_float(o[c + 3]) * inv);
                            v.z = pack_bf16(__uint_as_float(o[c + 4]) * inv, __uint_as_float(o[c + 5]) * inv);
                            v.w = pack_bf16(__uint_as_float(o[c + 6]) * inv, __uint_as_float(o[c + 7]) * inv);
                            *reinterpret_cast<uint4*>(dst + c) = v;
                        }
                    } else {
                        float* dst = static_cast<float*>(a.out) + (size_t)qrow * a.o_tok + (size_t)h * a.o_head +
                                     cb * 32;
#pragma unroll
                        for (int c = 0; c < 32; c += 4)
                            *reinterpret_cast<float4*>(dst + c) =
                                make_float4(__uint_as_float(o[c]) * inv, __uint_as_float(o[c + 1]) * inv,
                                            __uint_as_float(o[c + 2]) * inv, __uint_as_float(o[c + 3]) * inv);
                    }
                }
            }
        }
    }
    tc::fence_before_sync();
    __syncthreads();
    if (warp == 1) {
        tc::fence_after_sync();
        tc::tmem_dealloc(tbase, TMEM_COLS);
    }
}

}  // namespace pf

// Launch the causal prefill on device pointers.
//   q   [Sq,  q_tok stride,  hq heads of 128]   bf16
//   k,v [Skv, kv_tok stride, hkv heads of 128]  bf16
//   out [Sq,  o_tok stride,  hq heads of 128]   fp32 or bf16
static int launch_prefill(sa_ctx* ctx, const void* q, const void* k, const void* v, void* out, int out_dtype,
                          int Sq, int Skv, int q_pos0, int hq, int hkv, long long q_tok, long long kv_tok,
                          long long o_tok, float scale) {
    CUtensorMap mq, mk, mv;
    int rc = make_tmap_2d_bf16(&mq, q, (uint64_t)Sq, (uint64_t)hq * pf::D, (uint64_t)q_tok, pf::BM, 64);
    if (!rc) rc = make_tmap_2d_bf16(&mk, k, (uint64_t)Skv, (uint64_t)hkv * pf::D, (uint64_t)kv_tok, pf::BN, 64);
    if (!rc) rc = make_tmap_2d_bf16(&mv, v, (uint64_t)Skv, (uint64_t)hkv * pf::D, (uint64_t)kv_tok, pf::BN, 64);
    if (rc) return rc;
    pf::Args a;
    a.Sq = Sq; a.Skv = Skv; a.q_pos0 = q_pos0; a.hq = hq; a.hkv = hkv; a.G = hq / hkv;
    a.n_qtiles = (Sq + pf::BM - 1) / pf::BM;
    a.upk = a.G >= 2 ? a.G / 2 : 1;
    a.sl2 = scale * pf::LOG2E;
    a.out = out; a.o_tok = o_tok; a.o_head = pf::D;
    a.out_bf16 = out_dtype == SA_BF16;
    a.status = ctx->status;
    SA_CUDA_TRY(cudaFuncSetAttribute(pf::prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     pf::SMEM_BYTES));
    const int grid = a.n_qtiles * hkv * a.upk;
    pf::prefill_kernel<<<grid, pf::THREADS, pf::SMEM_BYTES, ctx->stream>>>(mq, mk, mv, a);
    SA_CUDA_TRY(cudaGetLastError());
    return SA_OK;
}

}  // namespace sa

SA_API int sa_attn_prefill(sa_ctx* ctx, const void* q, const void* k, const void* v, int Sq, int Skv,
                           int q_pos0, int d, int hq, int hkv, long long q_tok_stride,
                           long long kv_tok_stride, float scale, void* out, int out_dtype,
                           long long o_tok_stride, unsigned flags) {
    using namespace sa;
    clear_error();
    SA_CHECK_ARG(ctx != nullptr, "sa_attn_prefill: ctx is NULL");
    SA_CHECK_ARG(q && k && v && out, "sa_attn_prefill: null pointer");
    SA_CHECK_ARG(d == 128, "sa_attn_prefill: d = %d (the tensor-core path is built for d = 128)", d);
    SA_CHECK_ARG(Sq >= 1 && Skv >= 1 && q_pos0 >= 0, "sa_attn_prefill: Sq=%d Skv=%d q_pos0=%d", Sq, Skv, q_pos0);
    SA_CHECK_ARG(q_pos0 + Sq <= Skv, "sa_attn_prefill: queries [%d, %d) need keys beyond Skv=%d", q_pos0,
                 q_pos0 + Sq, Skv);
    SA_CHECK_ARG(hkv > 0 && hq % hkv == 0, "sa_attn_prefill: hq=%d hkv=%d", hq, hkv);
    const int G = hq / hkv;
    SA_CHECK_ARG(G == 1 || G % 2 == 0, "sa_attn_prefill: hq/hkv = %d (1 or even)", G);
    SA_CHECK_ARG(out_dtype == SA_F32 || out_dtype == SA_BF16, "sa_attn_prefill: out_dtype %d", out_dtype);
    SA_CHECK_ARG(q_tok_stride >= (long long)hq * d && kv_tok_stride >= (long long)hkv * d &&
                 o_tok_stride >= (long long)hq * d, "sa_attn_prefill: token strides too small");
    SA_CHECK_ARG(((uintptr_t)out & 15) == 0, "sa_attn_prefill: out not 16-byte aligned");
    SA_CHECK_ARG(!(flags & SA_HOST_PTRS), "sa_attn_prefill: host pointers are not supported (pass device memory)");
    DeviceGuard guard(ctx->device);
    return launch_prefill(ctx, q, k, v, out, out_dtype, Sq, Skv, q_pos0, hq, hkv, q_tok_stride, kv_tok_stride,
                          o_tok_stride, scale);
}
