// sa_gemm.cu -- tcgen05 GEMM for the Qwen3 projections:
//     C[M, N] = A[M, K] . W[N, K]^T        (the reference's ops::linear,
//                                           tensor_cpp/src/ops.cpp:315-369)
// with W in bf16 (the weights) and A given as two bf16 terms A = A_hi + A_lo
// (the fp32 activation split into its bf16 head and the bf16 rounding of the
// remainder), so one K-step is two MMAs and the product carries ~16 bits of
// activation mantissa: near-fp32 accuracy at tensor-core speed.
//
// Tile 128 (M) x 64 (N) x 64 (K), 4-stage TMA ring (128-byte swizzle), one
// lane issues tcgen05.mma into a 64-column TMEM accumulator, four warps run
// the epilogue (TMEM -> shared memory, then coalesced global accesses).
// Split-K over gridDim.z writes fp32 partials to scratch; the last CTA of a
// tile (arrival counter) sums them in split order -- deterministic -- and
// applies the epilogue:
//   STORE   C = acc                                  (fp32)
//   RESID   C += acc       (the residual stream, qwen3_ops.cpp:514,527)
//   SWIGLU  W holds [gate(32) ; up(32)] row blocks; out[:, n0/2 + i] =
//           silu(g_i) * u_i written as A_hi/A_lo of the next GEMM
//           (qwen3_mlp, qwen3_ops.cpp:265-296)
#include <cuda_bf16.h>
#include <cmath>

#include "sa_internal.h"
#include "sa_tc.cuh"
#include "sa_qwen3.h"

namespace sa {
namespace gm {

constexpr int BM = 128, BN = 64, BK = 64, STAGES = 4, THREADS = 192;
constexpr int A_BYTES = BM * BK * 2;          // 16 KB (one of hi / lo)
constexpr int W_BYTES = BN * BK * 2;          // 8 KB
constexpr int STAGE_BYTES = 2 * A_BYTES + W_BYTES;
constexpr int OFF_BAR = STAGES * STAGE_BYTES;
constexpr int SMEM_BYTES = OFF_BAR + 256 + 1024;

struct Args {
    int M, N, K, splits, k_blocks_per_split;
    int mode;
    float* C;                 // STORE / RESID: [M, ldc]
    long long ldc;
    __nv_bfloat16* out_hi;    // SWIGLU: [M, ldo]
    __nv_bfloat16* out_lo;
    long long ldo;
    float* part;              // split partials [tiles][splits][BM*BN]
    unsigned* counters;       // [tiles]
    int* status;
};

struct Bars {
    uint64_t full[STAGES], empty[STAGES], done;
    uint32_t tmem_base;
    int abort, last;
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

__device__ __forceinline__ float silu(float g) { return g / (1.f + expf(-g)); }

__device__ __forceinline__ void store_hilo(__nv_bfloat16* hi, __nv_bfloat16* lo, float v) {
    const __nv_bfloat16 h = __float2bfloat16_rn(v);
    *hi = h;
    *lo = __float2bfloat16_rn(v - __bfloat162float(h));
}

__global__ void __launch_bounds__(THREADS, 1)
gemm_kernel(const __grid_constant__ CUtensorMap ta_hi, const __grid_constant__ CUtensorMap ta_lo,
            const __grid_constant__ CUtensorMap tw, const Args a) {
    extern __shared__ unsigned char smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    unsigned char* sm = smem_raw + (((raw + 1023u) & ~1023u) - raw);
    Bars* B = reinterpret_cast<Bars*>(sm + OFF_BAR);
    volatile int* abort = &B->abort;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int n0 = blockIdx.x * BN, m0 = blockIdx.y * BM, kz = blockIdx.z;
    const int kb0 = kz * a.k_blocks_per_split;
    const int nkb = min(a.k_blocks_per_split, (a.K + BK - 1) / BK - kb0);

    if (tid == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&B->full[s], 1);
            mbar_init(&B->empty[s], 1);
        }
        mbar_init(&B->done, 1);
        B->abort = 0;
        fence_barrier_init();
    }
    if (warp == 1) tc::tmem_alloc(&B->tmem_base, 64);
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tacc = B->tmem_base;

    if (warp == 0) {
        if (lane == 0) {
            tc::prefetch_tmap(&ta_hi);
            tc::prefetch_tmap(&ta_lo);
            tc::prefetch_tmap(&tw);
            int issued = 0;
            for (int i = 0; i < nkb; ++i) {
                const int s = i % STAGES;
                if (i >= STAGES && !wait_ab(&B->empty[s], ((i / STAGES) & 1) ^ 1, abort, a.status)) break;
                unsigned char* st = sm + s * STAGE_BYTES;
                const int kx = (kb0 + i) * BK;
                mbar_arrive_expect_tx(&B->full[s], STAGE_BYTES);
                tc::tma_load_2d(st, &ta_hi, kx, m0, &B->full[s]);
                tc::tma_load_2d(st + A_BYTES, &ta_lo, kx, m0, &B->full[s]);
                tc::tma_load_2d(st + 2 * A_BYTES, &tw, kx, n0, &B->full[s]);
                issued = i + 1;
            }
            if (*abort)
                for (int i = max(0, issued - STAGES); i < issued; ++i)
                    mbar_wait(&B->full[i % STAGES], (i / STAGES) & 1, nullptr);
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc = tc::idesc_bf16_f32(BM, BN, false, false);
            for (int i = 0; i < nkb; ++i) {
                const int s = i % STAGES;
                if (!wait_ab(&B->full[s], (i / STAGES) & 1, abort, a.status)) break;
                tc::fence_after_sync();
                const uint32_t st = smem_u32(sm + s * STAGE_BYTES);
#pragma unroll
                for (int kk = 0; kk < BK / 16; ++kk) {
                    const uint64_t wd = tc::sdesc_sw128(st + 2 * A_BYTES + kk * 32, 16, 1024);
                    tc::mma_bf16(tacc, tc::sdesc_sw128(st + kk * 32, 16, 1024), wd, idesc, (i > 0 || kk > 0));
                    tc::mma_bf16(tacc, tc::sdesc_sw128(st + A_BYTES + kk * 32, 16, 1024), wd, idesc, 1u);
                }
                tc::mma_commit(&B->empty[s]);
            }
            tc::mma_commit(&B->done);
        }
    } else {
        // ------------------------------------------------ epilogue warps 2..5
        // The accumulator tile goes TMEM -> registers (thread = row) -> shared
        // memory (the pipeline stages are idle once `done` fired), and every
        // global access after that is coalesced: a warp covers contiguous
        // columns of a row, or contiguous float4s of a split partial.
        const int et = tid - 64;                       // 0..127
        const int quad = warp & 3;
        const int row = quad * 32 + lane;
        float* T = reinterpret_cast<float*>(sm);       // [BM][TP] fp32
        constexpr int TP = BN + 1;                     // padded row: conflict-free column writes
        const bool ok = wait_ab(&B->done, 0, abort, a.status);
        tc::fence_after_sync();
        {
            uint32_t r[32];
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                tc::tmem_ld32(tacc + ((uint32_t)(quad * 32) << 16) + 32 * h, r);
                tc::tmem_wait_ld();
#pragma unroll
                for (int c = 0; c < 32; ++c) T[row * TP + 32 * h + c] = nkb > 0 ? __uint_as_float(r[c]) : 0.f;
            }
        }
        asm volatile("bar.sync 1, 128;" ::: "memory");
        const int tile = blockIdx.y * gridDim.x + blockIdx.x;
        bool finish = ok;
        if (ok && a.splits > 1) {
            // partial [BM][BN] row-major, written as 2048 float4 by 128 threads
            float4* mine = reinterpret_cast<float4*>(a.part + ((size_t)tile * a.splits + kz) * (BM * BN));
#pragma unroll 4
            for (int i = 0; i < BM * BN / 4 / 128; ++i) {
                const int e4 = i * 128 + et, rr = e4 / (BN / 4), c4 = (e4 % (BN / 4)) * 4;
                const float* t = T + rr * TP + c4;
                mine[e4] = make_float4(t[0], t[1], t[2], t[3]);
            }
            __threadfence();
            asm volatile("bar.sync 1, 128;" ::: "memory");
            if (et == 0) B->last = atomicAdd(&a.counters[tile], 1u) == (unsigned)(a.splits - 1);
            asm volatile("bar.sync 1, 128;" ::: "memory");
            finish = B->last;
            if (finish) {
                __threadfence();
                // sum the partials in split order into T
                const float4* base = reinterpret_cast<const float4*>(a.part + (size_t)tile * a.splits * (BM * BN));
                for (int i = 0; i < BM * BN / 4 / 128; i += 4) {
                    float4 sacc[4];
#pragma unroll
                    for (int u = 0; u < 4; ++u) sacc[u] = make_float4(0.f, 0.f, 0.f, 0.f);
                    for (int z = 0; z < a.splits; ++z) {
                        float4 v[4];
#pragma unroll
                        for (int u = 0; u < 4; ++u) v[u] = __ldcg(base + (size_t)z * (BM * BN / 4) + (i + u) * 128 + et);
#pragma unroll
                        for (int u = 0; u < 4; ++u) {
                            sacc[u].x += v[u].x; sacc[u].y += v[u].y; sacc[u].z += v[u].z; sacc[u].w += v[u].w;
                        }
                    }
#pragma unroll
                    for (int u = 0; u < 4; ++u) {
                        const int e4 = (i + u) * 128 + et, rr = e4 / (BN / 4), c4 = (e4 % (BN / 4)) * 4;
                        float* t = T + rr * TP + c4;
                        t[0] = sacc[u].x; t[1] = sacc[u].y; t[2] = sacc[u].z; t[3] = sacc[u].w;
                    }
                }
                if (et == 0) a.counters[tile] = 0u;
                asm volatile("bar.sync 1, 128;" ::: "memory");
            }
        }
        if (finish) {
            if (a.mode == QW_EPI_SWIGLU) {
                // 32 outputs per row: a warp writes one row's 32 consecutive bf16 pairs
                const int i0 = n0 / 2;
#pragma unroll 4
                for (int i = 0; i < BM * (BN / 2) / 128; ++i) {
                    const int e = i * 128 + et, rr = e / (BN / 2), c = e % (BN / 2), m = m0 + rr;
                    if (m < a.M) {
                        const float val = silu(T[rr * TP + c]) * T[rr * TP + BN / 2 + c];
                        store_hilo(a.out_hi + (size_t)m * a.ldo + i0 + c, a.out_lo + (size_t)m * a.ldo + i0 + c, val);
                    }
                }
            } else {
                // a warp covers one row's BN columns as float2; loads of the
                // residual are issued 8 rows at a time before any store
                const int c2 = (et & 31) * 2, nv = a.N - n0;
                const bool full = nv >= BN && (a.ldc & 1) == 0;
                for (int i = 0; i < BM * (BN / 2) / 128; i += 8) {
                    float2 old[8];
                    if (a.mode == QW_EPI_RESID) {
#pragma unroll
                        for (int u = 0; u < 8; ++u) {
                            const int rr = ((i + u) * 128 + et) / (BN / 2), m = m0 + rr;
                            old[u] = make_float2(0.f, 0.f);
                            if (m < a.M) {
                                const float* cp = a.C + (size_t)m * a.ldc + n0 + c2;
                                if (full) old[u] = __ldcg(reinterpret_cast<const float2*>(cp));
                                else {
                                    if (c2 < nv) old[u].x = __ldcg(cp);
                                    if (c2 + 1 < nv) old[u].y = __ldcg(cp + 1);
                                }
                            }
                        }
                    }
#pragma unroll
                    for (int u = 0; u < 8; ++u) {
                        const int rr = ((i + u) * 128 + et) / (BN / 2), m = m0 + rr;
                        if (m >= a.M) continue;
                        float2 v = make_float2(T[rr * TP + c2], T[rr * TP + c2 + 1]);
                        if (a.mode == QW_EPI_RESID) { v.x += old[u].x; v.y += old[u].y; }
                        float* cp = a.C + (size_t)m * a.ldc + n0 + c2;
                        if (full) *reinterpret_cast<float2*>(cp) = v;
                        else {
                            if (c2 < nv) cp[0] = v.x;
                            if (c2 + 1 < nv) cp[1] = v.y;
                        }
                    }
                }
            }
        }
    }
    tc::fence_before_sync();
    __syncthreads();
    if (warp == 1) {
        tc::fence_after_sync();
        tc::tmem_dealloc(tacc, 64);
    }
}

}  // namespace gm

// C-side launcher used by the Qwen3 forward.  a_hi/a_lo: [M, K] bf16 row-major
// (lda elements per row); w: [N, K] bf16.  Scratch for split partials and the
// per-tile counters comes from `ws` (floats) / `counters` (zeroed).
int gemm_launch(cudaStream_t st, int* status, const __nv_bfloat16* a_hi, const __nv_bfloat16* a_lo,
                long long lda, const __nv_bfloat16* w, int M, int N, int K, int mode, float* C,
                long long ldc, __nv_bfloat16* out_hi, __nv_bfloat16* out_lo, long long ldo, int splits,
                float* ws, size_t ws_floats, unsigned* counters, size_t n_counters) {
    SA_CHECK_ARG(M > 0 && N > 0 && K > 0 && K % gm::BK == 0, "gemm: M=%d N=%d K=%d", M, N, K);
    SA_CHECK_ARG(mode != QW_EPI_SWIGLU || N % gm::BN == 0, "gemm: SwiGLU needs N %% 64 == 0");
    const int kblocks = K / gm::BK;
    if (splits < 1) splits = 1;
    if (splits > kblocks) splits = kblocks;
    if (mode == QW_EPI_SWIGLU) splits = 1;
    const int kbps = (kblocks + splits - 1) / splits;
    splits = (kblocks + kbps - 1) / kbps;
    const int nt = (N + gm::BN - 1) / gm::BN, mt = (M + gm::BM - 1) / gm::BM;
    if (splits > 1) {
        SA_CHECK_ARG((size_t)nt * mt * splits * gm::BM * gm::BN <= ws_floats, "gemm: scratch too small");
        SA_CHECK_ARG((size_t)nt * mt <= n_counters, "gemm: counters too small");
    }
    CUtensorMap mh, ml, mw;
    int rc = cached_tmap_2d_bf16(&mh, a_hi, (uint64_t)M, (uint64_t)K, (uint64_t)lda, gm::BM, gm::BK);
    if (!rc) rc = cached_tmap_2d_bf16(&ml, a_lo, (uint64_t)M, (uint64_t)K, (uint64_t)lda, gm::BM, gm::BK);
    if (!rc) rc = cached_tmap_2d_bf16(&mw, w, (uint64_t)N, (uint64_t)K, (uint64_t)K, gm::BN, gm::BK);
    if (rc) return rc;
    gm::Args a;
    a.M = M; a.N = N; a.K = K; a.splits = splits; a.k_blocks_per_split = kbps; a.mode = mode;
    a.C = C; a.ldc = ldc; a.out_hi = out_hi; a.out_lo = out_lo; a.ldo = ldo;
    a.part = ws; a.counters = counters; a.status = status;
    SA_RC_TRY(set_smem_attr_once((const void*)gm::gemm_kernel, gm::SMEM_BYTES));
    gm::gemm_kernel<<<dim3(nt, mt, splits), gm::THREADS, gm::SMEM_BYTES, st>>>(mh, ml, mw, a);
    SA_CUDA_TRY(cudaGetLastError());
    return SA_OK;
}

}  // namespace sa
