// sa_gemm.cu -- tcgen05 GEMM for the Qwen3 projections:
//     C[M, N] = A[M, K] . W[N, K]^T        (the reference's ops::linear,
//                                           tensor_cpp/src/ops.cpp:315-369)
// with W in bf16 (the weights) and A given as two bf16 terms A = A_hi + A_lo
// (the fp32 activation split into its bf16 head and the bf16 rounding of the
// remainder), so one K-step is two MMAs and the product carries ~16 bits of
// activation mantissa: near-fp32 accuracy at tensor-core speed.
//
// Tile 128 (M) x BN (N) x 64 (K), BN in {64, 128, 256}; a TMA ring of
// 128-byte-swizzled stages; one lane issues tcgen05.mma into a BN-column TMEM
// accumulator; four warps run the epilogue.
//
// Split-K runs inside a thread-block cluster: the `s` CTAs of a cluster share
// one output tile, each accumulates a contiguous range of K blocks, parks its
// fp32 partial tile in its own shared memory, and after a cluster barrier CTA
// r sums rows [128 r / s, 128 (r + 1) / s) of all s partials through
// distributed shared memory, in rank order (deterministic), and applies the
// epilogue to those rows.  No global scratch and no single-CTA reduction.
// Prompt GEMMs have M = 128 .. a few thousand rows, so at short prompts a
// tile's weights are the only large operand: the host picks BN and s per
// shape so that one wave of clusters covers the SMs with the fewest bytes per
// CTA (weights + the activation block + the partial exchange).
//
// Epilogues:
//   STORE   C = acc                                  (fp32)
//   RESID   C += acc       (the residual stream, qwen3_ops.cpp:514,527)
//   SWIGLU  W holds [gate(32) ; up(32)] row blocks; out[:, n0/2 + i] =
//           silu(g_i) * u_i written as A_hi/A_lo of the next GEMM
//           (qwen3_mlp, qwen3_ops.cpp:265-296)
//
// Launched with programmatic stream serialization: the producer streams the
// first stages' weight tiles before griddepcontrol.wait, every other access
// to global memory comes after it.
#include <cuda_bf16.h>
#include <cmath>
#include <mutex>
#include <map>
#include <tuple>

#include "sa_internal.h"
#include "sa_tc.cuh"
#include "sa_qwen3.h"

namespace sa {
namespace gm {

constexpr int BM = 128, BK = 64, THREADS = 192, MAX_SPLIT = 8;
constexpr int A_BYTES = BM * BK * 2;          // 16 KB (one of hi / lo)

template <int BN>
struct Cfg {
    static constexpr int STAGES = BN == 256 ? 3 : 4;
    static constexpr int W_BYTES = BN * BK * 2;
    static constexpr int STAGE_BYTES = 2 * A_BYTES + W_BYTES;
    static constexpr int TP = BN + 4;                        // partial-tile row pitch (floats)
    static constexpr int T_BYTES = BM * TP * 4;
    static constexpr int PIPE = STAGES * STAGE_BYTES;
    static constexpr int OFF_BAR = ((PIPE > T_BYTES ? PIPE : T_BYTES) + 1023) / 1024 * 1024;
    static constexpr int SMEM_BYTES = OFF_BAR + 256 + 1024;  // + barriers + alignment slack
};

struct Args {
    int M, N, K;
    int mode;
    float* C;                 // STORE / RESID: [M, ldc]
    long long ldc;
    __nv_bfloat16* out_hi;    // SWIGLU: [M, ldo]
    __nv_bfloat16* out_lo;
    long long ldo;
    int* status;
};

struct Bars {
    uint64_t full[4], empty[4], done;
    uint32_t tmem_base;
    int abort;
};

__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// shared::cluster address of the same shared-memory offset in CTA `rank`
__device__ __forceinline__ uint32_t map_rank(uint32_t saddr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
    return r;
}
__device__ __forceinline__ float4 ld_dsmem4(uint32_t caddr) {
    float4 v;
    asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(caddr) : "memory");
    return v;
}

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

__device__ __forceinline__ void store_hilo4(__nv_bfloat16* hi, __nv_bfloat16* lo, float4 v) {
    const __nv_bfloat162 h01 = __floats2bfloat162_rn(v.x, v.y), h23 = __floats2bfloat162_rn(v.z, v.w);
    const float2 f01 = __bfloat1622float2(h01), f23 = __bfloat1622float2(h23);
    const __nv_bfloat162 l01 = __floats2bfloat162_rn(v.x - f01.x, v.y - f01.y);
    const __nv_bfloat162 l23 = __floats2bfloat162_rn(v.z - f23.x, v.w - f23.y);
    uint2 uh, ul;
    uh.x = *reinterpret_cast<const uint32_t*>(&h01); uh.y = *reinterpret_cast<const uint32_t*>(&h23);
    ul.x = *reinterpret_cast<const uint32_t*>(&l01); ul.y = *reinterpret_cast<const uint32_t*>(&l23);
    *reinterpret_cast<uint2*>(hi) = uh;
    *reinterpret_cast<uint2*>(lo) = ul;
}

// Sum of the s partial tiles' float4 at byte offset `off` (rank order).
__device__ __forceinline__ float4 cluster_sum4(uint32_t t_base, uint32_t off, int s) {
    float4 v[MAX_SPLIT];
#pragma unroll
    for (int z = 0; z < MAX_SPLIT; ++z)
        if (z < s) v[z] = ld_dsmem4(map_rank(t_base + off, (uint32_t)z));
    float4 acc = v[0];
#pragma unroll
    for (int z = 1; z < MAX_SPLIT; ++z)
        if (z < s) { acc.x += v[z].x; acc.y += v[z].y; acc.z += v[z].z; acc.w += v[z].w; }
    return acc;
}

template <int BN>
__global__ void __launch_bounds__(THREADS, 1)
gemm_kernel(const __grid_constant__ CUtensorMap ta_hi, const __grid_constant__ CUtensorMap ta_lo,
            const __grid_constant__ CUtensorMap tw, const Args a) {
    using C_ = Cfg<BN>;
    constexpr int STAGES = C_::STAGES, STAGE_BYTES = C_::STAGE_BYTES, TP = C_::TP;
    extern __shared__ unsigned char smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    unsigned char* sm = smem_raw + (((raw + 1023u) & ~1023u) - raw);
    Bars* B = reinterpret_cast<Bars*>(sm + C_::OFF_BAR);
    volatile int* abort = &B->abort;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int n0 = blockIdx.x * BN, m0 = blockIdx.y * BM;
    const int s = gridDim.z;                        // the cluster spans the split dimension
    const int rank = s > 1 ? (int)cluster_rank() : 0;
    const int kblocks = a.K / BK, kbase = kblocks / s, krem = kblocks % s;
    const int nkb = kbase + (rank < krem ? 1 : 0);
    const int kb0 = rank * kbase + min(rank, krem);

    if (tid == 0) {
        for (int i = 0; i < STAGES; ++i) {
            mbar_init(&B->full[i], 1);
            mbar_init(&B->empty[i], 1);
        }
        mbar_init(&B->done, 1);
        B->abort = 0;
        fence_barrier_init();
    }
    if (warp == 1) tc::tmem_alloc(&B->tmem_base, BN);
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tacc = B->tmem_base;
    pdl_trigger();

    if (warp == 0) {
        if (lane == 0) {
            tc::prefetch_tmap(&ta_hi);
            tc::prefetch_tmap(&ta_lo);
            tc::prefetch_tmap(&tw);
            // weights do not depend on the previous kernel: stream the first
            // stages' W tiles before waiting for it
            const int pre = min(STAGES, nkb);
            for (int i = 0; i < pre; ++i) {
                unsigned char* st = sm + i * STAGE_BYTES;
                mbar_arrive_expect_tx(&B->full[i], STAGE_BYTES);
                tc::tma_load_2d(st + 2 * A_BYTES, &tw, (kb0 + i) * BK, n0, &B->full[i]);
            }
            pdl_wait();
            for (int i = 0; i < pre; ++i) {
                unsigned char* st = sm + i * STAGE_BYTES;
                tc::tma_load_2d(st, &ta_hi, (kb0 + i) * BK, m0, &B->full[i]);
                tc::tma_load_2d(st + A_BYTES, &ta_lo, (kb0 + i) * BK, m0, &B->full[i]);
            }
            int issued = pre;
            for (int i = pre; i < nkb; ++i) {
                const int st_i = i % STAGES;
                if (!wait_ab(&B->empty[st_i], ((i / STAGES) & 1) ^ 1, abort, a.status)) break;
                unsigned char* st = sm + st_i * STAGE_BYTES;
                const int kx = (kb0 + i) * BK;
                mbar_arrive_expect_tx(&B->full[st_i], STAGE_BYTES);
                tc::tma_load_2d(st, &ta_hi, kx, m0, &B->full[st_i]);
                tc::tma_load_2d(st + A_BYTES, &ta_lo, kx, m0, &B->full[st_i]);
                tc::tma_load_2d(st + 2 * A_BYTES, &tw, kx, n0, &B->full[st_i]);
                issued = i + 1;
            }
            if (*abort)   // let the copies still in flight land before the CTA moves on
                for (int i = max(0, issued - STAGES); i < issued; ++i)
                    mbar_wait(&B->full[i % STAGES], (i / STAGES) & 1, nullptr);
        } else {
            pdl_wait();
        }
        __syncwarp();
    } else if (warp == 1) {
        pdl_wait();
        if (lane == 0) {
            constexpr uint32_t idesc = tc::idesc_bf16_f32(BM, BN, false, false);
            for (int i = 0; i < nkb; ++i) {
                const int st_i = i % STAGES;
                if (!wait_ab(&B->full[st_i], (i / STAGES) & 1, abort, a.status)) break;
                tc::fence_after_sync();
                const uint32_t st = smem_u32(sm + st_i * STAGE_BYTES);
#pragma unroll
                for (int kk = 0; kk < BK / 16; ++kk) {
                    const uint64_t wd = tc::sdesc_sw128(st + 2 * A_BYTES + kk * 32, 16, 1024);
                    tc::mma_bf16(tacc, tc::sdesc_sw128(st + kk * 32, 16, 1024), wd, idesc, (i > 0 || kk > 0));
                    tc::mma_bf16(tacc, tc::sdesc_sw128(st + A_BYTES + kk * 32, 16, 1024), wd, idesc, 1u);
                }
                tc::mma_commit(&B->empty[st_i]);
            }
            tc::mma_commit(&B->done);
        }
        __syncwarp();
    } else {
        // ------------------------------------------------ epilogue warps 2..5
        // accumulator: TMEM -> registers (thread = row) -> partial tile T in
        // this CTA's shared memory (the pipeline stages are idle once `done`
        // fired: every MMA, and so every load it consumed, has completed)
        pdl_wait();
        const int quad = warp & 3;
        const int row = quad * 32 + lane;
        float* T = reinterpret_cast<float*>(sm);       // [BM][TP] fp32
        const bool ok = wait_ab(&B->done, 0, abort, a.status);
        tc::fence_after_sync();
        if (ok) {
            uint32_t r[32];
#pragma unroll 1
            for (int c0 = 0; c0 < BN; c0 += 32) {
                tc::tmem_ld32(tacc + ((uint32_t)(quad * 32) << 16) + c0, r);
                tc::tmem_wait_ld();
                float4* dst = reinterpret_cast<float4*>(T + row * TP + c0);
#pragma unroll
                for (int c = 0; c < 8; ++c)
                    dst[c] = nkb > 0 ? make_float4(__uint_as_float(r[4 * c]), __uint_as_float(r[4 * c + 1]),
                                                   __uint_as_float(r[4 * c + 2]), __uint_as_float(r[4 * c + 3]))
                                     : make_float4(0.f, 0.f, 0.f, 0.f);
            }
        }
    }
    // every partial tile of the cluster is in place after this barrier
    tc::fence_before_sync();
    if (s > 1) cluster_sync_all();
    else __syncthreads();

    if (warp >= 2 && !*abort) {
        const int et = tid - 64;                       // 0..127
        const uint32_t t_base = smem_u32(sm);
        const float* T = reinterpret_cast<const float*>(sm);
        const int r0 = BM * rank / s, r1 = BM * (rank + 1) / s;
        if (a.mode == QW_EPI_SWIGLU) {
            // item = (row, 4 outputs); output j of the tile pairs gate column
            // 64 (j / 32) + j % 32 with up column 64 (j / 32) + 32 + j % 32
            constexpr int J4 = BN / 8;
            const int items = (r1 - r0) * J4;
            for (int it = et; it < items; it += 128) {
                const int rr = r0 + it / J4, j = (it % J4) * 4, m = m0 + rr;
                const int gc = (j / 32) * 64 + (j % 32);
                float4 g, u;
                if (s > 1) {
                    g = cluster_sum4(t_base, (uint32_t)(rr * TP + gc) * 4u, s);
                    u = cluster_sum4(t_base, (uint32_t)(rr * TP + gc + 32) * 4u, s);
                } else {
                    g = *reinterpret_cast<const float4*>(T + rr * TP + gc);
                    u = *reinterpret_cast<const float4*>(T + rr * TP + gc + 32);
                }
                if (m < a.M) {
                    const float4 v = make_float4(silu(g.x) * u.x, silu(g.y) * u.y, silu(g.z) * u.z, silu(g.w) * u.w);
                    const size_t o = (size_t)m * a.ldo + n0 / 2 + j;
                    store_hilo4(a.out_hi + o, a.out_lo + o, v);
                }
            }
        } else {
            constexpr int C4 = BN / 4;
            const int items = (r1 - r0) * C4, nv = a.N - n0;
            const bool vec = (a.ldc & 3) == 0;
            for (int it = et; it < items; it += 128) {
                const int rr = r0 + it / C4, c = (it % C4) * 4, m = m0 + rr;
                const float4 v = s > 1 ? cluster_sum4(t_base, (uint32_t)(rr * TP + c) * 4u, s)
                                       : *reinterpret_cast<const float4*>(T + rr * TP + c);
                if (m >= a.M || c >= nv) continue;
                float* cp = a.C + (size_t)m * a.ldc + n0 + c;
                if (vec && c + 4 <= nv) {
                    float4 o = v;
                    if (a.mode == QW_EPI_RESID) {
                        const float4 old = __ldcg(reinterpret_cast<const float4*>(cp));
                        o.x += old.x; o.y += old.y; o.z += old.z; o.w += old.w;
                    }
                    *reinterpret_cast<float4*>(cp) = o;
                } else {
                    const float vv[4] = {v.x, v.y, v.z, v.w};
                    for (int u = 0; u < 4 && c + u < nv; ++u)
                        cp[u] = a.mode == QW_EPI_RESID ? cp[u] + vv[u] : vv[u];
                }
            }
        }
    }
    // no CTA leaves (freeing its partial tile) while a peer may still read it
    tc::fence_before_sync();
    if (s > 1) cluster_sync_all();
    else __syncthreads();
    if (warp == 1) {
        tc::fence_after_sync();
        tc::tmem_dealloc(tacc, BN);
    }
}

// ---------------------------------------------------------------- planning
// Clusters of `s` CTAs of the BN variant that fit on the device at once
// (cudaOccupancyMaxActiveClusters), cached per device.
template <int BN>
int max_clusters(int device, int s) {
    static std::mutex mu;
    static std::map<std::pair<int, int>, int> cache;
    std::lock_guard<std::mutex> lk(mu);
    auto it = cache.find({device, s});
    if (it != cache.end()) return it->second;
    int n = 0;
    if (set_smem_attr_once((const void*)gemm_kernel<BN>, Cfg<BN>::SMEM_BYTES) == SA_OK) {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(1, 1, s);
        cfg.blockDim = dim3(THREADS);
        cfg.dynamicSmemBytes = Cfg<BN>::SMEM_BYTES;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = 1;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = s;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        if (cudaOccupancyMaxActiveClusters(&n, gemm_kernel<BN>, &cfg) != cudaSuccess) n = 0;
        cudaGetLastError();
    } else {
        clear_error();
    }
    cache[{device, s}] = n;
    return n;
}

int max_clusters_bn(int bn, int device, int s) {
    return bn == 64 ? max_clusters<64>(device, s) : bn == 128 ? max_clusters<128>(device, s)
                                                             : max_clusters<256>(device, s);
}

}  // namespace gm

void gemm_prepare(int device) {
    for (int bn : {64, 128, 256})
        for (int s = 1; s <= gm::MAX_SPLIT; ++s) gm::max_clusters_bn(bn, device, s);
}

// Tile width and split count for one GEMM: the fewest bytes a CTA moves per
// wave of co-resident clusters (activation block + weight tile per K block,
// plus its share of the partial-tile exchange), times the number of waves.
GemmPlan gemm_plan(int device, int M, int N, int K, int mode) {
    GemmPlan best{64, 1};
    double best_cost = 1e30;
    const int mt = (M + gm::BM - 1) / gm::BM, kb = K / gm::BK;
    for (int bn : {64, 128, 256}) {
        const int nt = (N + bn - 1) / bn;
        for (int s = 1; s <= gm::MAX_SPLIT && s <= kb; ++s) {
            const int cap = gm::max_clusters_bn(bn, device, s);
            if (cap <= 0) continue;
            const long long clusters = (long long)nt * mt;
            const long long waves = (clusters + cap - 1) / cap;
            const double kbs = (double)((kb + s - 1) / s);
            const double main_b = kbs * gm::BK * (gm::BM * 4.0 + bn * 2.0);
            const double red_b = s > 1 ? gm::BM * bn * 4.0 * (s - 1) / s : 0.0;
            const double cost = (double)waves * (main_b + red_b + 65536.0);
            if (cost < best_cost * 0.98) {
                best_cost = cost;
                best = GemmPlan{bn, s};
            }
        }
    }
    (void)mode;
    return best;
}

// C-side launcher used by the Qwen3 forward.  a_hi/a_lo: [M, K] bf16 row-major
// (lda elements per row); w: [N, K] bf16.  No scratch memory: split-K partials
// are exchanged inside the cluster.
int gemm_launch(cudaStream_t st, int* status, const __nv_bfloat16* a_hi, const __nv_bfloat16* a_lo,
                long long lda, const __nv_bfloat16* w, int M, int N, int K, int mode, float* C,
                long long ldc, __nv_bfloat16* out_hi, __nv_bfloat16* out_lo, long long ldo, GemmPlan plan) {
    SA_CHECK_ARG(M > 0 && N > 0 && K > 0 && K % gm::BK == 0, "gemm: M=%d N=%d K=%d", M, N, K);
    SA_CHECK_ARG(plan.bn == 64 || plan.bn == 128 || plan.bn == 256, "gemm: tile width %d", plan.bn);
    SA_CHECK_ARG(plan.splits >= 1 && plan.splits <= gm::MAX_SPLIT && plan.splits <= K / gm::BK,
                 "gemm: %d splits", plan.splits);
    SA_CHECK_ARG(mode != QW_EPI_SWIGLU || N % plan.bn == 0, "gemm: SwiGLU needs N %% %d == 0", plan.bn);
    SA_CHECK_ARG(mode == QW_EPI_SWIGLU ? (ldo % 4 == 0 && ((uintptr_t)out_hi & 7) == 0 && ((uintptr_t)out_lo & 7) == 0)
                                       : (((uintptr_t)C & 15) == 0),
                 "gemm: output alignment");
    const int bn = plan.bn, s = plan.splits;
    const int nt = (N + bn - 1) / bn, mt = (M + gm::BM - 1) / gm::BM;
    CUtensorMap mh, ml, mw;
    int rc = cached_tmap_2d_bf16(&mh, a_hi, (uint64_t)M, (uint64_t)K, (uint64_t)lda, gm::BM, gm::BK);
    if (!rc) rc = cached_tmap_2d_bf16(&ml, a_lo, (uint64_t)M, (uint64_t)K, (uint64_t)lda, gm::BM, gm::BK);
    if (!rc) rc = cached_tmap_2d_bf16(&mw, w, (uint64_t)N, (uint64_t)K, (uint64_t)K, (uint32_t)bn, gm::BK);
    if (rc) return rc;
    gm::Args a;
    a.M = M; a.N = N; a.K = K; a.mode = mode;
    a.C = C; a.ldc = ldc; a.out_hi = out_hi; a.out_lo = out_lo; a.ldo = ldo;
    a.status = status;
    const void* fn = bn == 64 ? (const void*)gm::gemm_kernel<64>
                   : bn == 128 ? (const void*)gm::gemm_kernel<128> : (const void*)gm::gemm_kernel<256>;
    const int smem = bn == 64 ? gm::Cfg<64>::SMEM_BYTES
                   : bn == 128 ? gm::Cfg<128>::SMEM_BYTES : gm::Cfg<256>::SMEM_BYTES;
    SA_RC_TRY(set_smem_attr_once(fn, smem));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(nt, mt, s);
    cfg.blockDim = dim3(gm::THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    int na = 0;
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = 1;
    attr[na].val.clusterDim.y = 1;
    attr[na].val.clusterDim.z = s;
    ++na;
    static const bool no_pdl = std::getenv("SA_NO_PDL") != nullptr;
    if (!no_pdl) {
        attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[na].val.programmaticStreamSerializationAllowed = 1;
        ++na;
    }
    cfg.attrs = attr;
    cfg.numAttrs = na;
    void* args[] = {(void*)&mh, (void*)&ml, (void*)&mw, (void*)&a};
    SA_CUDA_TRY(cudaLaunchKernelExC(&cfg, fn, args));
    return SA_OK;
}

}  // namespace sa
