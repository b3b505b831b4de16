// sa_gemm.cu -- tcgen05 GEMM for the Qwen3 prompt projections:
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
// Split-K: at prompt lengths of a few hundred tokens one 128-row tile per
// weight slice cannot fill 148 SMs, so gridDim.z = s CTAs share a tile, each
// accumulating a contiguous range of K blocks.  Their fp32 partial sums go to
// s stacked planes part[z][M][N] by TMA tensor stores (staged in 128-byte
// swizzled shared memory, so the TMEM -> shared writes are conflict-free),
// and the NEXT kernel adds the s planes in plane order while it reads its
// input anyway (qknorm_rope_append for QKV, the residual RMSNorm for o_proj /
// down_proj, swiglu_hilo for gate/up; sa_qwen3_kernels.cu).  So a split GEMM
// needs no cross-CTA synchronisation and the sum is deterministic.
// (Exchanging partials inside a thread-block cluster measured 20-33 GB/s per
// SM through distributed shared memory on B200; ~3-5 us per GEMM.)
//
// Epilogues of unsplit GEMMs (s = 1), through a padded shared-memory tile so
// every global access is coalesced:
//   STORE   C = acc                                  (fp32)
//   RESID   C += acc       (the residual stream, qwen3_ops.cpp:514,527)
//   SWIGLU  W holds [gate(32) ; up(32)] row blocks; out[:, n0/2 + i] =
//           silu(g_i) * u_i written as A_hi/A_lo of the next GEMM
//           (qwen3_mlp, qwen3_ops.cpp:265-296)
//   RESID_NORM  C += acc, then the next GEMM's A = hi/lo(g . C) and the
//           tile's row sums of C^2 (that GEMM's RMSNorm, deferred: it scales
//           its accumulator rows by 1 / rms, qwen3_ops.cpp:450-456,516-520)
//   QKV_ROWS    QK-norm + RoPE of whole heads and the KV-cache append
//           (qwen3_attention, qwen3_ops.cpp:341-401), fp32 and/or bf16
// and, with a deferred RMSNorm on the A operand, every mode first scales its
// accumulator rows by 1 / rms(x) (GemmEpi in sa_qwen3.h).
//
// Launched with programmatic stream serialization: the producer streams the
// first stages' weight tiles before griddepcontrol.wait, every other access
// to global memory comes after it.
#include <cuda_bf16.h>
#include <cmath>
#include <map>
#include <mutex>

#include "sa_internal.h"
#include "sa_tc.cuh"
#include "sa_qwen3.h"
#include "sa_qwen3_dev.cuh"

namespace sa {
namespace gm {

constexpr int BM = 128, BK = 64, THREADS = 192, MAX_SPLIT = 8;
constexpr int A_BYTES = BM * BK * 2;          // 16 KB (one of hi / lo)

template <int BN>
struct Cfg {
    static constexpr int STAGES = BN == 256 ? 3 : 4;
    static constexpr int W_BYTES = BN * BK * 2;
    static constexpr int STAGE_BYTES = 2 * A_BYTES + W_BYTES;
    static constexpr int TP = BN + 4;                        // padded epilogue tile row pitch (floats)
    static constexpr int T_BYTES = BM * TP * 4;
    static constexpr int PIPE = STAGES * STAGE_BYTES;
    static constexpr int RS_OFF = T_BYTES;                   // [BM] row scales of a deferred RMSNorm
    static_assert(T_BYTES + BM * 4 <= PIPE && BN * BM * 4 <= PIPE, "epilogue staging must fit in the pipeline stages");
    static constexpr int OFF_BAR = (PIPE + 1023) / 1024 * 1024;
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
    GemmEpi e;                // deferred RMSNorm, RESID_NORM and QKV_ROWS operands
    int* status;
};

struct Bars {
    uint64_t full[4], empty[4], done;
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

// QW_EPI_QKV_ROWS: warp `quad` of the four epilogue warps takes rows quad,
// quad + 4, ... four at a time: the four rows' RoPE cos/sin and tile values
// are loaded before any is used (one load latency per four rows), then each
// row's BN / 128 heads (lane l: elements 4l..4l+3 of a head) are normalised,
// rotated and stored, their reductions interleaved.
template <int BN>
__device__ __forceinline__ void qkv_rows_epilogue(const Args& a, const float* T, const float* rs, bool scaled,
                                                  int m0, int n0, int quad, int lane) {
    constexpr int HPT = BN / 128, TP = Cfg<BN>::TP, D = 128, RB = 4;
    const GemmEpi& e = a.e;
    const int nqk = e.hq + e.hkv;                  // heads [nqk, nqk + hkv) are V heads
    const int h0 = n0 / D;
    const int i0 = (4 * lane) & (D / 2 - 1);
    const bool first = lane < 16;
    float4 nw[HPT];
#pragma unroll
    for (int hh = 0; hh < HPT; ++hh) {
        const int h = h0 + hh;
        const float* w = h < e.hq ? e.qn : e.kn;
        nw[hh] = h < nqk ? __ldg(reinterpret_cast<const float4*>(w) + lane) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll 1
    for (int r0 = quad; r0 < BM; r0 += 4 * RB) {
        float4 c4[RB], s4[RB];
        float ev[RB][HPT][4];
#pragma unroll
        for (int b = 0; b < RB; ++b) {
            const int rr = r0 + 4 * b, m = m0 + rr;
            const int pos = e.pos0 + (m < a.M ? m : m0);
            c4[b] = __ldg(reinterpret_cast<const float4*>(e.cos_t + (size_t)pos * (D / 2) + i0));
            s4[b] = __ldg(reinterpret_cast<const float4*>(e.sin_t + (size_t)pos * (D / 2) + i0));
            const float sc = scaled ? rs[rr] : 1.f;
#pragma unroll
            for (int hh = 0; hh < HPT; ++hh) {
                const float4 t4 = *reinterpret_cast<const float4*>(T + rr * TP + hh * D + 4 * lane);
                ev[b][hh][0] = t4.x * sc; ev[b][hh][1] = t4.y * sc; ev[b][hh][2] = t4.z * sc; ev[b][hh][3] = t4.w * sc;
            }
        }
#pragma unroll
        for (int b = 0; b < RB; ++b) {
            const int rr = r0 + 4 * b, m = m0 + rr;
            const int pos = e.pos0 + m, row = pos + e.row_shift;
            if (m >= a.M || row >= e.max_seq) break;   // rows only grow along the loop (warp-uniform)
            float ss[HPT];
#pragma unroll
            for (int hh = 0; hh < HPT; ++hh)
                ss[hh] = ev[b][hh][0] * ev[b][hh][0] + ev[b][hh][1] * ev[b][hh][1] + ev[b][hh][2] * ev[b][hh][2] +
                         ev[b][hh][3] * ev[b][hh][3];
#pragma unroll
            for (int o = 16; o; o >>= 1)
#pragma unroll
                for (int hh = 0; hh < HPT; ++hh) ss[hh] += __shfl_xor_sync(0xffffffffu, ss[hh], o);
            const float cs[4] = {c4[b].x, c4[b].y, c4[b].z, c4[b].w}, sn[4] = {s4[b].x, s4[b].y, s4[b].z, s4[b].w};
#pragma unroll
            for (int hh = 0; hh < HPT; ++hh) {
                const int h = h0 + hh;
                if (h >= nqk) {                    // V head: the projection as it is
                    const int vh = h - nqk;
                    const float4 v4 = make_float4(ev[b][hh][0], ev[b][hh][1], ev[b][hh][2], ev[b][hh][3]);
                    if (e.vc) *reinterpret_cast<float4*>(e.vc + ((size_t)vh * e.max_seq + row) * D + 4 * lane) = v4;
                    if (e.v_bf)
                        *reinterpret_cast<uint2*>(e.v_bf + ((size_t)pos * e.hkv + vh) * D + 4 * lane) = qd::bf16x4(v4);
                    continue;
                }
                // QK-norm (eps 1e-6 inside the sqrt) with the head's gain, then
                // rotate-half RoPE: element i pairs with i + 64 (lane l ^ 16)
                const float rms = sqrtf(ss[hh] / (float)D + 1e-6f);
                const float g4[4] = {nw[hh].x, nw[hh].y, nw[hh].z, nw[hh].w};
                float y[4], p[4], o[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) y[j] = (ev[b][hh][j] / rms) * g4[j];
#pragma unroll
                for (int j = 0; j < 4; ++j) p[j] = __shfl_xor_sync(0xffffffffu, y[j], 16);
#pragma unroll
                for (int j = 0; j < 4; ++j)
                    o[j] = first ? y[j] * cs[j] + (-p[j]) * sn[j] : y[j] * cs[j] + p[j] * sn[j];
                const float4 r4 = make_float4(o[0], o[1], o[2], o[3]);
                if (h < e.hq) {
                    const size_t off = ((size_t)m * e.hq + h) * D + 4 * lane;
                    if (e.q_out) *reinterpret_cast<float4*>(e.q_out + off) = r4;
                    if (e.q_bf) *reinterpret_cast<uint2*>(e.q_bf + off) = qd::bf16x4(r4);
                } else {
                    const int kh = h - e.hq;
                    if (e.kc) *reinterpret_cast<float4*>(e.kc + ((size_t)kh * e.max_seq + row) * D + 4 * lane) = r4;
                    if (e.k_bf)
                        *reinterpret_cast<uint2*>(e.k_bf + ((size_t)pos * e.hkv + kh) * D + 4 * lane) = qd::bf16x4(r4);
                }
            }
        }
    }
}

// QW_EPI_RESID_NORM: warp `quad` takes rows quad, quad + 4, ... four at a
// time (their residual loads issued before any is used); lane l holds the
// float4 columns 4l + 128 j of the tile.  Writes C, the next GEMM's A operand
// hi/lo(g . C) and the row's sum of C^2 over the tile at rowsq_out[tile][m].
template <int BN>
__device__ __forceinline__ void resid_norm_epilogue(const Args& a, const float* T, int m0, int n0, int quad,
                                                    int lane) {
    constexpr int V4 = BN / 128, TP = Cfg<BN>::TP;
    float4 gv[V4];
#pragma unroll
    for (int j = 0; j < V4; ++j) gv[j] = __ldg(reinterpret_cast<const float4*>(a.e.g + n0 + 128 * j) + lane);
#pragma unroll 1
    for (int r0 = quad; r0 < BM; r0 += 16) {
        float4 old[4][V4];
#pragma unroll
        for (int b = 0; b < 4; ++b) {
            const int m = m0 + r0 + 4 * b;
#pragma unroll
            for (int j = 0; j < V4; ++j)
                old[b][j] = m < a.M ? __ldcg(reinterpret_cast<const float4*>(a.C + (size_t)m * a.ldc + n0 + 128 * j) +
                                             lane)
                                    : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int b = 0; b < 4; ++b) {
            const int rr = r0 + 4 * b, m = m0 + rr;
            if (m >= a.M) break;
            float ss = 0.f;
#pragma unroll
            for (int j = 0; j < V4; ++j) {
                const float4 v = *reinterpret_cast<const float4*>(T + rr * TP + 128 * j + 4 * lane);
                const float4 x = make_float4(old[b][j].x + v.x, old[b][j].y + v.y, old[b][j].z + v.z,
                                             old[b][j].w + v.w);
                *(reinterpret_cast<float4*>(a.C + (size_t)m * a.ldc + n0 + 128 * j) + lane) = x;
                ss += x.x * x.x + x.y * x.y + x.z * x.z + x.w * x.w;
                const size_t o = (size_t)m * a.ldo + n0 + 128 * j + 4 * lane;
                store_hilo4(a.out_hi + o, a.out_lo + o,
                            make_float4(x.x * gv[j].x, x.y * gv[j].y, x.z * gv[j].z, x.w * gv[j].w));
            }
            ss = qd::warp_sum(ss);
            if (lane == 0) a.e.rowsq_out[(size_t)blockIdx.x * a.M + m] = ss;
        }
    }
}

template <int BN>
__global__ void __launch_bounds__(THREADS, 1)
gemm_kernel(const __grid_constant__ CUtensorMap ta_hi, const __grid_constant__ CUtensorMap ta_lo,
            const __grid_constant__ CUtensorMap tw, const __grid_constant__ CUtensorMap tpart, const Args a) {
    using C_ = Cfg<BN>;
    constexpr int STAGES = C_::STAGES, STAGE_BYTES = C_::STAGE_BYTES, TP = C_::TP;
    extern __shared__ unsigned char smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    unsigned char* sm = smem_raw + (((raw + 1023u) & ~1023u) - raw);
    Bars* B = reinterpret_cast<Bars*>(sm + C_::OFF_BAR);
    volatile int* abort = &B->abort;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int n0 = blockIdx.x * BN, m0 = blockIdx.y * BM;
    const int s = gridDim.z, z = blockIdx.z;
    const int kblocks = a.K / BK, kbase = kblocks / s, krem = kblocks % s;
    const int nkb = kbase + (z < krem ? 1 : 0);
    const int kb0 = z * kbase + min(z, krem);

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
        // The accumulator goes TMEM -> registers (thread = row) -> shared
        // memory; the pipeline stages are idle once `done` fired (every MMA,
        // and so every load it consumed, has completed).
        pdl_wait();
        const int et = tid - 64;                       // 0..127
        const int quad = warp & 3;
        const int row = quad * 32 + lane;
        // a deferred RMSNorm's row scale (thread et: row et), while the
        // mainloop runs; the partial sums come from the previous kernel
        float my_sc = 1.f;
        if (s == 1 && a.e.rowsq_in && m0 + et < a.M) {
            float ss = 0.f;
            for (int p = 0; p < a.e.rowsq_parts; ++p) ss += __ldcg(a.e.rowsq_in + (size_t)p * a.M + m0 + et);
            my_sc = 1.f / sqrtf(ss / a.e.norm_k + a.e.eps);
        }
        const bool ok = wait_ab(&B->done, 0, abort, a.status);
        tc::fence_after_sync();
        if (s > 1) {
            // split partial: 32-column boxes of 128 rows x 128 bytes, 128-byte
            // swizzle (16-byte chunk q of row r at chunk q ^ (r % 8)), stored
            // to plane z by TMA
            if (ok) {
                // up to four 32-column TMEM loads in flight before one wait
                constexpr int G = BN / 32 < 4 ? BN / 32 : 4;
                uint32_t r[G][32];
#pragma unroll 1
                for (int j0 = 0; j0 < BN / 32; j0 += G) {
#pragma unroll
                    for (int g = 0; g < G; ++g)
                        tc::tmem_ld32(tacc + ((uint32_t)(quad * 32) << 16) + 32 * (j0 + g), r[g]);
                    tc::tmem_wait_ld();
#pragma unroll
                    for (int g = 0; g < G; ++g) {
                        unsigned char* box = sm + (j0 + g) * (BM * 128) + row * 128;
#pragma unroll
                        for (int q = 0; q < 8; ++q)
                            *reinterpret_cast<float4*>(box + ((q ^ (row & 7)) << 4)) =
                                make_float4(__uint_as_float(r[g][4 * q]), __uint_as_float(r[g][4 * q + 1]),
                                            __uint_as_float(r[g][4 * q + 2]), __uint_as_float(r[g][4 * q + 3]));
                    }
                }
                fence_proxy_async_smem();              // the boxes' writes before the tensor stores read them
            }
            asm volatile("bar.sync 1, 128;" ::: "memory");
            if (et == 0 && ok && !*abort) {
                for (int j = 0; j < BN / 32; ++j) tc::tma_store_3d(&tpart, sm + j * (BM * 128), n0 + 32 * j, m0, z);
                tc::bulk_commit_wait_read();
            }
        } else {
            float* T = reinterpret_cast<float*>(sm);   // [BM][TP] fp32
            float* rs = reinterpret_cast<float*>(sm + C_::RS_OFF);
            const bool scaled = a.e.rowsq_in != nullptr;
            if (ok && scaled) rs[et] = my_sc;
            if (ok) {
                uint32_t r[32];
#pragma unroll 1
                for (int c0 = 0; c0 < BN; c0 += 32) {
                    tc::tmem_ld32(tacc + ((uint32_t)(quad * 32) << 16) + c0, r);
                    tc::tmem_wait_ld();
                    float4* dst = reinterpret_cast<float4*>(T + row * TP + c0);
#pragma unroll
                    for (int c = 0; c < 8; ++c)
                        dst[c] = make_float4(__uint_as_float(r[4 * c]), __uint_as_float(r[4 * c + 1]),
                                             __uint_as_float(r[4 * c + 2]), __uint_as_float(r[4 * c + 3]));
                }
            }
            asm volatile("bar.sync 1, 128;" ::: "memory");
            if (ok && !*abort) {
                if (a.mode == QW_EPI_SWIGLU) {
                    // item = (row, 4 outputs); output j of the tile pairs gate
                    // column 64 (j / 32) + j % 32 with up column + 32
                    constexpr int J4 = BN / 8;
                    for (int it = et; it < BM * J4; it += 128) {
                        const int rr = it / J4, j = (it % J4) * 4, m = m0 + rr;
                        if (m >= a.M) continue;
                        const int gc = (j / 32) * 64 + (j % 32);
                        float4 g = *reinterpret_cast<const float4*>(T + rr * TP + gc);
                        float4 u = *reinterpret_cast<const float4*>(T + rr * TP + gc + 32);
                        if (scaled) {
                            const float sc = rs[rr];
                            g = make_float4(g.x * sc, g.y * sc, g.z * sc, g.w * sc);
                            u = make_float4(u.x * sc, u.y * sc, u.z * sc, u.w * sc);
                        }
                        const float4 v = make_float4(silu(g.x) * u.x, silu(g.y) * u.y, silu(g.z) * u.z,
                                                     silu(g.w) * u.w);
                        const size_t o = (size_t)m * a.ldo + n0 / 2 + j;
                        store_hilo4(a.out_hi + o, a.out_lo + o, v);
                    }
                } else if (BN >= 128 && a.mode == QW_EPI_QKV_ROWS) {   // whole heads: the host checks the width
                    if constexpr (BN >= 128) qkv_rows_epilogue<BN>(a, T, rs, scaled, m0, n0, quad, lane);
                } else if (BN >= 128 && a.mode == QW_EPI_RESID_NORM) {
                    if constexpr (BN >= 128) resid_norm_epilogue<BN>(a, T, m0, n0, quad, lane);
                } else {
                    // a warp covers one row's BN columns as float4; residual
                    // loads are issued four rows at a time before any store
                    constexpr int C4 = BN / 4;
                    const int nv = a.N - n0;
                    const bool vec = (a.ldc & 3) == 0;
                    const bool resid = a.mode == QW_EPI_RESID;
                    for (int it0 = et; it0 < BM * C4; it0 += 4 * 128) {
                        float4 old[4];
#pragma unroll
                        for (int b = 0; b < 4; ++b) {
                            const int it = it0 + b * 128, rr = it / C4, c = (it % C4) * 4, m = m0 + rr;
                            old[b] = make_float4(0.f, 0.f, 0.f, 0.f);
                            if (resid && vec && it < BM * C4 && m < a.M && c + 4 <= nv)
                                old[b] = __ldcg(reinterpret_cast<const float4*>(a.C + (size_t)m * a.ldc + n0 + c));
                        }
#pragma unroll
                        for (int b = 0; b < 4; ++b) {
                            const int it = it0 + b * 128, rr = it / C4, c = (it % C4) * 4, m = m0 + rr;
                            if (it >= BM * C4 || m >= a.M || c >= nv) continue;
                            float4 v = *reinterpret_cast<const float4*>(T + rr * TP + c);
                            if (scaled) {
                                const float sc = rs[rr];
                                v = make_float4(v.x * sc, v.y * sc, v.z * sc, v.w * sc);
                            }
                            float* cp = a.C + (size_t)m * a.ldc + n0 + c;
                            if (vec && c + 4 <= nv) {
                                float4 o = v;
                                if (resid) { o.x += old[b].x; o.y += old[b].y; o.z += old[b].z; o.w += old[b].w; }
                                *reinterpret_cast<float4*>(cp) = o;
                            } else {
                                const float vv[4] = {v.x, v.y, v.z, v.w};
                                for (int q = 0; q < 4 && c + q < nv; ++q) cp[q] = resid ? cp[q] + vv[q] : vv[q];
                            }
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
        tc::tmem_dealloc(tacc, BN);
    }
}

// CTAs of the BN variant that fit on one SM, cached per device.
template <int BN>
int ctas_per_sm(int device) {
    static std::mutex mu;
    static std::map<int, int> cache;
    std::lock_guard<std::mutex> lk(mu);
    auto it = cache.find(device);
    if (it != cache.end()) return it->second;
    int n = 0;
    if (set_smem_attr_once((const void*)gemm_kernel<BN>, Cfg<BN>::SMEM_BYTES) != SA_OK ||
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, gemm_kernel<BN>, THREADS, Cfg<BN>::SMEM_BYTES) !=
            cudaSuccess) {
        cudaGetLastError();
        clear_error();
        n = 0;
    }
    cache[device] = n;
    return n;
}

int ctas_per_sm_bn(int bn, int device) {
    return bn == 64 ? ctas_per_sm<64>(device) : bn == 128 ? ctas_per_sm<128>(device) : ctas_per_sm<256>(device);
}

}  // namespace gm

void gemm_prepare(int device) {
    for (int bn : {64, 128, 256}) gm::ctas_per_sm_bn(bn, device);
}

// Tile width and split count for one GEMM.  Cost per wave of resident CTAs =
// the bytes one CTA streams (activation block + weight tile per K block) plus,
// for split plans, the partial planes the next kernel reads back (spread over
// the SMs, charged twice: plain loads run at about half the bulk-copy rate).
// `split_ok` is false where the consumer of the output cannot add planes.
GemmPlan gemm_plan(int device, int num_sms, int M, int N, int K, bool split_ok) {
    GemmPlan best{64, 1};
    double best_cost = 1e30;
    const int mt = (M + gm::BM - 1) / gm::BM, kb = K / gm::BK;
    for (int bn : {64, 128, 256}) {
        const int per_sm = gm::ctas_per_sm_bn(bn, device);
        if (per_sm <= 0) continue;
        const int nt = (N + bn - 1) / bn;
        for (int s = 1; s <= (split_ok ? gm::MAX_SPLIT : 1) && s <= kb; ++s) {
            const long long ctas = (long long)nt * mt * s;
            const long long slots = (long long)num_sms * per_sm;
            const long long waves = (ctas + slots - 1) / slots;
            const double kbs = (double)((kb + s - 1) / s);
            const double main_b = kbs * gm::BK * (gm::BM * 4.0 + bn * 2.0);
            const double planes = s > 1 ? 2.0 * s * (double)M * N * 4.0 / num_sms : 0.0;
            const double cost = (double)waves * (main_b + 65536.0) + planes;
            if (cost < best_cost * 0.98) {
                best_cost = cost;
                best = GemmPlan{bn, s};
            }
        }
    }
    return best;
}

// C-side launcher used by the Qwen3 forward.  a_hi/a_lo: [M, K] bf16 row-major
// (lda elements per row); w: [N, K] bf16.  plan.splits > 1 writes the split
// partials to planes part[z][M][N] (part_floats >= splits * M * N) instead of
// applying `mode`.
int gemm_launch(cudaStream_t st, int* status, const __nv_bfloat16* a_hi, const __nv_bfloat16* a_lo,
                long long lda, const __nv_bfloat16* w, int M, int N, int K, int mode, float* C,
                long long ldc, __nv_bfloat16* out_hi, __nv_bfloat16* out_lo, long long ldo, GemmPlan plan,
                float* part, size_t part_floats, const GemmEpi* epi) {
    SA_CHECK_ARG(M > 0 && N > 0 && K > 0 && K % gm::BK == 0, "gemm: M=%d N=%d K=%d", M, N, K);
    SA_CHECK_ARG(plan.bn == 64 || plan.bn == 128 || plan.bn == 256, "gemm: tile width %d", plan.bn);
    SA_CHECK_ARG(plan.splits >= 1 && plan.splits <= gm::MAX_SPLIT && plan.splits <= K / gm::BK,
                 "gemm: %d splits", plan.splits);
    const bool split = plan.splits > 1;
    if (split) {
        SA_CHECK_ARG(part && ((uintptr_t)part & 15) == 0 && (size_t)plan.splits * M * N <= part_floats && N % 4 == 0,
                     "gemm: partial planes too small (%d x %d x %d)", plan.splits, M, N);
        SA_CHECK_ARG(!epi || (!epi->rowsq_in && mode != QW_EPI_RESID_NORM && mode != QW_EPI_QKV_ROWS),
                     "gemm: fused epilogues need an unsplit plan");
    } else {
        SA_CHECK_ARG(mode != QW_EPI_SWIGLU || N % plan.bn == 0, "gemm: SwiGLU needs N %% %d == 0", plan.bn);
        SA_CHECK_ARG(mode == QW_EPI_QKV_ROWS ||
                         (mode == QW_EPI_SWIGLU
                              ? (ldo % 4 == 0 && ((uintptr_t)out_hi & 7) == 0 && ((uintptr_t)out_lo & 7) == 0)
                              : (C && ((uintptr_t)C & 15) == 0)),
                     "gemm: output alignment");
        if (mode == QW_EPI_RESID_NORM)
            SA_CHECK_ARG(epi && epi->g && epi->rowsq_out && plan.bn % 128 == 0 && N % plan.bn == 0 && ldc % 4 == 0 &&
                             ldo % 4 == 0 && ((uintptr_t)out_hi & 7) == 0 && ((uintptr_t)out_lo & 7) == 0 &&
                             ((uintptr_t)epi->g & 15) == 0,
                         "gemm: RESID_NORM operands (gain, row sums, tile width %d, N %d)", plan.bn, N);
        if (mode == QW_EPI_QKV_ROWS)
            SA_CHECK_ARG(epi && plan.bn % 128 == 0 && N % plan.bn == 0 && N == (epi->hq + 2 * epi->hkv) * 128 &&
                             epi->qn && epi->kn && epi->cos_t && epi->sin_t && (epi->q_out || epi->q_bf) &&
                             (epi->kc || epi->k_bf) && (epi->vc || epi->v_bf),
                         "gemm: QKV_ROWS operands (tile width %d, N %d)", plan.bn, N);
        if (epi && epi->rowsq_in)
            SA_CHECK_ARG(epi->rowsq_parts >= 1 && epi->norm_k > 0.f && mode != QW_EPI_RESID_NORM,
                         "gemm: deferred RMSNorm operands");
    }
    const int bn = plan.bn, s = plan.splits;
    const int nt = (N + bn - 1) / bn, mt = (M + gm::BM - 1) / gm::BM;
    CUtensorMap mh, ml, mw, mp;
    int rc = cached_tmap_2d_bf16(&mh, a_hi, (uint64_t)M, (uint64_t)K, (uint64_t)lda, gm::BM, gm::BK);
    if (!rc) rc = cached_tmap_2d_bf16(&ml, a_lo, (uint64_t)M, (uint64_t)K, (uint64_t)lda, gm::BM, gm::BK);
    if (!rc) rc = cached_tmap_2d_bf16(&mw, w, (uint64_t)N, (uint64_t)K, (uint64_t)K, (uint32_t)bn, gm::BK);
    if (!rc && split) rc = cached_tmap_3d_f32_planes(&mp, part, (uint64_t)M, (uint64_t)N, (uint64_t)s);
    if (rc) return rc;
    if (!split) mp = mw;   // unused by unsplit launches
    gm::Args a;
    a.M = M; a.N = N; a.K = K; a.mode = mode;
    a.C = C; a.ldc = ldc; a.out_hi = out_hi; a.out_lo = out_lo; a.ldo = ldo;
    a.e = epi ? *epi : GemmEpi{};
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
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    static const bool no_pdl = std::getenv("SA_NO_PDL") != nullptr;
    cfg.numAttrs = no_pdl ? 0 : 1;
    void* args[] = {(void*)&mh, (void*)&ml, (void*)&mw, (void*)&mp, (void*)&a};
    SA_CUDA_TRY(cudaLaunchKernelExC(&cfg, fn, args));
    return SA_OK;
}

}  // namespace sa
