// sa_decode.cu -- single-query (decode) streaming attention on B200.
//
// Replaces the reference's online-softmax block attention
// (attention/src/streaming_serial.cpp:20-71, streaming_omp.cpp:99-154,
// streaming_mpi.cpp:252-309; softmax update utils/softmax_online.h:40-87) and
// the decode attention of qwen3_decoder_layer_with_cache
// (tensor_cpp/src/qwen3_ops.cpp:860-900).
//
// Design (HBM-bound: every K/V byte is read exactly once).
//  * Grid = (KV splits, KV heads).  Each CTA owns one contiguous slice of the
//    sequence of one KV head and serves all G = hq/hkv query heads that share
//    it, so GQA never re-reads K/V.  Split counts fill 2 CTAs per SM.
//  * One producer warp streams the slice through shared memory with 1-D bulk
//    copies (cp.async.bulk, TMA engine) into a 3-stage mbarrier ring of 32 KB
//    (K+V) stages, with an L2 evict-first hint (the data is used once).
//  * Four consumer warps split each stage's rows.  Inside a warp, 8-lane groups
//    each own one row at a time; a lane holds D/8 columns of q (pre-scaled by
//    scale*log2 e) and of the output accumulator.  Scores are reduced with
//    three xor-shuffles; the (m, l, O) online-softmax recurrence runs per group
//    in the exp2 domain with an unnormalised O (normalised once at the end).
//  * States are combined across groups (shuffles) and warps (shared memory);
//    each CTA writes its (m, l, O/l) split partial, and the last CTA of a KV
//    head to finish (atomic arrival counter) merges all splits -- the
//    associative merge of streaming_omp.cpp:27-48 -- so a call is one launch.
#include <cuda_bf16.h>
#include <algorithm>
#include <cmath>

#include "sa_decode_plan.h"
#include "sa_internal.h"
#include "sa_ptx.cuh"
#include "sa_qwen3.h"
#include "sa_tc.cuh"

namespace sa {
namespace dec {

constexpr int NW = 4;                      // consumer warps
constexpr int THREADS = (NW + 1) * 32;     // + one producer warp
constexpr int STAGE_BYTES = 32768;         // K + V bytes per stage
constexpr int STAGES = 3;                  // ring depth of the general kernel (2 CTAs per SM)
constexpr int DEV_STAGES = 6;              // the decode step's kernel: 192 cached rows in flight
template <int NST>
constexpr int smem_bytes() { return NST * STAGE_BYTES + 2 * NST * 8 + 16; }
constexpr int SMEM_BYTES = smem_bytes<STAGES>();
constexpr int MAX_SPLITS = 1024;
constexpr float LOG2E = 1.4426950408889634f;
constexpr float LN2 = 0.6931471805599453f;

// Sequence-parallel exchange of one launch (world > 1): every rank holds a
// contiguous slice of the sequence and runs this kernel on it; the merging
// CTA of each KV head sends that head's (m, L, O/L) states as self-validating
// words to every rank's word area and merges all ranks' states, in rank
// order, into the output -- the Gather + merge of
// streaming_attention_mpi_simple (attention/src/streaming_mpi.cpp:252-309),
// with every rank ending up with the result.
constexpr int SP_MAX = 8;
struct SpArgs {
    int rank, world;
    // word areas of every rank (own at [rank]), each [2 slots][world][hq][d+2]:
    // per source rank and query head d words of O/L, then m (log2 domain), L
    unsigned long long* words[SP_MAX];
    unsigned* seq;    // this rank's instance count: slot = seq & 1, epoch = seq + 1
    unsigned* done;   // merging CTAs of this launch that finished (the last re-arms it)
};

struct Args {
    const void* q;
    const void* k;
    const void* v;
    long long kv_head_stride;   // elements between KV heads
    int T, hq, hkv;
    int rows_per_split, n_splits;
    float qscale;               // scale * log2(e)
    float* part_m;              // [hq][n_splits]  (log2 domain)
    float* part_l;              // [hq][n_splits]
    float* part_o;              // [hq][n_splits][D] normalised by l
    unsigned* counters;         // [hkv] arrival counters, zero between launches
    float* out;                 // [hq][D]
    float* out_m;               // optional [hq], natural-log domain
    float* out_l;               // optional [hq]
    int* status;
    // multi-query launches (gridDim.z > 1): query z reads q + z*q_stride,
    // attends rows [0, T + z*q_causal), at most rows_per_split, and writes
    // out + z*o_stride (n_splits == 1)
    long long q_stride, o_stride;
    int q_causal;
    // K and V are not written by the kernel before this one (SA_KV_STATIC):
    // launched programmatically, the producer streams the first ring stages
    // before griddepcontrol.wait; q and every global write come after it
    int kv_early;
    // when set, the row count is read on the device: T = *len_dev + 1 (the
    // KV-cache length before the token being decoded, plus that token), so a
    // captured launch stays valid as the cache grows
    const int* len_dev;
    SpArgs sp;                  // sp.world > 1: sequence-parallel exchange after the merge
};

// Unpack one 16-byte chunk into VEC floats.
template <typename KT> struct Chunk;
template <> struct Chunk<float> {
    static constexpr int VEC = 4;
    static __device__ __forceinline__ void load(const void* p, float* f) {
        float4 r = *reinterpret_cast<const float4*>(p);
        f[0] = r.x; f[1] = r.y; f[2] = r.z; f[3] = r.w;
    }
    // global memory written by a kernel that may still be draining (programmatic launch)
    static __device__ __forceinline__ void load_cg(const void* p, float* f) {
        float4 r = __ldcg(reinterpret_cast<const float4*>(p));
        f[0] = r.x; f[1] = r.y; f[2] = r.z; f[3] = r.w;
    }
};
template <> struct Chunk<__nv_bfloat16> {
    static constexpr int VEC = 8;
    static __device__ __forceinline__ void unpack(uint4 r, float* f) {
        const uint32_t w[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            f[2 * i] = __uint_as_float(w[i] << 16);
            f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
        }
    }
    static __device__ __forceinline__ void load(const void* p, float* f) {
        unpack(*reinterpret_cast<const uint4*>(p), f);
    }
    static __device__ __forceinline__ void load_cg(const void* p, float* f) {
        unpack(__ldcg(reinterpret_cast<const uint4*>(p)), f);
    }
};

template <typename KT, int D>
struct Shape {
    static constexpr int ELT = sizeof(KT);
    static constexpr int ROW_BYTES = D * ELT;
    static constexpr int STAGE_ROWS = STAGE_BYTES / (2 * ROW_BYTES);
    static constexpr int RW = STAGE_ROWS / NW;   // rows per warp per stage
    static constexpr int NR = RW / 4;            // rows per 8-lane group per stage
    static constexpr int VEC = Chunk<KT>::VEC;
    static constexpr int CPL = D / 8;            // columns per lane
    static constexpr int CH = CPL / VEC;         // 16-byte chunks per lane per row
    static_assert(NR >= 1 && CH >= 1, "tile shape");
};

// Fold state (m2, l2, o2) into (m, l, o); exp2 domain, unnormalised o.
__device__ __forceinline__ void combine_weights(float m, float m2, float& a, float& b, float& M) {
    M = fmaxf(m, m2);
    a = (m == -INFINITY) ? 0.f : ex2(m - M);
    b = (m2 == -INFINITY) ? 0.f : ex2(m2 - M);
}

// Shared-memory offsets of the final states [G][D+2] a sequence-parallel
// launch exchanges (at most (G*D + 2G) * 4 <= 2112 bytes, G*D <= 512) and
// of the sources' (m, L) (2 * G * world <= 128 floats): past the cross-warp
// reduction (NW*G*D floats) and the split weights of the merge
// (G*MAX_SPLITS + 2G floats), inside the stage ring (>= 96 KB).
constexpr int FIN_OFF = 64 * 1024;
constexpr int ML_OFF = FIN_OFF + 4096;
static_assert(FIN_OFF >= (8 * MAX_SPLITS + 2 * 8) * 4 && FIN_OFF >= NW * 512 * 4 &&
              ML_OFF + 2 * 8 * SP_MAX * 4 <= STAGES * STAGE_BYTES,
              "exchange buffers inside the stage ring, past the reduction scratch");

// The merging CTA of KV head kvh has the final (O/L, m, L) of its G query
// heads in fin[G][D+2]; send them to every rank, wait for every rank's,
// merge them in rank order and write out (and out_m / out_l).  The last
// merging CTA of the launch advances the instance count.  Two slots
// alternate: a rank writes instance i+2 into slot i&1 of a peer only after
// it has read that peer's instance i+1 words, which the peer sends after its
// launch i -- and so all its reads of slot i&1 -- completed.
template <int G, int D>
__device__ void sp_exchange(const Args& a, int kvh, const float* fin, float* ml) {
    constexpr int RW = D + 2;
    const SpArgs& s = a.sp;
    const int W = s.world, tid = threadIdx.x;
    const unsigned inst = __ldcg(s.seq);
    const int slot = (int)(inst & 1u);
    const unsigned epoch = inst + 1u;
    const size_t src_stride = (size_t)a.hq * RW;
    // send: consecutive threads store consecutive words of one destination
    for (int idx = tid; idx < W * G * RW; idx += THREADS) {
        const int r = idx / (G * RW), rem = idx - r * (G * RW);
        const int g = rem / RW, c = rem - g * RW;
        unsigned long long* dst = s.words[r] + ((size_t)slot * W + s.rank) * src_stride +
                                  (size_t)(kvh * G + g) * RW + c;
        st_u64_relaxed_sys(dst, epoch_word(epoch, fin[g * RW + c]));
    }
    // receive the sources' (m, L), then each output column from every source
    const unsigned long long* own = s.words[s.rank] + (size_t)slot * W * src_stride;
    for (int idx = tid; idx < G * W; idx += THREADS) {
        const int g = idx / W, src = idx - g * W;
        const unsigned long long* p = own + src * src_stride + (size_t)(kvh * G + g) * RW + D;
        ml[2 * idx] = wait_epoch_word(p, epoch, a.status);
        ml[2 * idx + 1] = wait_epoch_word(p + 1, epoch, a.status);
    }
    __syncthreads();
    for (int idx = tid; idx < G * D; idx += THREADS) {
        const int g = idx / D, col = idx - g * D;
        const int h = kvh * G + g;
        float M = -INFINITY;
        for (int src = 0; src < W; ++src) M = fmaxf(M, ml[2 * (g * W + src)]);
        float L = 0.f, O = 0.f;
        for (int src = 0; src < W; ++src) {
            const float ms = ml[2 * (g * W + src)];
            const float wt = (ms == -INFINITY) ? 0.f : ml[2 * (g * W + src) + 1] * ex2(ms - M);
            const float o = wait_epoch_word(own + src * src_stride + (size_t)h * RW + col, epoch, a.status);
            L += wt;
            O = fmaf(wt, o, O);
        }
        const bool failed = *reinterpret_cast<volatile int*>(a.status) != 0;
        a.out[(size_t)h * D + col] = failed ? nanf("") : (L > 0.f ? O / L : 0.f);
        if (col == 0 && a.out_m) {
            a.out_m[h] = L > 0.f ? M * LN2 : -INFINITY;
            a.out_l[h] = L > 0.f ? L : 1.f;
        }
    }
    __syncthreads();
    if (tid == 0) {
        __threadfence();
        if (atomicAdd(s.done, 1u) == (unsigned)(a.hkv - 1)) {
            *s.done = 0u;
            __stcg(s.seq, inst + 1u);
        }
    }
}

template <typename KT, int D, int G, int NST = STAGES>
__global__ void __launch_bounds__(THREADS, NST <= 3 ? 2 : 1) decode_kernel(const Args a) {
    using S = Shape<KT, D>;
    constexpr int SR = S::STAGE_ROWS, RB = S::ROW_BYTES, CPL = S::CPL, CH = S::CH, VEC = S::VEC;
    constexpr int DYN_ROWS = 8 * SR;   // rows per CTA when the length is read on the device

    pdl_trigger();
    // Launched inside the captured decode step (a.len_dev set), the kernel
    // plans its split from the cache length and streams the rows cached by
    // earlier steps before griddepcontrol.wait: the length and those rows
    // were written before the step's first kernel, an ordinary (not
    // programmatic) launch, so they are complete and visible here; only the
    // newest row (appended by the QKV kernel this kernel follows) and q need
    // the wait.  With kv_early the same holds for all of K and V.  Otherwise
    // every input may come from the previous kernel.
    if (!a.len_dev && !a.kv_early) pdl_wait();
    extern __shared__ __align__(128) unsigned char smem[];
    unsigned char* kbuf = smem;
    unsigned char* vbuf = smem + NST * SR * RB;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + NST * STAGE_BYTES);
    uint64_t* empty = full + NST;
    __shared__ float red_m[NW][G], red_l[NW][G];
    __shared__ int s_issued, s_consumed, s_last;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int kvh = blockIdx.y, split = blockIdx.x, qz = blockIdx.z;
    const int T = a.len_dev ? (*a.len_dev + 1) : a.T;
    // With the length read on the device the grid is planned for the cache's
    // capacity; the rows actually present are re-split here into about
    // DYN_ROWS rows per CTA, and CTAs past the last such split leave at once
    // (the merge then counts only the splits in use).
    int rps = a.rows_per_split, nsplit = a.n_splits;
    if (a.len_dev) {
        const Split sp = dev_split(T, a.n_splits, SR, DYN_ROWS);
        rps = sp.rps;
        nsplit = sp.nsplit;
        if (split >= nsplit) return;
    }
    const int t0 = split * rps;
    const int nrows = max(0, min(T + qz * a.q_causal - t0, rps));
    const int nst = (nrows + SR - 1) / SR;
    const KT* kg = static_cast<const KT*>(a.k) + (size_t)kvh * a.kv_head_stride + (size_t)t0 * D;
    const KT* vg = static_cast<const KT*>(a.v) + (size_t)kvh * a.kv_head_stride + (size_t)t0 * D;

    if (tid == 0) {
        for (int s = 0; s < NST; ++s) {
            mbar_init(full + s, 1);
            mbar_init(empty + s, NW);
        }
        fence_barrier_init();
        s_issued = 0;
        s_consumed = nst;
    }
    __syncthreads();

    float m[G], l[G], o[G][CPL];
    const int grp = lane >> 3, sub = lane & 7;

    if (warp == NW) {
        // ---------------- producer: one elected lane issues the bulk copies
        // device-length launches: every stage of rows cached by earlier steps
        // that fits the ring goes out before the wait for the previous
        // kernel, including the rows of the newest row's stage before it;
        // the newest row (appended by that kernel) follows the wait
        PreWait pw = pre_wait_plan(a.len_dev != nullptr, T, t0, nrows, SR, NST);
        if (a.kv_early && !a.len_dev) {   // every row is in place: fill the ring before the wait
            pw.pre = min(NST, pw.nst);
            pw.post0 = pw.pre;
        }
        const int pre = pw.pre, st_new = pw.st_new;
        const bool split_new = pw.split_new;
        const uint64_t pol = policy_evict_first();
        if (lane == 0) {
            for (int it = 0; it < pre; ++it) {
                const uint32_t bytes = (uint32_t)(min(SR, nrows - it * SR) * RB);
                mbar_arrive_expect_tx(full + it, 2 * bytes);
                bulk_g2s_hint(kbuf + it * SR * RB, kg + (size_t)it * SR * D, bytes, full + it, pol);
                bulk_g2s_hint(vbuf + it * SR * RB, vg + (size_t)it * SR * D, bytes, full + it, pol);
            }
            if (split_new) {
                const int rows = pw.head + 1;                        // the stage's rows, newest last
                mbar_arrive_expect_tx(full + st_new, 2 * (uint32_t)(rows * RB));
                if (rows > 1) {
                    const uint32_t bytes = (uint32_t)((rows - 1) * RB);
                    bulk_g2s_hint(kbuf + st_new * SR * RB, kg + (size_t)st_new * SR * D, bytes, full + st_new, pol);
                    bulk_g2s_hint(vbuf + st_new * SR * RB, vg + (size_t)st_new * SR * D, bytes, full + st_new, pol);
                }
            }
        }
        __syncwarp();
        if (a.len_dev || a.kv_early) pdl_wait();
        if (lane == 0) {
            int it = pre;
            if (split_new) {
                const int r = st_new * SR + pw.head;                 // the newest row, T - 1 - t0
                bulk_g2s_hint(kbuf + r * RB, kg + (size_t)r * D, RB, full + st_new, pol);
                bulk_g2s_hint(vbuf + r * RB, vg + (size_t)r * D, RB, full + st_new, pol);
                it = pw.post0;
            }
            for (; it < nst; ++it) {
                const int s = it % NST;
                if (it >= NST && !mbar_wait(empty + s, ((it / NST) & 1) ^ 1, a.status)) break;
                const int rows = min(SR, nrows - it * SR);
                const uint32_t bytes = (uint32_t)(rows * RB);
                mbar_arrive_expect_tx(full + s, 2 * bytes);
                bulk_g2s_hint(kbuf + s * SR * RB, kg + (size_t)it * SR * D, bytes, full + s, pol);
                bulk_g2s_hint(vbuf + s * SR * RB, vg + (size_t)it * SR * D, bytes, full + s, pol);
            }
            s_issued = it;
        }
    } else {
        // ---------------- consumers (q comes from the previous kernel)
        if (a.len_dev || a.kv_early) pdl_wait();
        float qr[G][CPL];
#pragma unroll
        for (int g = 0; g < G; ++g) {
            const KT* qh = static_cast<const KT*>(a.q) + (size_t)qz * a.q_stride + (size_t)(kvh * G + g) * D;
#pragma unroll
            for (int c = 0; c < CH; ++c) {
                Chunk<KT>::load_cg(qh + (sub + 8 * c) * VEC, &qr[g][c * VEC]);
#pragma unroll
                for (int e = 0; e < VEC; ++e) qr[g][c * VEC + e] *= a.qscale;
            }
            m[g] = -INFINITY;
            l[g] = 0.f;
#pragma unroll
            for (int i = 0; i < CPL; ++i) o[g][i] = 0.f;
        }

        int it = 0;
        for (; it < nst; ++it) {
            const int s = it % NST;
            if (!mbar_wait(full + s, (it / NST) & 1, a.status)) break;
            const int valid_rows = min(SR, nrows - it * SR);
            const unsigned char* ks = kbuf + s * SR * RB;
            const unsigned char* vs = vbuf + s * SR * RB;

            float sc[G][S::NR];
#pragma unroll
            for (int j = 0; j < S::NR; ++j) {
                const int r = warp * S::RW + grp + 4 * j;
                float kf[CPL];
#pragma unroll
                for (int c = 0; c < CH; ++c)
                    Chunk<KT>::load(ks + (size_t)r * RB + (sub + 8 * c) * 16, &kf[c * VEC]);
#pragma unroll
                for (int g = 0; g < G; ++g) {
                    float acc = 0.f;
#pragma unroll
                    for (int i = 0; i < CPL; ++i) acc = fmaf(qr[g][i], kf[i], acc);
                    sc[g][j] = acc;
                }
            }
#pragma unroll
            for (int g = 0; g < G; ++g)
#pragma unroll
                for (int j = 0; j < S::NR; ++j) {
                    float x = sc[g][j];
                    x += __shfl_xor_sync(0xffffffffu, x, 1);
                    x += __shfl_xor_sync(0xffffffffu, x, 2);
                    x += __shfl_xor_sync(0xffffffffu, x, 4);
                    sc[g][j] = x;
                }

            float p[G][S::NR];
#pragma unroll
            for (int g = 0; g < G; ++g) {
                float mx = m[g];
#pragma unroll
                for (int j = 0; j < S::NR; ++j)
                    if (warp * S::RW + grp + 4 * j < valid_rows) mx = fmaxf(mx, sc[g][j]);
                const float corr = (m[g] == -INFINITY) ? 0.f : ex2(m[g] - mx);
                float ps = 0.f;
#pragma unroll
                for (int j = 0; j < S::NR; ++j) {
                    const bool ok = warp * S::RW + grp + 4 * j < valid_rows;
                    p[g][j] = ok ? ex2(sc[g][j] - mx) : 0.f;
                    ps += p[g][j];
                }
                l[g] = l[g] * corr + ps;
#pragma unroll
                for (int i = 0; i < CPL; ++i) o[g][i] *= corr;
                m[g] = mx;
            }
#pragma unroll
            for (int j = 0; j < S::NR; ++j) {
                const int r = warp * S::RW + grp + 4 * j;
                if (r < valid_rows) {
                    float vf[CPL];
#pragma unroll
                    for (int c = 0; c < CH; ++c)
                        Chunk<KT>::load(vs + (size_t)r * RB + (sub + 8 * c) * 16, &vf[c * VEC]);
#pragma unroll
                    for (int g = 0; g < G; ++g)
#pragma unroll
                        for (int i = 0; i < CPL; ++i) o[g][i] = fmaf(p[g][j], vf[i], o[g][i]);
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(empty + s);
        }
        if (lane == 0 && it < nst) atomicMin(&s_consumed, it);

        // combine the 4 row groups of this warp (lanes with equal `sub` hold
        // the same columns)
#pragma unroll
        for (int off = 8; off <= 16; off <<= 1) {
#pragma unroll
            for (int g = 0; g < G; ++g) {
                const float m2 = __shfl_xor_sync(0xffffffffu, m[g], off);
                const float l2 = __shfl_xor_sync(0xffffffffu, l[g], off);
                float wa, wb, M;
                combine_weights(m[g], m2, wa, wb, M);
                l[g] = l[g] * wa + l2 * wb;
#pragma unroll
                for (int i = 0; i < CPL; ++i) {
                    const float o2 = __shfl_xor_sync(0xffffffffu, o[g][i], off);
                    o[g][i] = o[g][i] * wa + o2 * wb;
                }
                m[g] = M;
            }
        }
    }
    __syncthreads();

    // On an aborted pipeline, let copies still in flight land (bounded) before
    // the stage buffers are reused or the CTA exits.
    if (tid == 0 && s_consumed < s_issued) {
        for (int it = s_consumed; it < s_issued; ++it)
            mbar_wait(full + it % NST, (it / NST) & 1, nullptr);
    }
    __syncthreads();

    // cross-warp reduction through the (now idle) stage buffers
    float* red_o = reinterpret_cast<float*>(smem);   // [NW][G][D]
    if (warp < NW && grp == 0) {
#pragma unroll
        for (int g = 0; g < G; ++g) {
#pragma unroll
            for (int c = 0; c < CH; ++c)
#pragma unroll
                for (int e = 0; e < VEC; ++e)
                    red_o[(warp * G + g) * D + (sub + 8 * c) * VEC + e] = o[g][c * VEC + e];
            if (sub == 0) {
                red_m[warp][g] = m[g];
                red_l[warp][g] = l[g];
            }
        }
    }
    __syncthreads();

    const bool sp = a.sp.world > 1;
    float* fin = reinterpret_cast<float*>(smem + FIN_OFF);       // [G][D+2] (sequence-parallel)
    // A device-side wait that expired (this CTA's, or one of a split that
    // arrived before the merge) leaves NaN in the output, so a caller that
    // never reads the status word still sees the failure.
    const float bad = nanf("");
    bool failed = *reinterpret_cast<volatile int*>(a.status) != 0;
    for (int idx = tid; idx < G * D; idx += THREADS) {
        const int g = idx / D, col = idx % D;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < NW; ++w) M = fmaxf(M, red_m[w][g]);
        float L = 0.f, O = 0.f;
#pragma unroll
        for (int w = 0; w < NW; ++w) {
            const float wt = (red_m[w][g] == -INFINITY) ? 0.f : ex2(red_m[w][g] - M);
            L += red_l[w][g] * wt;
            O += red_o[(w * G + g) * D + col] * wt;
        }
        const int h = kvh * G + g;
        if (nsplit == 1) {
            if (sp) {   // this rank's state of head h, exchanged below
                fin[g * (D + 2) + col] = L > 0.f ? O / L : 0.f;
                if (col == 0) {
                    fin[g * (D + 2) + D] = M;
                    fin[g * (D + 2) + D + 1] = L;
                }
                continue;
            }
            // one split: this CTA holds the whole state; finalise in place
            a.out[(size_t)qz * a.o_stride + (size_t)h * D + col] = failed ? bad : (L > 0.f ? O / L : 0.f);
            if (col == 0 && a.out_m) {
                a.out_m[h] = L > 0.f ? M * LN2 : -INFINITY;
                a.out_l[h] = L > 0.f ? L : 1.f;
            }
            continue;
        }
        const size_t pi = (size_t)h * a.n_splits + split;
        a.part_o[pi * D + col] = L > 0.f ? O / L : 0.f;
        if (col == 0) {
            a.part_m[pi] = M;
            a.part_l[pi] = L;
        }
    }
    if (nsplit == 1) {
        if (sp) {
            __syncthreads();
            sp_exchange<G, D>(a, kvh, fin, reinterpret_cast<float*>(smem + ML_OFF));
        }
        return;
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) s_last = (atomicAdd(&a.counters[kvh], 1u) == (unsigned)(nsplit - 1));
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    failed = *reinterpret_cast<volatile int*>(a.status) != 0;

    // ---------------- last CTA of this KV head: merge the split partials
    float* wts = reinterpret_cast<float*>(smem);                 // [G][nsplit]
    float* hdr = wts + G * a.n_splits;                           // [G]: M, L
    const int ns = nsplit, pstride = a.n_splits;                  // splits in use; partials' row stride
    for (int g = warp; g < G; g += THREADS / 32) {
        const int h = kvh * G + g;
        float M = -INFINITY;
        for (int i = lane; i < ns; i += 32) M = fmaxf(M, __ldcg(a.part_m + (size_t)h * pstride + i));
#pragma unroll
        for (int off = 16; off; off >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off));
        float L = 0.f;
        for (int i = lane; i < ns; i += 32) {
            const float mi = __ldcg(a.part_m + (size_t)h * pstride + i);
            const float wi = (mi == -INFINITY) ? 0.f : __ldcg(a.part_l + (size_t)h * pstride + i) * ex2(mi - M);
            wts[g * ns + i] = wi;
            L += wi;
        }
#pragma unroll
        for (int off = 16; off; off >>= 1) L += __shfl_xor_sync(0xffffffffu, L, off);
        if (lane == 0) {
            hdr[2 * g] = M;
            hdr[2 * g + 1] = L;
        }
    }
    __syncthreads();
    for (int idx = tid; idx < G * D; idx += THREADS) {
        const int g = idx / D, col = idx % D;
        const int h = kvh * G + g;
        const float L = hdr[2 * g + 1];
        float O = 0.f;
        for (int i = 0; i < ns; ++i) O += wts[g * ns + i] * __ldcg(a.part_o + ((size_t)h * pstride + i) * D + col);
        if (sp) {
            fin[g * (D + 2) + col] = L > 0.f ? O / L : 0.f;
            if (col == 0) {
                fin[g * (D + 2) + D] = hdr[2 * g];
                fin[g * (D + 2) + D + 1] = L;
            }
            continue;
        }
        a.out[(size_t)h * D + col] = failed ? bad : (L > 0.f ? O / L : 0.f);
        if (col == 0 && a.out_m) {
            a.out_m[h] = L > 0.f ? hdr[2 * g] * LN2 : -INFINITY;
            a.out_l[h] = L > 0.f ? L : 1.f;
        }
    }
    if (tid == 0) a.counters[kvh] = 0u;
    if (sp) {
        __syncthreads();
        sp_exchange<G, D>(a, kvh, fin, reinterpret_cast<float*>(smem + ML_OFF));
    }
}

// Merge n partial states given in the natural-log domain (API layout
// part-major: m, l [n][hq]; o [n][hq][d]).
__global__ void merge_kernel(int n, int hq, int d, const float* __restrict__ m,
                             const float* __restrict__ l, const float* __restrict__ o,
                             float* __restrict__ out, float* __restrict__ out_m,
                             float* __restrict__ out_l) {
    const int h = blockIdx.x;
    float M = -INFINITY;
    for (int i = 0; i < n; ++i) M = fmaxf(M, m[(size_t)i * hq + h]);
    float L = 0.f;
    for (int i = 0; i < n; ++i) {
        const float mi = m[(size_t)i * hq + h];
        L += (mi == -INFINITY) ? 0.f : l[(size_t)i * hq + h] * ex2((mi - M) * LOG2E);
    }
    for (int c = threadIdx.x; c < d; c += blockDim.x) {
        float O = 0.f;
        for (int i = 0; i < n; ++i) {
            const float mi = m[(size_t)i * hq + h];
            const float wi = (mi == -INFINITY) ? 0.f : l[(size_t)i * hq + h] * ex2((mi - M) * LOG2E);
            O += wi * o[((size_t)i * hq + h) * d + c];
        }
        out[(size_t)h * d + c] = L > 0.f ? O / L : 0.f;
    }
    if (threadIdx.x == 0 && out_m) {
        out_m[h] = L > 0.f ? M : -INFINITY;
        out_l[h] = L > 0.f ? L : 1.f;
    }
}

using KernelFn = void (*)(const Args);

template <typename KT, int D>
static KernelFn pick_g(int G) {
    switch (G) {
        case 1: return decode_kernel<KT, D, 1>;
        case 2: return decode_kernel<KT, D, 2>;
        case 4: if constexpr (D <= 128) return decode_kernel<KT, D, 4>; else return nullptr;
        case 8: if constexpr (D <= 64) return decode_kernel<KT, D, 8>; else return nullptr;
        default: return nullptr;
    }
}

template <typename KT>
static KernelFn pick(int d, int G) {
    switch (d) {
        case 64: return pick_g<KT, 64>(G);
        case 128: return pick_g<KT, 128>(G);
        case 256: return pick_g<KT, 256>(G);
        default: return nullptr;
    }
}

static int stage_rows(int dtype, int d) { return STAGE_BYTES / (2 * d * (dtype == SA_F32 ? 4 : 2)); }

// The decode step's kernel (fp32 cache, head_dim 128): a DEV_STAGES-deep ring.
static KernelFn pick_dev(int d, int G) {
    if (d != 128) return nullptr;
    switch (G) {
        case 1: return decode_kernel<float, 128, 1, DEV_STAGES>;
        case 2: return decode_kernel<float, 128, 2, DEV_STAGES>;
        case 4: return decode_kernel<float, 128, 4, DEV_STAGES>;
        default: return nullptr;
    }
}

}  // namespace dec

// Plan the split of T rows over CTAs: about 2 CTAs per SM overall.
static void plan_splits(int num_sms, int T, int hkv, int stage_rows, int* n_splits, int* rows_per_split) {
    if (T <= 0) {
        *n_splits = 1;
        *rows_per_split = stage_rows;
        return;
    }
    const int slots = 2 * num_sms;
    int ns = slots / hkv;
    const int max_by_rows = (T + stage_rows - 1) / stage_rows;
    if (ns > max_by_rows) ns = max_by_rows;
    if (ns > dec::MAX_SPLITS) ns = dec::MAX_SPLITS;
    if (ns < 1) ns = 1;
    int rps = (T + ns - 1) / ns;
    rps = (rps + stage_rows - 1) / stage_rows * stage_rows;
    *rows_per_split = rps;
    *n_splits = (T + rps - 1) / rps;
}

// Validate a decode call's arguments (shared by the host- and device-pointer
// paths and by the entry point that takes caller-provided scratch).
static int check_decode_args(const char* fn, int dtype, const void* q, const void* k, const void* v,
                             long long stride, int T, int d, int hq, int hkv, int block) {
    SA_CHECK_ARG(dtype == SA_F32 || dtype == SA_BF16, "%s: dtype %d (want SA_F32 or SA_BF16)", fn, dtype);
    SA_CHECK_ARG(q && (T == 0 || (k && v)), "%s: null q/k/v", fn);
    SA_CHECK_ARG(T >= 0, "%s: T = %d", fn, T);
    SA_CHECK_ARG(block > 0, "%s: block = %d", fn, block);
    SA_CHECK_ARG(hkv > 0 && hq > 0 && hq % hkv == 0, "%s: hq = %d, hkv = %d", fn, hq, hkv);
    SA_CHECK_ARG(hkv <= SA_MAX_KV_HEADS, "%s: hkv = %d > %d", fn, hkv, SA_MAX_KV_HEADS);
    SA_CHECK_ARG(d == 64 || d == 128 || d == 256, "%s: d = %d (supported: 64, 128, 256)", fn, d);
    const int elt = dtype == SA_F32 ? 4 : 2;
    SA_CHECK_ARG(stride >= (long long)T * d || hkv == 1, "%s: kv_head_stride %lld < T*d", fn, stride);
    SA_CHECK_ARG(((stride * elt) % 16) == 0, "%s: kv_head_stride*%d bytes not 16-byte aligned", fn, elt);
    SA_CHECK_ARG(dec::pick<float>(d, hq / hkv) != nullptr,
                 "%s: hq/hkv = %d unsupported at d = %d", fn, hq / hkv, d);
    return SA_OK;
}

// Launch the decode kernel on device pointers.  `part` must hold
// hq*n_splits*(d+2) floats for the plan the call computes.
static int launch_decode(sa_ctx* ctx, int dtype, const void* q, const void* k, const void* v,
                         long long stride, int T, int d, int hq, int hkv, float scale, float* out,
                         float* out_m, float* out_l, const dec::SpArgs* sp = nullptr, bool kv_early = false) {
    SA_CHECK_ARG(T == 0 || (((uintptr_t)k | (uintptr_t)v) & 15) == 0, "decode: k/v not 16-byte aligned");
    SA_CHECK_ARG((((uintptr_t)q) & 15) == 0, "decode: q not 16-byte aligned");
    int ns, rps;
    const int sr = dec::stage_rows(dtype, d);
    plan_splits(ctx->num_sms, T, hkv, sr, &ns, &rps);
    const size_t npart = (size_t)hq * ns;
    int rc = ensure_ws(ctx, npart * (d + 2) * sizeof(float));
    if (rc) return rc;
    dec::Args a;
    a.q = q; a.k = k; a.v = v;
    a.kv_head_stride = hkv == 1 ? 0 : stride;
    a.T = T; a.hq = hq; a.hkv = hkv;
    a.rows_per_split = rps; a.n_splits = ns;
    a.qscale = scale * dec::LOG2E;
    float* ws = static_cast<float*>(ctx->ws);
    a.part_m = ws;
    a.part_l = ws + npart;
    a.part_o = ws + 2 * npart;
    a.counters = ctx->counters;
    a.out = out; a.out_m = out_m; a.out_l = out_l;
    a.status = ctx->status;
    a.q_stride = 0; a.o_stride = 0; a.q_causal = 1; a.kv_early = 0;
    a.len_dev = nullptr;
    a.sp = {};
    a.sp.world = 1;
    if (sp) a.sp = *sp;
    a.kv_early = kv_early ? 1 : 0;
    dec::KernelFn fn = dtype == SA_F32 ? dec::pick<float>(d, hq / hkv) : dec::pick<__nv_bfloat16>(d, hq / hkv);
    SA_CUDA_TRY(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, dec::SMEM_BYTES));
    if (kv_early) {
        SA_CUDA_TRY(launch_pdl(fn, dim3(ns, hkv), dim3(dec::THREADS), dec::SMEM_BYTES, ctx->stream, a));
    } else {
        fn<<<dim3(ns, hkv), dec::THREADS, dec::SMEM_BYTES, ctx->stream>>>(a);
        SA_CUDA_TRY(cudaGetLastError());
    }
    return SA_OK;
}

static int decode_common(const char* fn_name, sa_ctx* ctx, int dtype, const void* q, const void* k,
                         const void* v, long long stride, int T, int d, int hq, int hkv, int block,
                         float scale, float* out, float* m_out, float* l_out, unsigned flags,
                         const dec::SpArgs* sp = nullptr) {
    clear_error();
    SA_CHECK_ARG(ctx != nullptr, "%s: ctx is NULL", fn_name);
    SA_CHECK_ARG(out != nullptr, "%s: out is NULL", fn_name);
    int rc = check_decode_args(fn_name, dtype, q, k, v, stride, T, d, hq, hkv, block);
    if (rc) return rc;
    DeviceGuard guard(ctx->device);
    if (!(flags & SA_HOST_PTRS))
        return launch_decode(ctx, dtype, q, k, v, stride, T, d, hq, hkv, scale, out, m_out, l_out, sp,
                             (flags & SA_KV_STATIC) != 0);

    // Host buffers: stage through device memory on the context's stream.
    const int elt = dtype == SA_F32 ? 4 : 2;
    const size_t qb = align_up((size_t)hq * d * elt, 256);
    const size_t kvb = align_up((size_t)hkv * T * d * elt, 256);
    const size_t ob = align_up((size_t)hq * d * 4, 256);
    const size_t sb = align_up((size_t)hq * 4, 256);
    rc = ensure_stage(ctx, qb + 2 * kvb + ob + 2 * sb);
    if (rc) return rc;
    char* base = static_cast<char*>(ctx->stage);
    void* dq = base;
    void* dk = base + qb;
    void* dv = base + qb + kvb;
    float* dout = reinterpret_cast<float*>(base + qb + 2 * kvb);
    float* dm = reinterpret_cast<float*>(base + qb + 2 * kvb + ob);
    float* dl = reinterpret_cast<float*>(base + qb + 2 * kvb + ob + sb);
    cudaStream_t st = ctx->stream;
    const size_t row = (size_t)T * d * elt;
    SA_CUDA_TRY(cudaMemcpyAsync(dq, q, (size_t)hq * d * elt, cudaMemcpyHostToDevice, st));
    if (T > 0) {
        const size_t pitch = hkv == 1 ? row : (size_t)stride * elt;
        SA_CUDA_TRY(cudaMemcpy2DAsync(dk, row, k, pitch, row, hkv, cudaMemcpyHostToDevice, st));
        SA_CUDA_TRY(cudaMemcpy2DAsync(dv, row, v, pitch, row, hkv, cudaMemcpyHostToDevice, st));
    }
    rc = launch_decode(ctx, dtype, dq, dk, dv, (long long)T * d, T, d, hq, hkv, scale, dout,
                       m_out ? dm : nullptr, m_out ? dl : nullptr, sp);
    if (rc) return rc;
    SA_CUDA_TRY(cudaMemcpyAsync(out, dout, (size_t)hq * d * 4, cudaMemcpyDeviceToHost, st));
    if (m_out) {
        SA_CUDA_TRY(cudaMemcpyAsync(m_out, dm, (size_t)hq * 4, cudaMemcpyDeviceToHost, st));
        SA_CUDA_TRY(cudaMemcpyAsync(l_out, dl, (size_t)hq * 4, cudaMemcpyDeviceToHost, st));
    }
    return sync_and_check(ctx);
}

}  // namespace sa

SA_API int sa_attn_decode(sa_ctx* ctx, int dtype, const void* q, const void* k, const void* v,
                          long long kv_head_stride, int T, int d, int hq, int hkv, int block,
                          float scale, float* out, unsigned flags) {
    return sa::decode_common("sa_attn_decode", ctx, dtype, q, k, v, kv_head_stride, T, d, hq, hkv,
                             block, scale, out, nullptr, nullptr, flags);
}

SA_API int sa_attn_decode_partial(sa_ctx* ctx, int dtype, const void* q, const void* k,
                                  const void* v, long long kv_head_stride, int T, int d, int hq,
                                  int hkv, int block, float scale, float* m_out, float* l_out,
                                  float* o_out, unsigned flags) {
    SA_CHECK_ARG(m_out && l_out, "sa_attn_decode_partial: null m_out/l_out");
    return sa::decode_common("sa_attn_decode_partial", ctx, dtype, q, k, v, kv_head_stride, T, d, hq,
                             hkv, block, scale, o_out, m_out, l_out, flags);
}

SA_API int sa_attn_merge(sa_ctx* ctx, int n_parts, int hq, int d, const float* m, const float* l,
                         const float* o, float* out, float* m_out, float* l_out, unsigned flags) {
    sa::clear_error();
    SA_CHECK_ARG(ctx != nullptr, "sa_attn_merge: ctx is NULL");
    SA_CHECK_ARG(n_parts >= 1 && hq >= 1 && d >= 1, "sa_attn_merge: n_parts=%d hq=%d d=%d", n_parts, hq, d);
    SA_CHECK_ARG(m && l && o && out, "sa_attn_merge: null pointer");
    SA_CHECK_ARG((m_out == nullptr) == (l_out == nullptr), "sa_attn_merge: m_out/l_out must both be set or NULL");
    sa::DeviceGuard guard(ctx->device);
    cudaStream_t st = ctx->stream;
    if (!(flags & SA_HOST_PTRS)) {
        sa::dec::merge_kernel<<<hq, 128, 0, st>>>(n_parts, hq, d, m, l, o, out, m_out, l_out);
        SA_CUDA_TRY(cudaGetLastError());
        return SA_OK;
    }
    const size_t ml = sa::align_up((size_t)n_parts * hq * 4, 256);
    const size_t ob = sa::align_up((size_t)n_parts * hq * d * 4, 256);
    const size_t outb = sa::align_up((size_t)hq * d * 4, 256);
    const size_t sb = sa::align_up((size_t)hq * 4, 256);
    int rc = sa::ensure_stage(ctx, 2 * ml + ob + outb + 2 * sb);
    if (rc) return rc;
    char* b = static_cast<char*>(ctx->stage);
    float* dm = (float*)b;
    float* dl = (float*)(b + ml);
    float* dO = (float*)(b + 2 * ml);
    float* dout = (float*)(b + 2 * ml + ob);
    float* dmo = (float*)(b + 2 * ml + ob + outb);
    float* dlo = (float*)(b + 2 * ml + ob + outb + sb);
    SA_CUDA_TRY(cudaMemcpyAsync(dm, m, (size_t)n_parts * hq * 4, cudaMemcpyHostToDevice, st));
    SA_CUDA_TRY(cudaMemcpyAsync(dl, l, (size_t)n_parts * hq * 4, cudaMemcpyHostToDevice, st));
    SA_CUDA_TRY(cudaMemcpyAsync(dO, o, (size_t)n_parts * hq * d * 4, cudaMemcpyHostToDevice, st));
    sa::dec::merge_kernel<<<hq, 128, 0, st>>>(n_parts, hq, d, dm, dl, dO, dout, m_out ? dmo : nullptr,
                                              m_out ? dlo : nullptr);
    SA_CUDA_TRY(cudaGetLastError());
    SA_CUDA_TRY(cudaMemcpyAsync(out, dout, (size_t)hq * d * 4, cudaMemcpyDeviceToHost, st));
    if (m_out) {
        SA_CUDA_TRY(cudaMemcpyAsync(m_out, dmo, (size_t)hq * 4, cudaMemcpyDeviceToHost, st));
        SA_CUDA_TRY(cudaMemcpyAsync(l_out, dlo, (size_t)hq * 4, cudaMemcpyDeviceToHost, st));
    }
    return sa::sync_and_check(ctx);
}

namespace sa {
// Split-KV decode whose row count comes from device memory (T = *len_dev + 1)
// with a split plan fixed for max_T rows: splits past the current length are
// empty and drop out of the merge.  Scratch (partials, counters) is the
// caller's, sized by decode_dev_scratch_floats.  Used by the Qwen3 decode
// step, which is captured once in a CUDA graph and replayed per token.
size_t decode_dev_scratch_floats(int num_sms, int max_T, int d, int hq, int hkv, int* n_splits) {
    int ns, rps;
    plan_splits(num_sms, max_T, hkv, dec::stage_rows(SA_F32, d), &ns, &rps);
    if (n_splits) *n_splits = ns;
    return (size_t)hq * ns * (d + 2);
}

int decode_dev_launch(cudaStream_t st, int* status, int num_sms, const float* q, const float* k, const float* v,
                      long long kv_head_stride, const int* len_dev, int T_host, int max_T, int d, int hq, int hkv,
                      float scale, float* out, float* scratch, unsigned* counters) {
    int ns, rps;
    plan_splits(num_sms, max_T, hkv, dec::stage_rows(SA_F32, d), &ns, &rps);
    const size_t npart = (size_t)hq * ns;
    dec::Args a;
    a.q = q; a.k = k; a.v = v;
    a.kv_head_stride = kv_head_stride;
    a.T = len_dev ? max_T : T_host; a.hq = hq; a.hkv = hkv;
    a.rows_per_split = rps; a.n_splits = ns;
    a.qscale = scale * dec::LOG2E;
    a.part_m = scratch;
    a.part_l = scratch + npart;
    a.part_o = scratch + 2 * npart;
    a.counters = counters;
    a.out = out; a.out_m = nullptr; a.out_l = nullptr;
    a.status = status;
    a.q_stride = 0; a.o_stride = 0; a.q_causal = 1; a.kv_early = 0;
    a.len_dev = len_dev;
    a.sp = {};
    a.sp.world = 1;
    dec::KernelFn fn = dec::pick_dev(d, hq / hkv);
    int smem = dec::smem_bytes<dec::DEV_STAGES>();
    if (!fn) {
        fn = dec::pick<float>(d, hq / hkv);
        smem = dec::SMEM_BYTES;
    }
    SA_CHECK_ARG(fn != nullptr, "decode_dev: hq/hkv=%d d=%d unsupported", hq / hkv, d);
    SA_RC_TRY(set_smem_attr_once((const void*)fn, smem));
    SA_CUDA_TRY(launch_pdl_k(2, fn, dim3(ns, hkv), dim3(dec::THREADS), smem, st, a));
    return SA_OK;
}
}  // namespace sa

// ===========================================================================
// Allocation-free decode entry point.
//
// Some callers cannot call cudaMalloc: serving runtimes that reserve nearly
// all device memory for their own pools at start-up (a later cudaMalloc can
// fail or fragment their budget), and latency-critical loops that must not
// pay for cudaMalloc's implicit device synchronisation.  They also cannot
// create an sa_ctx, whose constructor allocates.  For them this entry point
// keeps the decode kernel's scratch -- the per-split (m, l, O) partials, the
// per-KV-head arrival counters and the status word -- in one file-scope
// device array of fixed size instead.  Every GPU that loads the library holds
// the array until the process exits; every call on a GPU shares it.
// ===========================================================================
#include <mutex>

#define SA_NOALLOC_MAX_DEVICES 64

static __device__ __align__(256) unsigned char g_noalloc_scratch[SA_NOALLOC_SCRATCH_BYTES];

namespace sa {

static std::mutex g_noalloc_mu;
static void* g_noalloc_addr[SA_NOALLOC_MAX_DEVICES] = {};

// Device address of g_noalloc_scratch on `device` (which must be current).
// In host code the array's name is only a host-side stand-in, so the address
// is looked up once per device and cached.
static int noalloc_scratch(int device, void** out) {
    SA_CHECK_ARG(device >= 0 && device < SA_NOALLOC_MAX_DEVICES, "noalloc: device %d", device);
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    if (!g_noalloc_addr[device]) {
        void* p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || p == nullptr)
            return set_error(SA_ERR_CUDA, "cudaGetSymbolAddress(static scratch) on device %d: %s",
                             device, cudaGetErrorString(e));
        g_noalloc_addr[device] = p;
    }
    *out = g_noalloc_addr[device];
    return SA_OK;
}

}  // namespace sa

SA_API int sa_attn_decode_noalloc(void* stream, int dtype, const void* q, const void* k,
                                  const void* v, long long kv_head_stride, int T, int d, int hq,
                                  int hkv, int block, float scale, float* out) {
    using namespace sa;
    clear_error();
    SA_CHECK_ARG(out != nullptr, "sa_attn_decode_noalloc: out is NULL");
    int rc = check_decode_args("sa_attn_decode_noalloc", dtype, q, k, v, kv_head_stride, T, d, hq,
                               hkv, block);
    if (rc) return rc;
    SA_CHECK_ARG((((uintptr_t)k | (uintptr_t)v | (uintptr_t)q) & 15) == 0,
                 "sa_attn_decode_noalloc: q/k/v not 16-byte aligned");
    // the GPU is the one that holds `out`
    cudaPointerAttributes attr;
    SA_CUDA_TRY(cudaPointerGetAttributes(&attr, out));
    SA_CHECK_ARG(attr.type == cudaMemoryTypeDevice || attr.type == cudaMemoryTypeManaged,
                 "sa_attn_decode_noalloc: out must be device memory");
    DeviceGuard guard(attr.device);
    int num_sms = 0;
    SA_CUDA_TRY(cudaDeviceGetAttribute(&num_sms, cudaDevAttrMultiProcessorCount, attr.device));

    int ns, rps;
    plan_splits(num_sms, T, hkv, dec::stage_rows(dtype, d), &ns, &rps);
    const size_t cnt_bytes = align_up((size_t)hkv * sizeof(unsigned), 256);
    const size_t st_bytes = 256;
    const size_t npart = (size_t)hq * ns;
    const size_t need = cnt_bytes + st_bytes + npart * (d + 2) * sizeof(float);
    if (need > SA_NOALLOC_SCRATCH_BYTES)
        return set_error(SA_ERR_ARG,
                         "sa_attn_decode_noalloc: hq=%d hkv=%d d=%d needs %zu scratch bytes, more than "
                         "the static maximum of %u (SA_NOALLOC_SCRATCH_BYTES); use sa_attn_decode",
                         hq, hkv, d, need, (unsigned)SA_NOALLOC_SCRATCH_BYTES);
    void* base = nullptr;
    rc = noalloc_scratch(attr.device, &base);
    if (rc) return rc;
    char* b = static_cast<char*>(base);
    unsigned* counters = reinterpret_cast<unsigned*>(b);
    int* status = reinterpret_cast<int*>(b + cnt_bytes);
    float* part = reinterpret_cast<float*>(b + cnt_bytes + st_bytes);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    // The kernel's last CTA leaves the counters at zero, but a call that ended
    // early could not; start every call from zero, status word included (it
    // follows the counters), so that only this call's own failure shows.
    SA_CUDA_TRY(cudaMemsetAsync(counters, 0, cnt_bytes + sizeof(int), st));

    dec::Args a;
    a.q = q; a.k = k; a.v = v;
    a.kv_head_stride = hkv == 1 ? 0 : kv_head_stride;
    a.T = T; a.hq = hq; a.hkv = hkv;
    a.rows_per_split = rps; a.n_splits = ns;
    a.qscale = scale * dec::LOG2E;
    a.part_m = part;
    a.part_l = part + npart;
    a.part_o = part + 2 * npart;
    a.counters = counters;
    a.out = out; a.out_m = nullptr; a.out_l = nullptr;
    a.status = status;
    a.q_stride = 0; a.o_stride = 0; a.q_causal = 1; a.kv_early = 0;
    a.len_dev = nullptr;
    a.sp = {};
    a.sp.world = 1;
    dec::KernelFn fn = dtype == SA_F32 ? dec::pick<float>(d, hq / hkv) : dec::pick<__nv_bfloat16>(d, hq / hkv);
    SA_CUDA_TRY(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, dec::SMEM_BYTES));
    fn<<<dim3(ns, hkv), dec::THREADS, dec::SMEM_BYTES, st>>>(a);
    SA_CUDA_TRY(cudaGetLastError());
    return SA_OK;
}

// ===========================================================================
// One decode step over a device-resident KV cache: append the new token's
// K/V row at `pos`, then attend over rows [0, pos].  The reference does the
// same per layer in qwen3_decoder_layer_with_cache: kv_cache->update(...)
// (tensor_cpp/src/qwen3_ops.cpp:849, kv_cache.h:94-130) followed by attention
// over the cached prefix (:876-885).  The cache is [hkv][max_seq][d], the
// KVCache layout (kv_cache.h:24-25) with batch 1.
// ===========================================================================
SA_API int sa_attn_decode_step(sa_ctx* ctx, int dtype, const void* q, const void* k_new,
                               const void* v_new, void* k_cache, void* v_cache, int max_seq,
                               int pos, int d, int hq, int hkv, int block, float scale, float* out,
                               unsigned flags) {
    using namespace sa;
    clear_error();
    SA_CHECK_ARG(ctx != nullptr, "sa_attn_decode_step: ctx is NULL");
    SA_CHECK_ARG(out && k_new && v_new && k_cache && v_cache, "sa_attn_decode_step: null pointer");
    SA_CHECK_ARG(pos >= 0 && max_seq > 0, "sa_attn_decode_step: pos = %d, max_seq = %d", pos, max_seq);
    if (pos >= max_seq)
        return set_error(SA_ERR_FULL, "sa_attn_decode_step: KV cache full, cannot append at %d (max_seq %d)",
                         pos, max_seq);
    const long long stride = (long long)max_seq * d;
    int rc = check_decode_args("sa_attn_decode_step", dtype, q, k_cache, v_cache, stride, pos + 1, d, hq,
                               hkv, block);
    if (rc) return rc;
    DeviceGuard guard(ctx->device);
    const int elt = dtype == SA_F32 ? 4 : 2;
    const size_t row = (size_t)d * elt, pitch = (size_t)stride * elt;
    cudaStream_t st = ctx->stream;
    char* kc = static_cast<char*>(k_cache) + (size_t)pos * row;
    char* vc = static_cast<char*>(v_cache) + (size_t)pos * row;
    const bool host = flags & SA_HOST_PTRS;
    const cudaMemcpyKind kind = host ? cudaMemcpyHostToDevice : cudaMemcpyDeviceToDevice;
    SA_CUDA_TRY(cudaMemcpy2DAsync(kc, pitch, k_new, row, row, hkv, kind, st));
    SA_CUDA_TRY(cudaMemcpy2DAsync(vc, pitch, v_new, row, row, hkv, kind, st));
    if (!host)
        return launch_decode(ctx, dtype, q, k_cache, v_cache, stride, pos + 1, d, hq, hkv, scale, out,
                             nullptr, nullptr);
    const size_t qb = align_up((size_t)hq * d * elt, 256);
    rc = ensure_stage(ctx, qb + (size_t)hq * d * 4);
    if (rc) return rc;
    char* dq = static_cast<char*>(ctx->stage);
    float* dout = reinterpret_cast<float*>(dq + qb);
    SA_CUDA_TRY(cudaMemcpyAsync(dq, q, (size_t)hq * d * elt, cudaMemcpyHostToDevice, st));
    rc = launch_decode(ctx, dtype, dq, k_cache, v_cache, stride, pos + 1, d, hq, hkv, scale, dout,
                       nullptr, nullptr);
    if (rc) return rc;
    SA_CUDA_TRY(cudaMemcpyAsync(out, dout, (size_t)hq * d * 4, cudaMemcpyDeviceToHost, st));
    return sync_and_check(ctx);
}

// ===========================================================================
// Sequence-parallel decode over several GPUs (one rank per GPU).
//
// streaming_attention_mpi_simple (attention/src/streaming_mpi.cpp:252-309)
// splits the sequence over MPI ranks, gathers every rank's (m, l, O) on
// rank 0 and merges them there.  Here each rank's decode launch does the
// exchange itself: the merging CTA of every KV head stores its heads' states
// as self-validating words into every rank's word area (plain 8-byte stores
// over NVLink into CUDA IPC mappings, or peer pointers inside one process)
// and merges all ranks' states in rank order.  No collective library, no
// separate merge launch, and every rank gets the result.
// ===========================================================================
#include <cstring>

struct sa_sp {
    sa_ctx* ctx = nullptr;
    int device = 0, rank = 0, world = 1;
    int max_hq = 0, max_d = 0;
    size_t words_bytes = 0;
    unsigned long long* words = nullptr;       // own word area
    unsigned* ctl = nullptr;                   // [0] instance count, [1] arrivals
    unsigned long long* peer[sa::dec::SP_MAX] = {};
    bool opened[sa::dec::SP_MAX] = {};         // peer[r] is an IPC mapping to close
    bool connected = false;
    unsigned char uuid[16] = {};
};

namespace sa {
namespace {
constexpr uint32_t SP_MAGIC = 0x50534153u;   // "SASP"
struct SpHandle {                            // the SA_SP_HANDLE_BYTES blob
    cudaIpcMemHandle_t ipc;
    unsigned char uuid[16];
    int32_t rank, world;
    uint64_t words_bytes;
    uint32_t magic;
};
static_assert(sizeof(SpHandle) <= SA_SP_HANDLE_BYTES, "handle size");

void sp_close_peers(sa_sp* sp) {
    for (int r = 0; r < dec::SP_MAX; ++r) {
        if (sp->opened[r] && sp->peer[r]) cudaIpcCloseMemHandle(sp->peer[r]);
        sp->opened[r] = false;
        sp->peer[r] = nullptr;
    }
    sp->connected = false;
}
}  // namespace
}  // namespace sa

SA_API int sa_sp_create(sa_ctx* ctx, int rank, int world, int max_hq, int max_d, sa_sp** out) {
    using namespace sa;
    clear_error();
    SA_CHECK_ARG(ctx && out, "sa_sp_create: null argument");
    *out = nullptr;
    SA_CHECK_ARG(world >= 1 && world <= dec::SP_MAX, "sa_sp_create: world = %d (1..%d)", world, dec::SP_MAX);
    SA_CHECK_ARG(rank >= 0 && rank < world, "sa_sp_create: rank %d of %d", rank, world);
    SA_CHECK_ARG(max_hq >= 1 && max_hq <= 4096 && (max_d == 64 || max_d == 128 || max_d == 256),
                 "sa_sp_create: max_hq = %d, max_d = %d", max_hq, max_d);
    DeviceGuard guard(ctx->device);
    sa_sp* sp = new sa_sp();
    sp->ctx = ctx;
    sp->device = ctx->device;
    sp->rank = rank;
    sp->world = world;
    sp->max_hq = max_hq;
    sp->max_d = max_d;
    sp->words_bytes = align_up((size_t)2 * world * max_hq * (max_d + 2) * sizeof(unsigned long long), 4096);
    cudaDeviceProp prop;
    if (cudaGetDeviceProperties(&prop, ctx->device) != cudaSuccess ||
        cudaMalloc(&sp->words, sp->words_bytes) != cudaSuccess ||
        cudaMalloc(&sp->ctl, 2 * sizeof(unsigned)) != cudaSuccess ||
        cudaMemset(sp->words, 0, sp->words_bytes) != cudaSuccess ||
        cudaMemset(sp->ctl, 0, 2 * sizeof(unsigned)) != cudaSuccess) {
        const cudaError_t e = cudaGetLastError();
        cudaFree(sp->words);
        cudaFree(sp->ctl);
        delete sp;
        return set_error(SA_ERR_OOM, "sa_sp_create: %s", cudaGetErrorString(e));
    }
    std::memcpy(sp->uuid, &prop.uuid, sizeof(sp->uuid));
    sp->peer[rank] = sp->words;
    sp->connected = world == 1;
    *out = sp;
    return SA_OK;
}

SA_API int sa_sp_handle(sa_sp* sp, void* handle) {
    using namespace sa;
    clear_error();
    SA_CHECK_ARG(sp && handle, "sa_sp_handle: null argument");
    DeviceGuard guard(sp->device);
    SpHandle h;
    std::memset(&h, 0, sizeof(h));
    SA_CUDA_TRY(cudaIpcGetMemHandle(&h.ipc, sp->words));
    std::memcpy(h.uuid, sp->uuid, sizeof(h.uuid));
    h.rank = sp->rank;
    h.world = sp->world;
    h.words_bytes = sp->words_bytes;
    h.magic = SP_MAGIC;
    std::memset(handle, 0, SA_SP_HANDLE_BYTES);
    std::memcpy(handle, &h, sizeof(h));
    return SA_OK;
}

SA_API int sa_sp_connect(sa_sp* sp, const void* handles) {
    using namespace sa;
    clear_error();
    SA_CHECK_ARG(sp && handles, "sa_sp_connect: null argument");
    if (sp->world == 1) return SA_OK;
    SA_CHECK_ARG(!sp->connected, "sa_sp_connect: already connected");
    DeviceGuard guard(sp->device);
    const unsigned char* hb = static_cast<const unsigned char*>(handles);
    for (int r = 0; r < sp->world; ++r) {
        SpHandle h;
        std::memcpy(&h, hb + (size_t)r * SA_SP_HANDLE_BYTES, sizeof(h));
        const char* bad = nullptr;
        if (h.magic != SP_MAGIC) bad = "is not an sa_sp handle";
        else if (h.rank != r || h.world != sp->world) bad = "names another rank or world size";
        else if (h.words_bytes != sp->words_bytes) bad = "was created with other max_hq / max_d";
        else if (r != sp->rank && std::memcmp(h.uuid, sp->uuid, sizeof(h.uuid)) == 0)
            bad = "is on this rank's GPU (the exchange waits across ranks: one GPU per rank)";
        if (bad) {
            sp_close_peers(sp);
            sp->peer[sp->rank] = sp->words;
            return set_error(SA_ERR_ARG, "sa_sp_connect: handle %d %s", r, bad);
        }
        if (r == sp->rank) continue;
        void* p = nullptr;
        const cudaError_t e = cudaIpcOpenMemHandle(&p, h.ipc, cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess) {
            cudaGetLastError();
            sp_close_peers(sp);
            sp->peer[sp->rank] = sp->words;
            return set_error(SA_ERR_CUDA, "sa_sp_connect: opening rank %d's word area failed: %s", r,
                             cudaGetErrorString(e));
        }
        sp->peer[r] = static_cast<unsigned long long*>(p);
        sp->opened[r] = true;
    }
    sp->peer[sp->rank] = sp->words;
    sp->connected = true;
    return SA_OK;
}

SA_API int sa_sp_connect_local(sa_sp* const* sps, int n) {
    using namespace sa;
    clear_error();
    SA_CHECK_ARG(sps && n >= 1 && n <= dec::SP_MAX, "sa_sp_connect_local: n = %d", n);
    for (int i = 0; i < n; ++i) {
        SA_CHECK_ARG(sps[i] && sps[i]->rank == i && sps[i]->world == n,
                     "sa_sp_connect_local: entry %d is not rank %d of %d", i, i, n);
        SA_CHECK_ARG(!sps[i]->connected || n == 1, "sa_sp_connect_local: rank %d already connected", i);
        SA_CHECK_ARG(sps[i]->words_bytes == sps[0]->words_bytes,
                     "sa_sp_connect_local: rank %d was created with other max_hq / max_d", i);
        for (int j = 0; j < i; ++j)
            SA_CHECK_ARG(sps[j]->device != sps[i]->device,
                         "sa_sp_connect_local: ranks %d and %d share GPU %d (one GPU per rank)", j, i,
                         sps[i]->device);
    }
    for (int i = 0; i < n; ++i) {
        DeviceGuard guard(sps[i]->device);
        for (int j = 0; j < n; ++j) {
            if (j == i) continue;
            int can = 0;
            SA_CUDA_TRY(cudaDeviceCanAccessPeer(&can, sps[i]->device, sps[j]->device));
            SA_CHECK_ARG(can, "sa_sp_connect_local: GPU %d cannot access GPU %d", sps[i]->device,
                         sps[j]->device);
            const cudaError_t e = cudaDeviceEnablePeerAccess(sps[j]->device, 0);
            if (e != cudaSuccess && e != cudaErrorPeerAccessAlreadyEnabled)
                return set_error(SA_ERR_CUDA, "sa_sp_connect_local: peer access %d -> %d: %s", sps[i]->device,
                                 sps[j]->device, cudaGetErrorString(e));
            cudaGetLastError();
        }
    }
    for (int i = 0; i < n; ++i) {
        for (int j = 0; j < n; ++j) sps[i]->peer[j] = sps[j]->words;
        sps[i]->connected = true;
    }
    return SA_OK;
}

SA_API int sa_sp_destroy(sa_sp* sp) {
    using namespace sa;
    clear_error();
    if (!sp) return SA_OK;
    DeviceGuard guard(sp->device);
    cudaDeviceSynchronize();
    sp_close_peers(sp);
    cudaFree(sp->words);
    cudaFree(sp->ctl);
    delete sp;
    return SA_OK;
}

SA_API int sa_attn_decode_sp(sa_sp* sp, int dtype, const void* q, const void* k, const void* v,
                             long long kv_head_stride, int T_local, int d, int hq, int hkv, int block,
                             float scale, float* out, float* m_out, float* l_out, unsigned flags) {
    using namespace sa;
    clear_error();
    SA_CHECK_ARG(sp != nullptr, "sa_attn_decode_sp: sp is NULL");
    SA_CHECK_ARG(sp->connected, "sa_attn_decode_sp: rank %d of %d is not connected (sa_sp_connect)", sp->rank,
                 sp->world);
    SA_CHECK_ARG((m_out == nullptr) == (l_out == nullptr), "sa_attn_decode_sp: m_out/l_out must both be set or NULL");
    SA_CHECK_ARG(hq <= sp->max_hq && d <= sp->max_d, "sa_attn_decode_sp: hq = %d, d = %d exceed the word area's "
                 "max_hq = %d, max_d = %d", hq, d, sp->max_hq, sp->max_d);
    if (sp->world == 1)
        return decode_common("sa_attn_decode_sp", sp->ctx, dtype, q, k, v, kv_head_stride, T_local, d, hq, hkv,
                             block, scale, out, m_out, l_out, flags);
    dec::SpArgs a{};
    a.rank = sp->rank;
    a.world = sp->world;
    for (int r = 0; r < sp->world; ++r) a.words[r] = sp->peer[r];
    a.seq = sp->ctl;
    a.done = sp->ctl + 1;
    return decode_common("sa_attn_decode_sp", sp->ctx, dtype, q, k, v, kv_head_stride, T_local, d, hq, hkv,
                         block, scale, out, m_out, l_out, flags, &a);
}

// ===========================================================================
// fp32 attention of several query rows: ops::self_attention with no mask or
// the causal mask (tensor_cpp/src/ops.cpp:514-641, create_causal_mask
// qwen3_ops.cpp:240-259) and self_attention_streaming_blockwise
// (ops.cpp:1383-1450), fp32 like the reference.  Causal rows whose limit lies
// inside the sequence run on the prompt-attention kernel (head_dim 128); the
// other rows -- full visibility, rows whose limit is past the last key, other
// head sizes -- on the decode kernel's multi-query launch (one CTA per query
// and KV head).
// ===========================================================================
namespace sa {
static int attn_prompt_dev(sa_ctx* ctx, const float* q, const float* k, const float* v, int Sq, int Skv, int q_pos0,
                           int causal, int d, int hq, int hkv, long long qs, long long kvs, float scale, float* out,
                           long long os) {
    const int G = hq / hkv;
    int i0 = 0;
    if (causal && d == 128 && (G == 1 || G == 2 || G == 4 || G == 8 || G == 16)) {
        const int n_causal = std::min(Sq, Skv - q_pos0);   // rows whose last key is inside the sequence
        if (n_causal > 0) {
            SA_RC_TRY(prompt_attn_launch(ctx->stream, ctx->status, q, qs, k, v, kvs,
                                         (long long)(hkv - 1) * (kvs / d) + Skv, q_pos0 + 1, n_causal, d, hq, hkv,
                                         scale, out, os, nullptr, nullptr));
            i0 = n_causal;
        }
    }
    if (i0 >= Sq) return SA_OK;
    dec::KernelFn fn = dec::pick<float>(d, G);
    SA_CHECK_ARG(fn != nullptr, "sa_attn_prompt_f32: hq/hkv = %d at d = %d takes only causal rows inside the "
                 "sequence (d = 128)", G, d);
    SA_CUDA_TRY(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, dec::SMEM_BYTES));
    for (int z0 = i0; z0 < Sq; z0 += 65535) {
        const int nz = std::min(65535, Sq - z0);
        dec::Args a;
        a.q = q + (size_t)z0 * qs;
        a.k = k;
        a.v = v;
        a.kv_head_stride = kvs;
        a.T = causal ? q_pos0 + z0 + 1 : Skv;
        a.hq = hq;
        a.hkv = hkv;
        a.rows_per_split = Skv;                    // one split: query z sees min(T + z*causal, Skv) rows
        a.n_splits = 1;
        a.qscale = scale * dec::LOG2E;
        a.part_m = a.part_l = a.part_o = nullptr;  // one split: no partials
        a.counters = ctx->counters;
        a.out = out + (size_t)z0 * os;
        a.out_m = a.out_l = nullptr;
        a.status = ctx->status;
        a.q_stride = qs;
        a.o_stride = os;
        a.q_causal = causal ? 1 : 0;
        a.kv_early = 0;
        a.len_dev = nullptr;
        a.sp = {};
        a.sp.world = 1;
        fn<<<dim3(1, hkv, nz), dec::THREADS, dec::SMEM_BYTES, ctx->stream>>>(a);
        SA_CUDA_TRY(cudaGetLastError());
    }
    return SA_OK;
}
}  // namespace sa

SA_API int sa_attn_prompt_f32(sa_ctx* ctx, const float* q, const float* k, const float* v, int Sq, int Skv,
                              int q_pos0, int causal, int d, int hq, int hkv, long long q_tok_stride,
                              long long kv_head_stride, float scale, float* out, long long o_tok_stride,
                              unsigned flags) {
    using namespace sa;
    clear_error();
    SA_CHECK_ARG(ctx && q && out && (Skv == 0 || (k && v)), "sa_attn_prompt_f32: null argument");
    SA_CHECK_ARG(Sq >= 1 && Skv >= 1 && q_pos0 >= 0, "sa_attn_prompt_f32: Sq = %d, Skv = %d, q_pos0 = %d", Sq, Skv,
                 q_pos0);
    SA_CHECK_ARG(!causal || q_pos0 < Skv, "sa_attn_prompt_f32: q_pos0 = %d leaves query 0 without keys (Skv = %d)",
                 q_pos0, Skv);
    SA_CHECK_ARG(d == 64 || d == 128 || d == 256, "sa_attn_prompt_f32: d = %d (64, 128, 256)", d);
    SA_CHECK_ARG(hkv >= 1 && hq >= hkv && hq % hkv == 0 && hkv <= 65535, "sa_attn_prompt_f32: hq = %d, hkv = %d", hq,
                 hkv);
    SA_CHECK_ARG(q_tok_stride >= (long long)hq * d && o_tok_stride >= (long long)hq * d &&
                     kv_head_stride >= (long long)Skv * d,
                 "sa_attn_prompt_f32: strides below the row sizes");
    SA_CHECK_ARG(q_tok_stride % 4 == 0 && o_tok_stride % 4 == 0 && kv_head_stride % d == 0,
                 "sa_attn_prompt_f32: strides must be multiples of 4 elements (kv: of d)");
    DeviceGuard guard(ctx->device);
    if (!(flags & SA_HOST_PTRS)) {
        SA_CHECK_ARG((((uintptr_t)q | (uintptr_t)k | (uintptr_t)v | (uintptr_t)out) & 15) == 0,
                     "sa_attn_prompt_f32: pointers must be 16-byte aligned");
        return attn_prompt_dev(ctx, q, k, v, Sq, Skv, q_pos0, causal, d, hq, hkv, q_tok_stride, kv_head_stride,
                               scale, out, o_tok_stride);
    }
    // host buffers: dense device copies, then the output back with its stride
    const size_t row = (size_t)hq * d * 4, kvrow = (size_t)Skv * d * 4;
    const size_t qb = align_up((size_t)Sq * row, 256), kvb = align_up((size_t)hkv * kvrow, 256);
    SA_RC_TRY(ensure_stage(ctx, 2 * qb + 2 * kvb));
    char* base = static_cast<char*>(ctx->stage);
    float* dq = reinterpret_cast<float*>(base);
    float* dk = reinterpret_cast<float*>(base + qb);
    float* dv = reinterpret_cast<float*>(base + qb + kvb);
    float* dout = reinterpret_cast<float*>(base + qb + 2 * kvb);
    cudaStream_t st = ctx->stream;
    SA_CUDA_TRY(cudaMemcpy2DAsync(dq, row, q, (size_t)q_tok_stride * 4, row, Sq, cudaMemcpyHostToDevice, st));
    SA_CUDA_TRY(cudaMemcpy2DAsync(dk, kvrow, k, (size_t)kv_head_stride * 4, kvrow, hkv, cudaMemcpyHostToDevice, st));
    SA_CUDA_TRY(cudaMemcpy2DAsync(dv, kvrow, v, (size_t)kv_head_stride * 4, kvrow, hkv, cudaMemcpyHostToDevice, st));
    SA_RC_TRY(attn_prompt_dev(ctx, dq, dk, dv, Sq, Skv, q_pos0, causal, d, hq, hkv, (long long)hq * d,
                              (long long)Skv * d, scale, dout, (long long)hq * d));
    SA_CUDA_TRY(cudaMemcpy2DAsync(out, (size_t)o_tok_stride * 4, dout, row, row, Sq, cudaMemcpyDeviceToHost, st));
    return sync_and_check(ctx);
}
