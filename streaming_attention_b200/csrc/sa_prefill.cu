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
//  * One CTA per unit of two 128-row query "slots" that read the same K/V
//    tiles: two query heads of one KV group at the same query tile (hq/hkv
//    even), or one head at two neighbouring query tiles (hq/hkv odd).  The two
//    slots' softmaxes alternate with the tensor core: while one slot's
//    softmax runs, the tensor core computes the other slot's P.V and next S.
//  * Warp roles (12 warps): warp 0 issues TMA loads (Q of both slots once; K
//    and V tiles of 128 keys into separate 2-deep rings, 128-byte swizzle);
//    warp 1 owns TMEM and one lane issues every tcgen05.mma; warps 4-7 and
//    8-11 are the softmax warpgroups of slots 0 and 1 (one thread per query
//    row = TMEM lane; warp w reads lanes 32*(w%4)..).  The launch grants 168
//    registers a thread; the first warpgroup gives back down to 72 and the
//    softmax warpgroups take 216 (128*72 + 256*216 = 384*168).
//  * TMEM (512 columns): S of slot x at 128x (128 fp32 columns); P, the bf16
//    probabilities, written back over the upper half of S (64 columns of bf16
//    pairs); O of slot x at 256 + 128x.
//  * S = Q K^T: M=128, N=128, K=128 (8 MMAs of K=16, A and B K-major from
//    shared memory).  O += P V: M=128, N=128, K=128 (8 MMAs), A = P read from
//    TMEM, B = V MN-major from shared memory (the V tile as loaded: keys x d).
//    S of the next tile overwrites the TMEM columns that the P.V just issued
//    reads P from; it is issued right behind that P.V by the same thread, and
//    the tensor core executes one thread's MMAs in issue order (the same
//    reliance as NVIDIA's CUTLASS sm100 FMHA forward mainloop, which issues
//    P.V and the next Q.K^T over shared TMEM columns back to back).  The
//    commit that signals S(j+1) also covers the P.V of tile j, so the softmax
//    may rescale O as soon as it sees S(j+1).
//  * Online softmax in the exp2 domain (scale*log2 e folded into the scores)
//    with a lazy rescale: the running max used for the exponent only moves
//    when a row's max grows by more than 8 (2^8 headroom in P), and only then
//    is the row's O accumulator in TMEM loaded, scaled and stored back.  From
//    the second tile on, the exponentials are computed speculatively against
//    the running max while the tile's max is found in the same pass; the
//    warp redoes the tile only when one of its rows crossed the threshold,
//    which keeps the max reduction off the softmax's critical path.  The
//    kernel can evaluate a fraction of the exponentials on the FMA pipe
//    (exp2_poly, template parameter POLY); the shipped instance keeps them all
//    on the SFU, which measured fastest.
//  * Causal: a slot's KV range stops at the last key its last row may see;
//    only tiles crossing the diagonal are masked.  Heavy (late) query tiles
//    are scheduled first.
//  * Every mbarrier wait is bounded; a timeout sets the status word, stops all
//    roles, lets in-flight copies and MMAs land, frees TMEM and returns.
#include <cuda_bf16.h>
#include <cmath>

#include "sa_internal.h"
#include "sa_qwen3.h"
#include "sa_tc.cuh"

namespace sa {
namespace pf {

constexpr int BM = 128, BN = 128, D = 128;
constexpr int KST = 2, VST = 2;                // K and V ring depths
constexpr int THREADS = 384;
constexpr int REG_CTRL = 72, REG_SOFTMAX = 216;   // 128*72 + 256*216 == THREADS*168
constexpr int BOX_BYTES = 128 * 128;           // one [128 rows x 64 bf16] box (16 KB)
constexpr int TILE_BYTES = 2 * BOX_BYTES;      // a [128 x 128] bf16 tile as two boxes
constexpr int OFF_Q = 0;                       // slot x at OFF_Q + x * TILE_BYTES
constexpr int OFF_K = 2 * TILE_BYTES;
constexpr int OFF_V = OFF_K + KST * TILE_BYTES;
constexpr int OFF_BAR = OFF_V + VST * TILE_BYTES;  // 196608
constexpr int SMEM_BYTES = OFF_BAR + 256 + 1024;   // + barriers + alignment slack
constexpr uint32_t TMEM_COLS = 512;
__device__ __forceinline__ uint32_t col_s(int x) { return (uint32_t)x * 128u; }
__device__ __forceinline__ uint32_t col_p(int x) { return (uint32_t)x * 128u + 64u; }
__device__ __forceinline__ uint32_t col_o(int x) { return 256u + (uint32_t)x * 128u; }
constexpr float LOG2E = 1.4426950408889634f;
constexpr float RESCALE_THRESHOLD = 8.0f;      // log2 units

// One launch covers up to MAX_PIECES "pieces": a block of Sq query rows
// (rows q_row0.. of the Q tensor) against a block of Skv keys (rows kv_row0..
// of the K/V tensors), query i seeing key j of the block when j <= q_pos0 + i.
// A sequence-parallel rank splits its long causal key ranges into pieces of
// similar length (so no CTA carries a whole row's keys) and merges them by
// their log-sum-exp; a plain prefill is one piece.
constexpr int MAX_PIECES = kPrefillMaxPieces;
struct Piece {
    int q_row0, kv_row0;
    int Sq, Skv, q_pos0;
    int n_qtiles;
    int cta0;                   // first CTA of the piece
    void* out;                  // [Sq] rows at o_tok; bf16 or fp32 (Args::out_bf16)
    float* lse;                 // [Sq][hq] log2-domain log-sum-exp of the scaled scores, or null
};

struct Args {
    int hq, hkv, G;
    int pair_heads;             // 1: slots are heads (h, h+1) of one q tile; 0: q tiles (2p, 2p+1) of one head
    int units_per_row;          // units per heavy-first row of the schedule
    float sl2;                  // scale * log2(e)
    void* out_lo;               // bf16 output of a one-piece launch: the rounding remainder, bf16(o - out)
    long long o_tok, o_head;    // element strides of the outputs (and out_lo)
    int out_bf16;
    int n_pieces;
    Piece pc[MAX_PIECES];
    int* status;
};

struct Bars {
    uint64_t q_full;
    uint64_t k_full[KST], k_empty[KST], v_full[VST], v_empty[VST];
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

// 2^x on the FMA pipe, for x <= 8 (clamped below at -126): x = n + f with n
// the nearest integer (taken from the low mantissa bits of x + 1.5*2^23) and
// f in [-0.5, 0.5]; 2^f by a degree-3 polynomial fitted here to 2^f on that
// interval (max relative error 7.5e-5, far below the bf16 rounding of P);
// 2^n added to the exponent field with an integer add.  No transcendental-
// unit instruction is used.
__device__ __forceinline__ float exp2_poly(float x) {
    x = fmaxf(x, -126.f);
    const float t = x + 12582912.f;
    const float f = x - (t - 12582912.f);
    float p = fmaf(0.0551716685295105f, f, 0.2426111251115799f);
    p = fmaf(p, f, 0.6932609677314758f);
    p = fmaf(p, f, 0.9999280571937561f);
    return __int_as_float(__float_as_int(p) + (__float_as_int(t) << 23));
}

// Every POLY-th exponential (by column) on the FMA pipe; 0: all on the SFU.
template <int POLY>
__device__ __forceinline__ float exp2_mix(float x, int c) {
    if constexpr (POLY > 0) {
        if ((c % POLY) == POLY - 1) return exp2_poly(x);
    }
    return ex2(x);
}

// Max of a row's 128 raw scores (eight independent chains).
__device__ __forceinline__ float row_max(const float* sc) {
    float mx[8];
#pragma unroll
    for (int c = 0; c < 8; ++c) mx[c] = sc[c];
#pragma unroll
    for (int c = 8; c < BN; c += 8)
#pragma unroll
        for (int i = 0; i < 8; ++i) mx[i] = fmaxf(mx[i], sc[c + i]);
    return fmaxf(fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])), fmaxf(fmaxf(mx[4], mx[5]), fmaxf(mx[6], mx[7])));
}

// P = 2^(sc*sl2 + nm) for one row's 128 scores, written to TMEM at p_addr as
// 64 columns of bf16 pairs (two tcgen05.st of 32 columns, not waited for);
// returns the fp32 row sum.  With TRACK_MAX the max of the raw scores is
// found in the same pass and written to *mx_out.
template <int POLY, bool TRACK_MAX>
__device__ __forceinline__ float emit_p(const float* sc, float sl2, float nm, uint32_t p_addr, float* mx_out) {
    float ps[4] = {0.f, 0.f, 0.f, 0.f};
    float mx[8];
    if constexpr (TRACK_MAX) {
#pragma unroll
        for (int i = 0; i < 8; ++i) mx[i] = sc[i];
    }
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {
        uint32_t pk[32];
#pragma unroll
        for (int c = hf * 64; c < hf * 64 + 64; c += 2) {
            if constexpr (TRACK_MAX) {
                mx[c & 7] = fmaxf(mx[c & 7], sc[c]);
                mx[(c + 1) & 7] = fmaxf(mx[(c + 1) & 7], sc[c + 1]);
            }
            const float e0 = exp2_mix<POLY>(fmaf(sc[c], sl2, nm), c);
            const float e1 = exp2_mix<POLY>(fmaf(sc[c + 1], sl2, nm), c + 1);
            ps[(c >> 1) & 3] += e0 + e1;
            pk[(c >> 1) & 31] = pack_bf16(e0, e1);
        }
        tc::tmem_st32(p_addr + hf * 32, pk);
    }
    if constexpr (TRACK_MAX)
        *mx_out = fmaxf(fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])), fmaxf(fmaxf(mx[4], mx[5]), fmaxf(mx[6], mx[7])));
    return (ps[0] + ps[1]) + (ps[2] + ps[3]);
}

template <int POLY>
__global__ void __launch_bounds__(THREADS, 1)
prefill_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
               const __grid_constant__ CUtensorMap tv, const __grid_constant__ Args a) {
    extern __shared__ unsigned char smem_raw[];
    // 1024-byte alignment for the 128-byte-swizzled operand tiles
    const uint32_t raw = smem_u32(smem_raw);
    unsigned char* sm = smem_raw + (((raw + 1023u) & ~1023u) - raw);
    Bars* B = reinterpret_cast<Bars*>(sm + OFF_BAR);
    volatile int* abort = &B->abort;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    // ---- this CTA's piece, then its unit: heads, first query rows and KV
    // extent of its two slots
    int pi = 0;
    while (pi + 1 < a.n_pieces && (int)blockIdx.x >= a.pc[pi + 1].cta0) ++pi;
    const Piece P = a.pc[pi];      // in registers: the softmax loop reads its bounds every tile
    const int local = (int)blockIdx.x - P.cta0;
    const int rowi = local / a.units_per_row;
    const int u = local % a.units_per_row;
    int head[2], q0[2], nkv[2];
    bool on[2];
    int kvh;
    if (a.pair_heads) {
        const int qt = P.n_qtiles - 1 - rowi;                       // heavy tiles first
        const int upk = a.G / 2;
        kvh = u / upk;
        head[0] = kvh * a.G + 2 * (u % upk);
        head[1] = head[0] + 1;
        q0[0] = q0[1] = qt * BM;
        on[0] = on[1] = true;
    } else {
        const int n_pairs = (P.n_qtiles + 1) / 2;
        const int qp = n_pairs - 1 - rowi;
        head[0] = head[1] = u;
        kvh = u / a.G;
        q0[0] = 2 * qp * BM;
        q0[1] = q0[0] + BM;
        on[0] = true;
        on[1] = q0[1] < P.Sq;
    }
    for (int x = 0; x < 2; ++x) {
        const int last_row = min(q0[x] + BM - 1, P.Sq - 1);
        const int last_key = min(P.Skv - 1, P.q_pos0 + last_row);
        nkv[x] = on[x] ? last_key / BN + 1 : 0;
    }
    const int n_kv = max(nkv[0], nkv[1]);

    if (tid == 0) {
        mbar_init(&B->q_full, 1);
        for (int s = 0; s < KST; ++s) {
            mbar_init(&B->k_full[s], 1);
            mbar_init(&B->k_empty[s], 1);
        }
        for (int s = 0; s < VST; ++s) {
            mbar_init(&B->v_full[s], 1);
            mbar_init(&B->v_empty[s], 1);
        }
        for (int x = 0; x < 2; ++x) {
            mbar_init(&B->s_full[x], 1);
            mbar_init(&B->p_full[x], 4);      // one arrival per softmax warp
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

    if (warp < 4) {
      asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(REG_CTRL));
      if (warp == 0) {
        // ------------------------------------------------ TMA producer
        if (lane == 0) {
            tc::prefetch_tmap(&tq);
            tc::prefetch_tmap(&tk);
            tc::prefetch_tmap(&tv);
            mbar_arrive_expect_tx(&B->q_full, (on[1] ? 2 : 1) * TILE_BYTES);
            for (int x = 0; x < 2; ++x) {
                if (!on[x]) continue;
                for (int kb = 0; kb < 2; ++kb)
                    tc::tma_load_2d(sm + OFF_Q + x * TILE_BYTES + kb * BOX_BYTES, &tq, head[x] * D + kb * 64,
                                    P.q_row0 + q0[x], &B->q_full);
            }
            int k_issued = 0, v_issued = 0;
            for (int j = 0; j < n_kv; ++j) {
                const int ks = j % KST, vs = j % VST;
                if (j >= KST && !wait_ab(&B->k_empty[ks], ((j / KST) & 1) ^ 1, abort, a.status)) break;
                mbar_arrive_expect_tx(&B->k_full[ks], TILE_BYTES);
                for (int kb = 0; kb < 2; ++kb)
                    tc::tma_load_2d(sm + OFF_K + ks * TILE_BYTES + kb * BOX_BYTES, &tk, kvh * D + kb * 64,
                                    P.kv_row0 + j * BN, &B->k_full[ks]);
                k_issued = j + 1;
                if (j >= VST && !wait_ab(&B->v_empty[vs], ((j / VST) & 1) ^ 1, abort, a.status)) break;
                mbar_arrive_expect_tx(&B->v_full[vs], TILE_BYTES);
                for (int kb = 0; kb < 2; ++kb)
                    tc::tma_load_2d(sm + OFF_V + vs * TILE_BYTES + kb * BOX_BYTES, &tv, kvh * D + kb * 64,
                                    P.kv_row0 + j * BN, &B->v_full[vs]);
                v_issued = j + 1;
            }
            if (*abort) {
                // let the loads still in flight land before the CTA exits
                mbar_wait(&B->q_full, 0, nullptr);
                for (int j = max(0, k_issued - KST); j < k_issued; ++j)
                    mbar_wait(&B->k_full[j % KST], (j / KST) & 1, nullptr);
                for (int j = max(0, v_issued - VST); j < v_issued; ++j)
                    mbar_wait(&B->v_full[j % VST], (j / VST) & 1, nullptr);
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------ MMA issuer
        // Per KV tile j and slot x: P.V(j) once the slot's P is in TMEM, then
        // S(j+1) over the same TMEM columns, issued right behind it.  The
        // other slot's softmax runs meanwhile.
        if (lane == 0) {
            constexpr uint32_t idS = tc::idesc_bf16_f32(BM, BN, false, false);
            constexpr uint32_t idO = tc::idesc_bf16_f32(BM, D, false, true);
            const uint32_t sQ = smem_u32(sm + OFF_Q), sK = smem_u32(sm + OFF_K), sV = smem_u32(sm + OFF_V);
            auto act = [&](int x, int j) { return j < nkv[x]; };
            auto issue_S = [&](int x, int j) {
                const uint32_t q = sQ + x * TILE_BYTES, k = sK + (j % KST) * TILE_BYTES;
#pragma unroll
                for (int kk = 0; kk < D / 16; ++kk) {
                    const uint32_t off = (kk >> 2) * BOX_BYTES + (kk & 3) * 32;
                    tc::mma_bf16(tbase + col_s(x), tc::sdesc_sw128(q + off, 16, 1024),
                                 tc::sdesc_sw128(k + off, 16, 1024), idS, kk > 0);
                }
            };
            auto issue_PV = [&](int x, int j) {
                const uint32_t v = sV + (j % VST) * TILE_BYTES;
#pragma unroll
                for (int kk = 0; kk < BN / 16; ++kk)
                    tc::mma_bf16_ts(tbase + col_o(x), tbase + col_p(x) + kk * 8,
                                    tc::sdesc_sw128(v + kk * 2048, BOX_BYTES, 1024), idO,
                                    (j > 0 || kk > 0) ? 1u : 0u);
            };
            bool ok = wait_ab(&B->q_full, 0, abort, a.status) && wait_ab(&B->k_full[0], 0, abort, a.status);
            tc::fence_after_sync();
            if (ok) {
                for (int x = 0; x < 2; ++x)
                    if (act(x, 0)) {
                        issue_S(x, 0);
                        tc::mma_commit(&B->s_full[x]);
                    }
                tc::mma_commit(&B->k_empty[0]);
            }
            for (int j = 0; ok && j < n_kv; ++j) {
                if (!(ok = wait_ab(&B->v_full[j % VST], (j / VST) & 1, abort, a.status))) break;
                bool k_next = false;
                for (int x = 0; ok && x < 2; ++x) {
                    if (!act(x, j)) continue;
                    if (!(ok = wait_ab(&B->p_full[x], j & 1, abort, a.status))) break;
                    tc::fence_after_sync();
                    issue_PV(x, j);
                    if (j + 1 == nkv[x]) {
                        tc::mma_commit(&B->o_full[x]);
                        continue;
                    }
                    if (!k_next) {
                        const int j1 = j + 1;
                        if (!(ok = wait_ab(&B->k_full[j1 % KST], (j1 / KST) & 1, abort, a.status))) break;
                        k_next = true;
                    }
                    issue_S(x, j + 1);
                    tc::mma_commit(&B->s_full[x]);
                }
                if (!ok) break;
                tc::mma_commit(&B->v_empty[j % VST]);
                if (k_next) tc::mma_commit(&B->k_empty[(j + 1) % KST]);
            }
            // all issued MMAs complete before TMEM is released
            tc::mma_commit(&B->drain);
            mbar_wait(&B->drain, 0, nullptr);
        }
      }
    } else {
        asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(REG_SOFTMAX));
        // ------------------------------------------------ softmax warpgroups
        const int x = (warp - 4) >> 2;
        const bool my_on = x ? on[1] : on[0];
        const int my_q0 = x ? q0[1] : q0[0], my_nkv = x ? nkv[1] : nkv[0], h = x ? head[1] : head[0];
        if (my_on) {
            const int quad = warp & 3;
            const int row = quad * 32 + lane;
            const uint32_t lane_addr = tbase + ((uint32_t)(quad * 32) << 16);
            const int qrow = my_q0 + row;
            const int limit = P.q_pos0 + qrow;          // last visible key of this row
            const float sl2 = a.sl2;
            float m = -INFINITY, l = 0.f;               // m in scaled log2 units
            bool ok = true;
            for (int j = 0; j < my_nkv; ++j) {
                if (!(ok = wait_ab(&B->s_full[x], j & 1, abort, a.status))) break;
                tc::fence_after_sync();
                uint32_t u32[BN];
#pragma unroll
                for (int cb = 0; cb < BN / 32; ++cb) tc::tmem_ld32p(lane_addr + col_s(x) + cb * 32, u32 + cb * 32);
                tc::tmem_wait_ld();
                float* sc = reinterpret_cast<float*>(u32);
                const int k0 = j * BN;
                if (k0 + BN - 1 > P.q_pos0 + my_q0 || k0 + BN > P.Skv) {
#pragma unroll
                    for (int c = 0; c < BN; ++c)
                        if (k0 + c > limit || k0 + c >= P.Skv) sc[c] = -INFINITY;
                }
                const uint32_t p_addr = lane_addr + col_p(x);
                float alpha = 1.f, sum;
                if (j == 0) {
                    // first tile: every row sees key 0, so its max is finite
                    const float mxs = row_max(sc) * sl2;
                    m = mxs;
                    sum = emit_p<POLY, false>(sc, sl2, (m == -INFINITY) ? 0.f : -m, p_addr, nullptr);
                } else {
                    // speculative: exponentials against the running max while the
                    // tile's max is found in the same pass; redone only if some row's
                    // max grew by more than the rescale threshold
                    float mxr;
                    sum = emit_p<POLY, true>(sc, sl2, -m, p_addr, &mxr);
                    const float mxs = mxr * sl2;
                    const bool need = mxs > m + RESCALE_THRESHOLD;
                    if (__any_sync(0xffffffffu, need)) {
                        if (need) {
                            alpha = ex2(m - mxs);
                            m = mxs;
                        }
                        // rescale this row's O accumulator (warp-collective TMEM
                        // access); the P.V of tile j-1 completed before S(j) was issued
#pragma unroll 1
                        for (int cb = 0; cb < D / 32; ++cb) {
                            uint32_t o[32];
                            tc::tmem_ld32(lane_addr + col_o(x) + cb * 32, o);
                            tc::tmem_wait_ld();
#pragma unroll
                            for (int c = 0; c < 32; ++c) o[c] = __float_as_uint(__uint_as_float(o[c]) * alpha);
                            tc::tmem_st32(lane_addr + col_o(x) + cb * 32, o);
                        }
                        tc::tmem_wait_st();        // the first P stores land before they are replaced
                        sum = emit_p<POLY, false>(sc, sl2, -m, p_addr, nullptr);
                    }
                }
                l = l * alpha + sum;
                tc::tmem_wait_st();
                tc::fence_before_sync();
                __syncwarp();
                if (lane == 0) mbar_arrive(&B->p_full[x]);
            }
            if (ok && wait_ab(&B->o_full[x], 0, abort, a.status)) {
                tc::fence_after_sync();
                const float inv = l > 0.f ? 1.f / l : 0.f;
                const bool store = qrow < P.Sq;
                if (store && P.lse) P.lse[(size_t)qrow * a.hq + h] = l > 0.f ? m + log2f(l) : -INFINITY;
#pragma unroll 1
                for (int cb = 0; cb < D / 32; ++cb) {
                    uint32_t o[32];
                    tc::tmem_ld32(lane_addr + col_o(x) + cb * 32, o);
                    tc::tmem_wait_ld();
                    if (!store) continue;
                    if (a.out_bf16) {
                        const size_t off = (size_t)qrow * a.o_tok + (size_t)h * a.o_head + cb * 32;
                        __nv_bfloat16* dst = static_cast<__nv_bfloat16*>(P.out) + off;
                        __nv_bfloat16* dlo = a.out_lo ? static_cast<__nv_bfloat16*>(a.out_lo) + off : nullptr;
#pragma unroll
                        for (int c = 0; c < 32; c += 8) {
                            float f[8];
#pragma unroll
                            for (int j = 0; j < 8; ++j) f[j] = __uint_as_float(o[c + j]) * inv;
                            uint4 v;
                            v.x = pack_bf16(f[0], f[1]);
                            v.y = pack_bf16(f[2], f[3]);
                            v.z = pack_bf16(f[4], f[5]);
                            v.w = pack_bf16(f[6], f[7]);
                            *reinterpret_cast<uint4*>(dst + c) = v;
                            if (dlo) {   // remainders after the bf16 rounding above
                                const uint32_t hv[4] = {v.x, v.y, v.z, v.w};
                                uint32_t lv[4];
#pragma unroll
                                for (int j = 0; j < 4; ++j)
                                    lv[j] = pack_bf16(f[2 * j] - __uint_as_float(hv[j] << 16),
                                                      f[2 * j + 1] - __uint_as_float(hv[j] & 0xffff0000u));
                                *reinterpret_cast<uint4*>(dlo + c) = make_uint4(lv[0], lv[1], lv[2], lv[3]);
                            }
                        }
                    } else {
                        float* dst = static_cast<float*>(P.out) + (size_t)qrow * a.o_tok + (size_t)h * a.o_head +
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

// Launch the prefill over a table of pieces (PrefillPiece in sa_qwen3.h):
//   q    [q_rows,  q_tok stride,  hq heads of 128]   bf16
//   k,v  [kv_rows, kv_tok stride, hkv heads of 128]  bf16
// each piece's output [Sq rows, o_tok stride, hq heads of 128] in out_dtype.
int prefill_pieces_launch(cudaStream_t st, int* status, const void* q, int q_rows, long long q_tok, const void* k,
                          const void* v, int kv_rows, long long kv_tok, int hq, int hkv, float scale, int out_dtype,
                          long long o_tok, const PrefillPiece* pieces, int n, void* out_lo) {
    SA_CHECK_ARG(n >= 1 && n <= pf::MAX_PIECES && hkv >= 1 && hq % hkv == 0 && (n == 1 || !out_lo),
                 "prefill: %d pieces, hq %d, hkv %d", n, hq, hkv);
    CUtensorMap mq, mk, mv;
    int rc = make_tmap_2d_bf16(&mq, q, (uint64_t)q_rows, (uint64_t)hq * pf::D, (uint64_t)q_tok, pf::BM, 64);
    if (!rc) rc = make_tmap_2d_bf16(&mk, k, (uint64_t)kv_rows, (uint64_t)hkv * pf::D, (uint64_t)kv_tok, pf::BN, 64);
    if (!rc) rc = make_tmap_2d_bf16(&mv, v, (uint64_t)kv_rows, (uint64_t)hkv * pf::D, (uint64_t)kv_tok, pf::BN, 64);
    if (rc) return rc;
    pf::Args a;
    a.hq = hq; a.hkv = hkv; a.G = hq / hkv;
    a.pair_heads = (a.G % 2 == 0) ? 1 : 0;
    a.units_per_row = a.pair_heads ? hkv * (a.G / 2) : hq;
    a.sl2 = scale * pf::LOG2E;
    a.o_tok = o_tok; a.o_head = pf::D;
    a.out_bf16 = out_dtype == SA_BF16;
    a.out_lo = a.out_bf16 ? out_lo : nullptr;
    a.status = status;
    a.n_pieces = n;
    int grid = 0;
    for (int i = 0; i < n; ++i) {
        const PrefillPiece& s = pieces[i];
        SA_CHECK_ARG(s.Sq >= 1 && s.Skv >= 1 && s.q_pos0 >= 0 && s.q_row0 >= 0 && s.kv_row0 >= 0 &&
                         s.q_row0 + s.Sq <= q_rows && s.kv_row0 + s.Skv <= kv_rows && s.out,
                     "prefill: piece %d (q rows %d+%d of %d, keys %d+%d of %d)", i, s.q_row0, s.Sq, q_rows, s.kv_row0,
                     s.Skv, kv_rows);
        pf::Piece& P = a.pc[i];
        P.q_row0 = s.q_row0; P.kv_row0 = s.kv_row0;
        P.Sq = s.Sq; P.Skv = s.Skv; P.q_pos0 = s.q_pos0;
        P.n_qtiles = (s.Sq + pf::BM - 1) / pf::BM;
        P.cta0 = grid;
        P.out = s.out;
        P.lse = s.lse;
        const int rows = a.pair_heads ? P.n_qtiles : (P.n_qtiles + 1) / 2;
        grid += rows * a.units_per_row;
    }
    // All exponentials on the SFU: with 128-key tiles the softmax is issue-bound,
    // and moving every 8th/4th/3rd exponential to exp2_poly measured 3%/5%/9%
    // slower on config 3 (S=8192, 16/8 heads).
    auto kern = pf::prefill_kernel<0>;
    SA_RC_TRY(set_smem_attr_once((const void*)kern, pf::SMEM_BYTES));
    kern<<<grid, pf::THREADS, pf::SMEM_BYTES, st>>>(mq, mk, mv, a);
    SA_CUDA_TRY(cudaGetLastError());
    return SA_OK;
}

// Launch the causal prefill on device pointers (one piece).
//   q   [Sq,  q_tok stride,  hq heads of 128]   bf16
//   k,v [Skv, kv_tok stride, hkv heads of 128]  bf16
//   out [Sq,  o_tok stride,  hq heads of 128]   fp32 or bf16
int prefill_launch(cudaStream_t st, int* status, const void* q, const void* k, const void* v, void* out,
                   int out_dtype, int Sq, int Skv, int q_pos0, int hq, int hkv, long long q_tok, long long kv_tok,
                   long long o_tok, float scale, void* out_lo) {
    PrefillPiece p;
    p.q_row0 = 0; p.kv_row0 = 0;
    p.Sq = Sq; p.Skv = Skv; p.q_pos0 = q_pos0;
    p.out = out;
    p.lse = nullptr;
    return prefill_pieces_launch(st, status, q, Sq, q_tok, k, v, Skv, kv_tok, hq, hkv, scale, out_dtype, o_tok, &p, 1,
                                 out_lo);
}

static int launch_prefill(sa_ctx* ctx, const void* q, const void* k, const void* v, void* out, int out_dtype,
                          int Sq, int Skv, int q_pos0, int hq, int hkv, long long q_tok, long long kv_tok,
                          long long o_tok, float scale) {
    return prefill_launch(ctx->stream, ctx->status, q, k, v, out, out_dtype, Sq, Skv, q_pos0, hq, hkv, q_tok,
                          kv_tok, o_tok, scale);
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
    SA_CHECK_ARG(out_dtype == SA_F32 || out_dtype == SA_BF16, "sa_attn_prefill: out_dtype %d", out_dtype);
    SA_CHECK_ARG(q_tok_stride >= (long long)hq * d && kv_tok_stride >= (long long)hkv * d &&
                 o_tok_stride >= (long long)hq * d, "sa_attn_prefill: token strides too small");
    SA_CHECK_ARG(((uintptr_t)out & 15) == 0, "sa_attn_prefill: out not 16-byte aligned");
    SA_CHECK_ARG(!(flags & SA_HOST_PTRS), "sa_attn_prefill: host pointers are not supported (pass device memory)");
    DeviceGuard guard(ctx->device);
    return launch_prefill(ctx, q, k, v, out, out_dtype, Sq, Skv, q_pos0, hq, hkv, q_tok_stride, kv_tok_stride,
                          o_tok_stride, scale);
}
