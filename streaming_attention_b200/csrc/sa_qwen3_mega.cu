// sa_qwen3_mega.cu -- the single-token Qwen3 decode step as one persistent
// kernel: every layer's RMSNorm + QKV projection, QK-norm + RoPE + KV-cache
// append + attention, o_proj + residual, RMSNorm + gate/up + SwiGLU,
// down_proj + residual, then the final norm, lm_head and argmax, for one
// token, in one cooperative launch with one CTA per SM.
//
// Replaces, for greedy decode, the per-token sequence of qwen3_forward_with_cache
// (tensor_cpp/src/qwen3_ops.cpp:936-1014 -> qwen3_decoder_layer_with_cache
// :620-934) followed by ops::argmax (ops.cpp:213-272) over the last logits.
//
// Opt-in (SA_QWEN3_MEGA=1; see mega_supported for the measured comparison).
// Why one kernel: a decode step moves 1.19 GB of weights but is a chain of
// ~170 small dependent operations; as separate kernels each pays launch and
// first-byte latency and the weight stream stops between them.  Here each CTA
// owns a fixed part of every weight matrix and streams those rows, in step
// order, through a ring of shared-memory slots with 1-D bulk copies
// (sa_mega_plan.h is the schedule).  The copies run ahead of the computation
// across phase boundaries, so HBM keeps streaming while CTAs wait at the grid
// barriers that separate the dependent phases:
//   A  QKV GEMV over RMSNorm(x)                    -> qkv
//   B  QK-norm + RoPE, KV-cache append, attention  -> attn   (split-KV, the
//      last CTA of each KV head merges the splits' (m, l, O))
//   C  o_proj GEMV, residual add                   -> x
//   D  gate/up GEMV over RMSNorm(x), SwiGLU        -> act
//   E  down_proj GEMV, residual add                -> x
//   F  (after the last layer) final RMSNorm, lm_head GEMV, argmax -> next token
// Activations written by other CTAs are read through L2 (ld.global.cg); the
// grid barrier is a counter plus generation word with a release fence before
// arriving; every wait (ring slot, barrier) is bounded by %globaltimer and an
// expired wait sets the status word and an abort flag that stops all CTAs,
// which let their in-flight copies land before returning.
// Numerics are those of the multi-kernel path: bf16 weights, fp32 activations,
// residual stream and KV cache, exp2-domain online softmax.
#include <cuda_bf16.h>
#include <cmath>
#include <cstdlib>

#include "sa_internal.h"
#include "sa_mega_plan.h"
#include "sa_ptx.cuh"
#include "sa_qwen3.h"
#include "sa_tc.cuh"

namespace sa {
namespace mk {

constexpr int THREADS = 512, NWARP = THREADS / 32;
constexpr int SLOT_BYTES = 12288, NSLOT = 16;   // one slot per warp
constexpr int MAXR = 6;                          // rows a 12 KB slot holds at most (hidden >= 1024 rows)
constexpr int ROWS_PER_SPLIT = 128;              // attention: cached rows per CTA
constexpr int D = 128;
constexpr int XS_FLOATS = 3072;      // largest activation vector (hidden, q dim or inter)
constexpr int MAXG = 2;              // query heads per KV head
constexpr int RED_FLOATS = NWARP * MAXG * (D + 2);
constexpr int OFF_RING = 0;
constexpr int OFF_XS = OFF_RING + NSLOT * SLOT_BYTES;
constexpr int OFF_RED = OFF_XS + XS_FLOATS * 4;
constexpr int OFF_RES = OFF_RED + RED_FLOATS * 4;
constexpr int OFF_QK = OFF_RES + 32 * 4;
constexpr int OFF_BAR = OFF_QK + (MAXG + 2) * D * 4;
constexpr int OFF_MISC = OFF_BAR + NSLOT * 8;
constexpr int SMEM_BYTES = OFF_MISC + 64 + 128;   // + alignment slack

struct Args {
    Plan plan;
    const MegaLayer* layers;   // [L]
    int hq, hkv, G, max_seq, splits;
    float eps, qscale;         // RMSNorm eps; log2(e) / sqrt(head_dim)
    const __nv_bfloat16* embed;
    const __nv_bfloat16* lm_head;
    const float* final_norm;
    float* kc;
    float* vc;
    const float* cos_t;
    const float* sin_t;
    float* x;
    float* qkv;
    float* attn;
    float* act;
    float* part;                // [hkv][splits][G][D + 2]
    unsigned* head_cnt;         // [hkv], zero between launches
    unsigned long long* amax;   // zero between launches
    unsigned* gbar;             // [0] arrivals, [1] generation, [2] abort
    int* state;                 // [0] position of the token, [1] tokens generated
    int64_t* ids;               // [0] the token to forward; receives the next one
    int64_t* toks;
    int toks_cap;
    int* status;
};

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ uint32_t ordered_f32(float f) {
    const uint32_t u = __float_as_uint(f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__device__ __forceinline__ bool aborted(const Args& a) { return *(volatile unsigned*)(a.gbar + 2) != 0u; }

__device__ __forceinline__ void raise_abort(const Args& a) {
    atomicExch(a.status, SA_STATUS_TIMEOUT);
    atomicExch(a.gbar + 2, 1u);
}

__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ unsigned atom_add_acq_rel(unsigned* p, unsigned v) {
    unsigned old;
    asm volatile("atom.add.acq_rel.gpu.global.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}

// All CTAs of the grid reach this point; false if the step was aborted.
// Arrival is an acquire-release add on the counter (the CTA's writes, ordered
// before thread 0 by the CTA barrier, are released with it); the last CTA
// resets the counter and releases the generation word the others acquire.
__device__ bool grid_sync(const Args& a, int* flag) {
    __syncthreads();
    if (threadIdx.x == 0) {
        bool ok = true;
        unsigned* cnt = a.gbar;
        unsigned* gen = a.gbar + 1;
        const unsigned g = ld_acquire(gen);
        if (atom_add_acq_rel(cnt, 1u) == gridDim.x - 1) {
            asm volatile("st.relaxed.gpu.global.u32 [%0], %1;" ::"l"(cnt), "r"(0u) : "memory");
            asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(gen), "r"(1u) : "memory");
        } else {
            const unsigned long long t0 = globaltimer();
            for (unsigned it = 1; ld_acquire(gen) == g; ++it) {
                if ((it & 255u) == 0u) {
                    if (aborted(a)) { ok = false; break; }
                    if (globaltimer() - t0 > kWaitLimitNs) {
                        raise_abort(a);
                        ok = false;
                        break;
                    }
                }
            }
        }
        *flag = ok ? 1 : 0;
    }
    __syncthreads();
    return *flag != 0;
}

// Wait for a warp's ring slot; the outcome is the same for every lane (lane
// 0 waits with the time limit and shares the result, the others then observe
// the completed phase themselves).
__device__ bool wait_slot_warp(const Args& a, uint64_t* bar, uint32_t parity) {
    int ok = 0;
    if ((threadIdx.x & 31) == 0) {
        ok = mbar_try_wait(bar, parity);
        if (!ok) {
            const unsigned long long t0 = globaltimer();
            while (!(ok = mbar_try_wait(bar, parity))) {
                if (aborted(a)) break;
                if (globaltimer() - t0 > kWaitLimitNs) {
                    raise_abort(a);
                    break;
                }
            }
        }
    }
    ok = __shfl_sync(0xffffffffu, ok, 0);
    if (!ok) return false;
    return mbar_wait(bar, parity, nullptr);   // already complete: returns at once
}

__device__ __forceinline__ const __nv_bfloat16* matrix_of(const Args& a, const Job& j) {
    if (j.phase == PH_F) return a.lm_head;
    const MegaLayer& L = a.layers[j.layer];
    return j.phase == PH_A ? L.wqkv : j.phase == PH_C ? L.wo : j.phase == PH_D ? L.wgu : L.wd;
}

__device__ __forceinline__ void issue(const Args& a, const Job& j, unsigned char* slot, uint64_t* bar,
                                      uint64_t policy) {
    const __nv_bfloat16* m = matrix_of(a, j);
    fence_proxy_async_smem();                          // the slot's previous reads come first
    mbar_arrive_expect_tx(bar, (uint32_t)(j.bytes0 + j.bytes1));
    bulk_g2s_hint(slot, m + j.src0, (uint32_t)j.bytes0, bar, policy);
    if (j.bytes1) bulk_g2s_hint(slot + j.bytes0, m + j.src1, (uint32_t)j.bytes1, bar, policy);
}

// xs[i] = v[i] * rsqrt(mean(v^2) + eps) * gain[i] for v read from global
// (through L2); gain == nullptr: xs = v.
__device__ void load_act(const Args& a, const float* v, int n, const float* gain, float* xs, float* red) {
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
    float ss = 0.f;
    for (int i = t; i < n / 4; i += THREADS) {
        const float4 q = __ldcg(reinterpret_cast<const float4*>(v) + i);
        reinterpret_cast<float4*>(xs)[i] = q;
        ss = fmaf(q.x, q.x, fmaf(q.y, q.y, fmaf(q.z, q.z, fmaf(q.w, q.w, ss))));
    }
    if (!gain) {
        __syncthreads();
        return;
    }
    ss = warp_sum(ss);
    if (lane == 0) red[warp] = ss;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int w = 0; w < NWARP; ++w) tot += red[w];
    const float scale = 1.f / sqrtf(tot / (float)n + a.eps);
    for (int i = t; i < n; i += THREADS) xs[i] = xs[i] * scale * gain[i];
    __syncthreads();
}

__global__ void __launch_bounds__(THREADS, 1) decode_step_kernel(const __grid_constant__ Args a) {
    extern __shared__ unsigned char smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    unsigned char* sm = smem_raw + (((raw + 127u) & ~127u) - raw);
    unsigned char* ring = sm + OFF_RING;
    float* xs = reinterpret_cast<float*>(sm + OFF_XS);
    float* red = reinterpret_cast<float*>(sm + OFF_RED);
    float* qk = reinterpret_cast<float*>(sm + OFF_QK);
    uint64_t* full = reinterpret_cast<uint64_t*>(sm + OFF_BAR);
    int* misc = reinterpret_cast<int*>(sm + OFF_MISC);

    const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
    const int cta = blockIdx.x;
    const Plan& p = a.plan;
    const int H = p.H, QD = p.QD, G = a.G, hkv = a.hkv;
    const int KD = hkv * D;
    const int pos = __ldcg(a.state);
    long long tok = __ldcg(reinterpret_cast<const long long*>(a.ids));
    if (tok < 0 || tok >= p.V) {           // argmax / the host only ever give valid ids
        if (t == 0) atomicExch(a.status, SA_STATUS_BAD_INDEX);
        tok = 0;
    }
    const uint64_t policy = policy_evict_first();   // each weight is read once per step

    if (t == 0) {
        for (int s = 0; s < NSLOT; ++s) mbar_init(&full[s], 1);
        fence_barrier_init();
    }
    __syncthreads();
    // Warp w owns ring slot w and processes jobs w, w + 16, w + 32, ... of the
    // CTA's schedule: it issues the copy of its next job as soon as it has
    // finished the current one, so each warp keeps one copy in flight and the
    // jobs of a phase run side by side on the 16 warps.
    Sched sch;
    make_sched(p, cta, sch);
    Job cur;
    unsigned kj = (unsigned)warp;   // schedule index of the current job
    bool have = job_at(p, sch, (int)kj, cur);
    if (have && lane == 0) issue(a, cur, ring + warp * SLOT_BYTES, &full[warp], policy);
    unsigned long long best = 0ull;   // lm_head argmax key of the warp (lane 0)
    int* fail = misc + 2;
    if (t == 0) *fail = 0;
    __syncthreads();

    // the warp's jobs of (layer, phase); then the whole CTA; false on abort
    auto run_phase = [&](int layer, int phase) -> bool {
        while (have && cur.layer == layer && cur.phase == phase) {
            if (!wait_slot_warp(a, &full[warp], (kj / NSLOT) & 1u)) {
                if (lane == 0) *fail = 1;
                break;
            }
            const unsigned char* slot = ring + warp * SLOT_BYTES;
            const int rb = row_bytes(p, phase), K = rb / 2;
            const int nr = phase == PH_D ? 2 * cur.n : cur.n;
            float acc[MAXR];
#pragma unroll
            for (int r = 0; r < MAXR; ++r) acc[r] = 0.f;
            const float4* x4 = reinterpret_cast<const float4*>(xs);
            for (int c = lane; c < K / 8; c += 32) {
                const float4 xa = x4[2 * c], xb = x4[2 * c + 1];
#pragma unroll
                for (int r = 0; r < MAXR; ++r) {
                    if (r >= nr) break;
                    const uint4 w = reinterpret_cast<const uint4*>(slot + (size_t)r * rb)[c];
                    float v = acc[r];
                    v = fmaf(__uint_as_float(w.x << 16), xa.x, v);
                    v = fmaf(__uint_as_float(w.x & 0xffff0000u), xa.y, v);
                    v = fmaf(__uint_as_float(w.y << 16), xa.z, v);
                    v = fmaf(__uint_as_float(w.y & 0xffff0000u), xa.w, v);
                    v = fmaf(__uint_as_float(w.z << 16), xb.x, v);
                    v = fmaf(__uint_as_float(w.z & 0xffff0000u), xb.y, v);
                    v = fmaf(__uint_as_float(w.w << 16), xb.z, v);
                    v = fmaf(__uint_as_float(w.w & 0xffff0000u), xb.w, v);
                    acc[r] = v;
                }
            }
#pragma unroll
            for (int r = 0; r < MAXR; ++r) acc[r] = warp_sum(acc[r]);
            __syncwarp();
            // the slot is free: the warp's next job (16 further in the schedule)
            const Job done = cur;
            kj += NSLOT;
            have = job_at(p, sch, (int)kj, cur);
            if (have && lane == 0) issue(a, cur, ring + warp * SLOT_BYTES, &full[warp], policy);
            if (lane == 0) {
                for (int i = 0; i < done.n && i < MAXR; ++i) {
                    const int o = done.first + i;
                    float v = 0.f;
#pragma unroll
                    for (int r = 0; r < MAXR; ++r)
                        if (r == i) v = acc[r];
                    if (phase == PH_A) {
                        a.qkv[o] = v;
                    } else if (phase == PH_C || phase == PH_E) {
                        a.x[o] = __ldcg(a.x + o) + v;
                    } else if (phase == PH_D) {
                        float u = 0.f;
#pragma unroll
                        for (int r = 0; r < MAXR; ++r)
                            if (r == done.n + i) u = acc[r];
                        a.act[o] = (v / (1.f + expf(-v))) * u;
                    } else {
                        const unsigned long long key = ((unsigned long long)ordered_f32(v) << 32) |
                                                       (unsigned long long)(0xffffffffu - (uint32_t)o);
                        best = key > best ? key : best;
                    }
                }
            }
        }
        __syncthreads();
        return *fail == 0;
    };

    // attention of this CTA's (KV head, split); the last split of each head merges
    auto attention = [&](int layer) {
        const int T = pos + 1;
        int S = (T + ROWS_PER_SPLIT - 1) / ROWS_PER_SPLIT;   // about ROWS_PER_SPLIT cached rows per CTA
        if (S > a.splits) S = a.splits;
        if (cta >= hkv * S) return;
        const int h = cta / S, s = cta % S;
        const int r0 = (int)((long long)T * s / S), r1 = (int)((long long)T * (s + 1) / S);
        const MegaLayer& L = a.layers[layer];
        const size_t head_base = ((size_t)layer * hkv + h) * a.max_seq * D;
        // q of the G query heads (normed, roped, prescaled), new k (normed, roped), new v
        if (warp < G + 2) {
            const int kind = warp < G ? 0 : warp == G ? 1 : 2;
            const float* src = kind == 0 ? a.qkv + (size_t)(h * G + warp) * D
                             : kind == 1 ? a.qkv + QD + (size_t)h * D : a.qkv + QD + KD + (size_t)h * D;
            const float4 v4 = __ldcg(reinterpret_cast<const float4*>(src) + lane);
            float e[4] = {v4.x, v4.y, v4.z, v4.w};
            if (kind < 2) {
                const float* nw = kind == 0 ? L.q_norm : L.k_norm;
                const float ss = warp_sum(e[0] * e[0] + e[1] * e[1] + e[2] * e[2] + e[3] * e[3]);
                const float rms = sqrtf(ss / (float)D + 1e-6f);
#pragma unroll
                for (int i = 0; i < 4; ++i) e[i] = (e[i] / rms) * nw[4 * lane + i];
                float pr[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) pr[i] = __shfl_xor_sync(0xffffffffu, e[i], 16);
                const float* cr = a.cos_t + (size_t)pos * (D / 2);
                const float* sr = a.sin_t + (size_t)pos * (D / 2);
                const bool first = lane < 16;
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const int ix = (4 * lane + i) & (D / 2 - 1);
                    const float c = cr[ix], sn = sr[ix];
                    e[i] = first ? e[i] * c + (-pr[i]) * sn : e[i] * c + pr[i] * sn;
                }
                if (kind == 0)
#pragma unroll
                    for (int i = 0; i < 4; ++i) e[i] *= a.qscale;
            }
            const int slotq = kind == 0 ? warp : G + kind - 1;
            reinterpret_cast<float4*>(qk + slotq * D)[lane] = make_float4(e[0], e[1], e[2], e[3]);
            if (s == S - 1 && kind > 0) {   // the split holding row pos appends the new K / V row
                float* dst = (kind == 1 ? a.kc : a.vc) + head_base + (size_t)pos * D;
                // the k row is stored roped and normed, unscaled (kind 1); v as produced (kind 2)
                reinterpret_cast<float4*>(dst)[lane] = make_float4(e[0], e[1], e[2], e[3]);
            }
        }
        __syncthreads();
        // rows r0 .. r1-1: group of 8 lanes per row, lane sub holds dims 16 sub .. 16 sub + 15
        const int sub = lane & 7;
        float qv[MAXG][16], o[MAXG][16], m[MAXG], l[MAXG];
#pragma unroll
        for (int g = 0; g < MAXG; ++g) {
            m[g] = -INFINITY;
            l[g] = 0.f;
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                o[g][i] = 0.f;
                qv[g][i] = g < G ? qk[g * D + 16 * sub + i] : 0.f;
            }
        }
        // the loop bound is the same for every lane of the warp (the score
        // shuffles below are warp-wide); a group past r1 computes nothing
        for (int base = r0 + warp * 4; base < r1; base += NWARP * 4) {
            const int r = base + (lane >> 3);
            const bool valid = r < r1;
            float kv[16], vv[16];
            if (valid) {
                const float* kr = r == pos ? qk + G * D : a.kc + head_base + (size_t)r * D;
                const float* vr = r == pos ? qk + (G + 1) * D : a.vc + head_base + (size_t)r * D;
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const float4 k4 = reinterpret_cast<const float4*>(kr + 16 * sub)[i];
                    kv[4 * i] = k4.x; kv[4 * i + 1] = k4.y; kv[4 * i + 2] = k4.z; kv[4 * i + 3] = k4.w;
                }
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const float4 v4 = reinterpret_cast<const float4*>(vr + 16 * sub)[i];
                    vv[4 * i] = v4.x; vv[4 * i + 1] = v4.y; vv[4 * i + 2] = v4.z; vv[4 * i + 3] = v4.w;
                }
            } else {
#pragma unroll
                for (int i = 0; i < 16; ++i) kv[i] = vv[i] = 0.f;
            }
#pragma unroll
            for (int g = 0; g < MAXG; ++g) {
                if (g >= G) break;
                float sc = 0.f;
#pragma unroll
                for (int i = 0; i < 16; ++i) sc = fmaf(qv[g][i], kv[i], sc);
                sc += __shfl_xor_sync(0xffffffffu, sc, 1);
                sc += __shfl_xor_sync(0xffffffffu, sc, 2);
                sc += __shfl_xor_sync(0xffffffffu, sc, 4);
                if (valid) {
                    const float mn = fmaxf(m[g], sc);
                    const float c = ex2(m[g] - mn), pw = ex2(sc - mn);
                    l[g] = fmaf(l[g], c, pw);
#pragma unroll
                    for (int i = 0; i < 16; ++i) o[g][i] = fmaf(o[g][i], c, pw * vv[i]);
                    m[g] = mn;
                }
            }
        }
        // merge the four row groups of the warp (lanes sub, sub + 8, sub + 16, sub + 24)
#pragma unroll
        for (int off = 8; off <= 16; off <<= 1) {
#pragma unroll
            for (int g = 0; g < MAXG; ++g) {
                if (g >= G) break;
                const float mo = __shfl_xor_sync(0xffffffffu, m[g], off);
                const float lo = __shfl_xor_sync(0xffffffffu, l[g], off);
                const float mn = fmaxf(m[g], mo);
                const float ca = m[g] == -INFINITY ? 0.f : ex2(m[g] - mn);
                const float cb = mo == -INFINITY ? 0.f : ex2(mo - mn);
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    const float oo = __shfl_xor_sync(0xffffffffu, o[g][i], off);
                    o[g][i] = o[g][i] * ca + oo * cb;
                }
                l[g] = l[g] * ca + lo * cb;
                m[g] = mn;
            }
        }
        if (lane < 8) {
#pragma unroll
            for (int g = 0; g < MAXG; ++g) {
                if (g >= G) break;
                float* dst = red + (warp * MAXG + g) * (D + 2);
#pragma unroll
                for (int i = 0; i < 16; ++i) dst[16 * sub + i] = o[g][i];
                if (lane == 0) {
                    dst[D] = m[g];
                    dst[D + 1] = l[g];
                }
            }
        }
        __syncthreads();
        // the CTA's partial (m, l, O) per query head
        if (t < G * D) {
            const int g = t / D, d = t % D;
            float M = -INFINITY;
            for (int w = 0; w < NWARP; ++w) M = fmaxf(M, red[(w * MAXG + g) * (D + 2) + D]);
            float Ls = 0.f, Os = 0.f;
            if (M != -INFINITY)
                for (int w = 0; w < NWARP; ++w) {
                    const float* src = red + (w * MAXG + g) * (D + 2);
                    if (src[D] == -INFINITY) continue;
                    const float c = ex2(src[D] - M);
                    Ls = fmaf(src[D + 1], c, Ls);
                    Os = fmaf(src[d], c, Os);
                }
            float* pp = a.part + ((size_t)(h * S + s) * G + g) * (D + 2);
            pp[d] = Os;
            if (d == 0) {
                pp[D] = M;
                pp[D + 1] = Ls;
            }
        }
        __threadfence();
        __syncthreads();
        if (t == 0) misc[1] = atomicAdd(a.head_cnt + h, 1u) == (unsigned)(S - 1) ? 1 : 0;
        __syncthreads();
        if (misc[1]) {   // the head's last split: merge all S partials
            __threadfence();
            if (t < G * D) {
                const int g = t / D, d = t % D;
                float M = -INFINITY;
                for (int k = 0; k < S; ++k) M = fmaxf(M, __ldcg(a.part + ((size_t)(h * S + k) * G + g) * (D + 2) + D));
                float Ls = 0.f, Os = 0.f;
                for (int k = 0; k < S; ++k) {
                    const float* pp = a.part + ((size_t)(h * S + k) * G + g) * (D + 2);
                    const float mk = __ldcg(pp + D);
                    if (mk == -INFINITY) continue;
                    const float c = ex2(mk - M);
                    Ls = fmaf(__ldcg(pp + D + 1), c, Ls);
                    Os = fmaf(__ldcg(pp + d), c, Os);
                }
                a.attn[(size_t)(h * G + g) * D + d] = Os / Ls;
            }
            if (t == 0) a.head_cnt[h] = 0u;
        }
    };

    bool ok = true;
    // the token's embedding row -> the residual rows this CTA updates in C and E
    {
        int b, e;
        part(H, cta, p.n_cta, &b, &e);
        const __nv_bfloat16* er = a.embed + (size_t)tok * H;
        for (int i = b + t; i < e; i += THREADS) a.x[i] = __bfloat162float(er[i]);
    }
    ok = grid_sync(a, misc);
    for (int layer = 0; ok && layer < p.L; ++layer) {
        const MegaLayer& L = a.layers[layer];
        load_act(a, a.x, H, L.in_norm, xs, red);
        if (!(ok = run_phase(layer, PH_A))) break;
        if (!(ok = grid_sync(a, misc))) break;
        attention(layer);
        if (!(ok = grid_sync(a, misc))) break;
        load_act(a, a.attn, QD, nullptr, xs, red);
        if (!(ok = run_phase(layer, PH_C))) break;
        if (!(ok = grid_sync(a, misc))) break;
        load_act(a, a.x, H, L.post_norm, xs, red);
        if (!(ok = run_phase(layer, PH_D))) break;
        if (!(ok = grid_sync(a, misc))) break;
        load_act(a, a.act, p.I, nullptr, xs, red);
        if (!(ok = run_phase(layer, PH_E))) break;
        if (!(ok = grid_sync(a, misc))) break;
    }
    if (ok) {
        load_act(a, a.x, H, a.final_norm, xs, red);
        ok = run_phase(p.L, PH_F);
    }
    if (ok) {
        // the CTA's best (logit, first index) into the grid's key
        unsigned long long* bw = reinterpret_cast<unsigned long long*>(red);
        if (lane == 0) bw[warp] = best;
        __syncthreads();
        if (t == 0) {
            unsigned long long b2 = 0ull;
            for (int w = 0; w < NWARP; ++w) b2 = bw[w] > b2 ? bw[w] : b2;
            if (b2) atomicMax(a.amax, b2);
        }
        ok = grid_sync(a, misc);
    }
    if (ok && cta == 0 && t == 0) {
        const unsigned long long k = __ldcg(a.amax);
        const long long next = (long long)(0xffffffffu - (uint32_t)(k & 0xffffffffull));
        *a.ids = next;
        const int n = a.state[1];
        if (n < a.toks_cap) a.toks[n] = next;
        a.state[1] = n + 1;
        a.state[0] = pos + 1;
        *a.amax = 0ull;
    }
    if (!ok && have && lane == 0) {
        // let the warp's copy still in flight land before the CTA exits
        mbar_wait(&full[warp], (kj / NSLOT) & 1u, nullptr);
    }
}

}  // namespace mk

// ---------------------------------------------------------------- host side
// Shapes the single-launch step handles: head_dim 128, one or two query heads
// per KV head, activation vectors that fit its shared-memory buffer, and at
// least one CTA per KV head.  (Rows of every matrix then fit a ring slot.)
// It is selected with SA_QWEN3_MEGA=1: on Qwen3-0.6B it measured 1.40 ms per
// token against 0.94 ms for the CUDA graph of separate kernels at the time
// (the five grid barriers and latency-bound phases of a layer cost ~48 us,
// the graph's kernels ~33 us; the graph has since reached 0.74 ms), so the
// graph is the default.
bool mega_supported(const sa_qwen3_config& c, int num_sms) {
    const int G = c.hkv > 0 && c.hq % c.hkv == 0 ? c.hq / c.hkv : 0;
    const char* on = std::getenv("SA_QWEN3_MEGA");
    return on && on[0] == '1' && c.head_dim == mk::D && (G == 1 || G == 2) && c.hidden % 8 == 0 &&
           c.inter % 32 == 0 && c.hidden <= mk::XS_FLOATS && c.hq * mk::D <= mk::XS_FLOATS &&
           c.inter <= mk::XS_FLOATS && num_sms >= c.hkv;
}

int mega_grid(int device) {
    static int cached[64] = {0};
    if (device >= 0 && device < 64 && cached[device]) return cached[device];
    int sms = 0, coop = 0, per_sm = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess ||
        cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, device) != cudaSuccess || !coop) {
        cudaGetLastError();
        return 0;
    }
    if (set_smem_attr_once((const void*)mk::decode_step_kernel, mk::SMEM_BYTES) != SA_OK) return 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, mk::decode_step_kernel, mk::THREADS,
                                                      mk::SMEM_BYTES) != cudaSuccess ||
        per_sm < 1) {
        cudaGetLastError();
        return 0;
    }
    if (device >= 0 && device < 64) cached[device] = sms;
    return sms;
}

int launch_decode_mega(cudaStream_t st, int grid, const MegaParams& q) {
    mk::Args a;
    a.plan.n_cta = grid;
    a.plan.L = q.L;
    a.plan.H = q.H;
    a.plan.I = q.I;
    a.plan.QD = q.hq * mk::D;
    a.plan.NQKV = (q.hq + 2 * q.hkv) * mk::D;
    a.plan.V = q.V;
    a.plan.slot_bytes = mk::SLOT_BYTES;
    a.plan.max_rows = mk::MAXR;
    a.layers = q.layers;
    a.hq = q.hq;
    a.hkv = q.hkv;
    a.G = q.hq / q.hkv;
    a.max_seq = q.max_seq;
    a.splits = grid / q.hkv;
    a.eps = q.eps;
    a.qscale = 1.4426950408889634f / sqrtf((float)mk::D);
    a.embed = q.embed;
    a.lm_head = q.lm_head;
    a.final_norm = q.final_norm;
    a.kc = q.kc;
    a.vc = q.vc;
    a.cos_t = q.cos_t;
    a.sin_t = q.sin_t;
    a.x = q.x;
    a.qkv = q.qkv;
    a.attn = q.attn;
    a.act = q.act;
    a.part = q.part;
    a.head_cnt = q.head_cnt;
    a.amax = q.amax;
    a.gbar = q.gbar;
    a.state = q.state;
    a.ids = q.ids;
    a.toks = q.toks;
    a.toks_cap = q.toks_cap;
    a.status = q.status;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(mk::THREADS);
    cfg.dynamicSmemBytes = mk::SMEM_BYTES;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    SA_CUDA_TRY(cudaLaunchKernelEx(&cfg, mk::decode_step_kernel, a));
    return SA_OK;
}

}  // namespace sa
