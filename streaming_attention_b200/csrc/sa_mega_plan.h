// sa_mega_plan.h -- the weight-copy schedule of the single-launch Qwen3
// decode step (sa_qwen3_mega.cu), shared by its copy issuer and its compute
// threads, and compiled on the host by a CPU test that checks, for every
// CTA, that the copies stay inside the weight matrices, fit a ring slot and
// cover every row exactly once.
//
// Every CTA owns a contiguous part of each matrix's rows and streams them, in
// a fixed order, through a ring of shared-memory slots: per layer the fused
// QKV rows (phase A), o_proj rows (C), gate/up row pairs (D) and down_proj
// rows (E); after the last layer the lm_head rows (F).  A job is one slot: up
// to `slot_bytes / row_bytes` consecutive rows, or, in phase D, up to
// slot_bytes / (2 row_bytes) consecutive (gate, up) pairs of one 32-row block
// of the interleaved gate/up matrix (gate rows at 64 b + i, up rows at
// 64 b + 32 + i) copied as two runs.
#pragma once
#include <cstdint>

#ifndef __CUDACC__
#define SA_HD
#else
#define SA_HD __host__ __device__
#endif

namespace sa {
namespace mk {

enum : int { PH_A = 0, PH_C = 1, PH_D = 2, PH_E = 3, PH_F = 4, PH_END = 5 };

struct Plan {
    int n_cta;
    int L, H, I, QD, NQKV, V;
    int slot_bytes;
    int max_rows;      // rows one job may hold (the compute threads' row capacity)
};

// Rows [*b, *e) of n rows owned by CTA c of n_cta.
SA_HD inline void part(int n, int c, int n_cta, int* b, int* e) {
    *b = (int)((long long)n * c / n_cta);
    *e = (int)((long long)n * (c + 1) / n_cta);
}

// Rows of the matrix of phase ph, and the bytes of one row (bf16).
SA_HD inline int phase_rows(const Plan& p, int ph) {
    return ph == PH_A ? p.NQKV : ph == PH_C ? p.H : ph == PH_D ? p.I : ph == PH_E ? p.H : p.V;
}
SA_HD inline int row_bytes(const Plan& p, int ph) {
    return 2 * (ph == PH_C ? p.QD : ph == PH_E ? p.I : p.H);
}

struct Job {
    int layer, phase;
    int first, n;                   // rows (pairs in phase D) first .. first + n - 1
    long long src0, src1;           // element offsets into the phase's matrix (src1: up run, phase D)
    int bytes0, bytes1;             // bytes of each run (bytes1 = 0 outside phase D)
};

// Position in a CTA's job sequence.
struct Iter {
    int layer = 0, phase = PH_A, next = -1;   // next row / pair (-1: not started in this phase)
};

// The CTA's next job; false once the sequence (ending with phase F) is done.
SA_HD inline bool next_job(const Plan& p, int cta, Iter& it, Job& j) {
    while (it.phase != PH_END) {
        const int N = phase_rows(p, it.phase);
        int b, e;
        part(N, cta, p.n_cta, &b, &e);
        if (it.next < 0) it.next = b;
        if (it.next < e) {
            const int rb = row_bytes(p, it.phase);
            j.layer = it.layer;
            j.phase = it.phase;
            j.first = it.next;
            if (it.phase == PH_D) {
                int cap = p.slot_bytes / (2 * rb);
                if (cap > p.max_rows / 2) cap = p.max_rows / 2;
                const int in_block = 32 - it.next % 32;
                int n = e - it.next;
                if (n > cap) n = cap;
                if (n > in_block) n = in_block;
                const long long g = 64LL * (it.next / 32) + it.next % 32;   // gate row of the first pair
                j.n = n;
                j.src0 = g * (rb / 2);
                j.src1 = (g + 32) * (rb / 2);
                j.bytes0 = j.bytes1 = n * rb;
            } else {
                int cap = p.slot_bytes / rb;
                if (cap > p.max_rows) cap = p.max_rows;
                int n = e - it.next;
                if (n > cap) n = cap;
                j.n = n;
                j.src0 = (long long)it.next * (rb / 2);
                j.src1 = 0;
                j.bytes0 = n * rb;
                j.bytes1 = 0;
            }
            it.next += j.n;
            return true;
        }
        // advance to the next phase
        it.next = -1;
        if (it.phase == PH_F) {
            it.phase = PH_END;
        } else if (it.phase == PH_E) {
            if (++it.layer < p.L) it.phase = PH_A;
            else it.phase = PH_F;
        } else {
            ++it.phase;
        }
    }
    return false;
}

// ---- direct access: job k of a CTA's schedule in O(1) -------------------------
// The schedule next_job walks, laid out so that any job can be found without
// walking: each phase's row (pair) range and job count are the same for every
// layer.
struct Sched {
    int b[5], e[5];       // the CTA's rows (pairs in phase D) per phase
    int cap[5];           // rows (pairs) per job
    int nj[5];            // jobs per phase (per layer for A..E)
    int per_layer;        // jobs of one layer
    int total;            // jobs of the whole schedule
};

SA_HD inline int ceil_div(int a, int b) { return (a + b - 1) / b; }

// Jobs of the pair range [p0, p1) in phase D: runs split at 32-pair blocks,
// each run cut into chunks of cap pairs.
SA_HD inline int d_jobs(int p0, int p1, int cap) {
    if (p1 <= p0) return 0;
    const int fb = p0 / 32, lb = (p1 - 1) / 32;
    if (fb == lb) return ceil_div(p1 - p0, cap);
    return ceil_div(32 * (fb + 1) - p0, cap) + (lb - fb - 1) * ceil_div(32, cap) + ceil_div(p1 - 32 * lb, cap);
}

// First pair and pair count of the i-th phase-D job of [p0, p1).
SA_HD inline void d_job(int p0, int p1, int cap, int i, int* first, int* n) {
    const int fb = p0 / 32, lb = (p1 - 1) / 32;
    int f, end;
    if (fb == lb) {
        f = p0 + i * cap;
        end = p1;
    } else {
        const int c0 = ceil_div(32 * (fb + 1) - p0, cap), cpb = ceil_div(32, cap);
        const int cm = (lb - fb - 1) * cpb;
        if (i < c0) {
            f = p0 + i * cap;
            end = 32 * (fb + 1);
        } else if (i < c0 + cm) {
            const int j = i - c0, blk = fb + 1 + j / cpb;
            f = 32 * blk + (j % cpb) * cap;
            end = 32 * (blk + 1);
        } else {
            f = 32 * lb + (i - c0 - cm) * cap;
            end = p1;
        }
    }
    *first = f;
    *n = (end - f) < cap ? (end - f) : cap;
}

SA_HD inline void make_sched(const Plan& p, int cta, Sched& s) {
    for (int ph = 0; ph < 5; ++ph) {
        part(phase_rows(p, ph), cta, p.n_cta, &s.b[ph], &s.e[ph]);
        const int rb = row_bytes(p, ph);
        int cap = ph == PH_D ? p.slot_bytes / (2 * rb) : p.slot_bytes / rb;
        const int lim = ph == PH_D ? p.max_rows / 2 : p.max_rows;
        if (cap > lim) cap = lim;
        s.cap[ph] = cap;
        s.nj[ph] = ph == PH_D ? d_jobs(s.b[ph], s.e[ph], cap)
                              : (s.e[ph] > s.b[ph] ? ceil_div(s.e[ph] - s.b[ph], cap) : 0);
    }
    s.per_layer = s.nj[PH_A] + s.nj[PH_C] + s.nj[PH_D] + s.nj[PH_E];
    s.total = p.L * s.per_layer + s.nj[PH_F];
}

// Job k of the schedule (the one next_job gives after k steps); false past the end.
SA_HD inline bool job_at(const Plan& p, const Sched& s, int k, Job& j) {
    if (k < 0 || k >= s.total) return false;
    int ph, idx;
    if (k >= p.L * s.per_layer) {
        j.layer = p.L;
        ph = PH_F;
        idx = k - p.L * s.per_layer;
    } else {
        j.layer = k / s.per_layer;
        idx = k % s.per_layer;
        ph = PH_A;
        while (idx >= s.nj[ph]) idx -= s.nj[ph++];
    }
    j.phase = ph;
    const int rb = row_bytes(p, ph);
    if (ph == PH_D) {
        d_job(s.b[ph], s.e[ph], s.cap[ph], idx, &j.first, &j.n);
        const long long g = 64LL * (j.first / 32) + j.first % 32;
        j.src0 = g * (rb / 2);
        j.src1 = (g + 32) * (rb / 2);
        j.bytes0 = j.bytes1 = j.n * rb;
    } else {
        j.first = s.b[ph] + idx * s.cap[ph];
        const int left = s.e[ph] - j.first;
        j.n = left < s.cap[ph] ? left : s.cap[ph];
        j.src0 = (long long)j.first * (rb / 2);
        j.src1 = 0;
        j.bytes0 = j.n * rb;
        j.bytes1 = 0;
    }
    return true;
}

}  // namespace mk
}  // namespace sa
