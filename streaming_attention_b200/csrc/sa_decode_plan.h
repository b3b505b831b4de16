// sa_decode_plan.h -- the split and copy schedule of the decode attention
// kernel (sa_decode.cu) when it reads the cache length on the device (the
// captured decode step), shared by the kernel and a CPU test that enumerates
// it (tests/test_decode_plan.py compiles this header with g++).
//
// The grid is planned for the cache's capacity; each CTA re-splits the T rows
// present into splits of a whole number of stages (dev_split).  A CTA's
// producer then issues its copies in two groups around griddepcontrol.wait
// (pre_wait_plan): rows cached by earlier steps may go before the wait, since
// they were written before the step's first, ordinary launch; the newest row
// (T - 1, appended by the kernel this one follows) and q only after it.
#pragma once

#ifndef __CUDACC__
#define SA_DHD
#else
#define SA_DHD __host__ __device__
#endif

namespace sa {
namespace dec {

SA_DHD inline int plan_min(int a, int b) { return a < b ? a : b; }

struct Split {
    int rps;      // rows per split, a multiple of the stage rows
    int nsplit;   // splits in use (every one non-empty)
};

// About `dyn_rows` rows per split, at most `cap` splits, for t >= 1 rows of
// `sr`-row stages.
SA_DHD inline Split dev_split(int t, int cap, int sr, int dyn_rows) {
    int want = (t + dyn_rows - 1) / dyn_rows;
    want = want < 1 ? 1 : (want > cap ? cap : want);
    Split s;
    s.rps = ((t + want - 1) / want + sr - 1) / sr * sr;
    s.nsplit = (t + s.rps - 1) / s.rps;
    return s;
}

// The copies of one CTA over rows [0, nrows) of its split (first row t0 of T,
// stages of sr rows into a ring of `ring` slots; stage i uses slot i % ring):
//  * stages [0, pre) whole, before the wait;
//  * with split_new, stage st_new (< ring, the split's last stage, which ends
//    with the newest row T - 1): its first `head` rows before the wait, the
//    newest row after it, both counted on the stage's one barrier phase;
//  * stages [post0, nst) after the wait, through the ring.
// Without a device length everything goes after the wait (pre = post0 = 0).
struct PreWait {
    int nst;       // stages of the split
    int pre;       // whole stages before the wait
    int st_new;    // stage holding the newest row (nst if this split lacks it)
    int head;      // rows of stage st_new before the newest row
    int post0;     // first stage issued after the wait
    bool split_new;
};

SA_DHD inline PreWait pre_wait_plan(bool len_dev, int T, int t0, int nrows, int sr, int ring) {
    PreWait p;
    p.nst = (nrows + sr - 1) / sr;
    const int rel_new = T - 1 - t0;                         // >= 0 for a split in use
    const bool has_new = len_dev && rel_new < nrows;        // then it is the split's last row
    p.st_new = has_new ? rel_new / sr : p.nst;
    p.pre = len_dev ? plan_min(ring, plan_min(p.nst, p.st_new)) : 0;
    p.split_new = has_new && p.st_new < ring;
    p.head = p.split_new ? rel_new - p.st_new * sr : 0;
    p.post0 = p.split_new ? p.st_new + 1 : p.pre;
    return p;
}

}  // namespace dec
}  // namespace sa
