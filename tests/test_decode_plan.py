"""The split and copy schedule of the decode attention kernel inside the
captured decode step (streaming_attention_b200/csrc/sa_decode_plan.h),
enumerated on the CPU: for every cache length T, split cap, stage size and
ring depth, the splits are non-empty, a whole number of stages and cover the
T rows exactly once; each CTA's copies cover its rows exactly once; no copy
issued before griddepcontrol.wait contains the newest row T - 1 (which the
previous kernel appends); the stage that holds the newest row is the split's
last, uses a ring slot no earlier stage uses, and its one barrier phase
expects exactly the rows copied into it.  CPU only (the header compiles with
g++)."""
import os
import shutil
import subprocess

import pytest

from conftest import ROOT

CXX = "/usr/bin/g++" if os.path.exists("/usr/bin/g++") else shutil.which("g++")

CHECK = r'''
#include <cstdio>
#include <cstdlib>
#include <vector>
#include "sa_decode_plan.h"
using namespace sa::dec;
#define FAIL(...) do { printf(__VA_ARGS__); printf(" T=%d cap=%d sr=%d ring=%d\n", T, cap, sr, ring); return 1; } while (0)
int main(int argc, char** argv) {
    const int t_max = atoi(argv[1]);
    const int srs[] = {8, 16, 32, 64};
    const int caps[] = {1, 2, 5, 16, 128, 1024};
    const int rings[] = {3, 6};
    long long ctas = 0, split_stage = 0, late_new = 0;
    for (int sr : srs)
    for (int cap : caps)
    for (int ring : rings)
    for (int T = 1; T <= t_max; ++T) {
        const Split sp = dev_split(T, cap, sr, 8 * sr);
        if (sp.rps % sr || sp.rps <= 0 || sp.nsplit < 1 || sp.nsplit > cap) FAIL("split shape rps=%d n=%d", sp.rps, sp.nsplit);
        std::vector<int> cov(T, 0);
        for (int s = 0; s < sp.nsplit; ++s) {
            const int t0 = s * sp.rps;
            int nrows = T - t0 < sp.rps ? T - t0 : sp.rps;
            if (nrows <= 0) FAIL("empty split %d", s);
            ++ctas;
            const PreWait pw = pre_wait_plan(true, T, t0, nrows, sr, ring);
            if (pw.nst != (nrows + sr - 1) / sr) FAIL("nst");
            std::vector<int> rc(nrows, 0);
            std::vector<int> slot_used(ring, 0);
            auto stage_rows = [&](int it) { int e = (it + 1) * sr; return (e < nrows ? e : nrows) - it * sr; };
            // before the wait
            if (pw.pre > ring || pw.pre > pw.nst) FAIL("pre %d", pw.pre);
            for (int it = 0; it < pw.pre; ++it) {
                slot_used[it % ring]++;
                for (int r = it * sr; r < it * sr + stage_rows(it); ++r) {
                    if (t0 + r == T - 1) FAIL("newest row before the wait (stage %d)", it);
                    rc[r]++;
                }
            }
            if (pw.split_new) {
                ++split_stage;
                if (pw.st_new != pw.nst - 1 || pw.st_new >= ring || pw.st_new != pw.pre) FAIL("split stage %d", pw.st_new);
                if (slot_used[pw.st_new % ring]) FAIL("slot reuse");
                if (pw.st_new * sr + pw.head != T - 1 - t0) FAIL("newest row position");
                if (pw.head + 1 != stage_rows(pw.st_new)) FAIL("expected rows of the split stage");
                for (int r = pw.st_new * sr; r < pw.st_new * sr + pw.head; ++r) {
                    if (t0 + r == T - 1) FAIL("newest row in the split stage's head");
                    rc[r]++;
                }
                rc[pw.st_new * sr + pw.head]++;          // after the wait
                if (pw.post0 != pw.st_new + 1) FAIL("post0");
            } else {
                if (pw.post0 != pw.pre) FAIL("post0 without split");
                if (pw.st_new < pw.nst) ++late_new;       // newest row in a stage issued after the wait
            }
            // after the wait, through the ring
            for (int it = pw.post0; it < pw.nst; ++it)
                for (int r = it * sr; r < it * sr + stage_rows(it); ++r) rc[r]++;
            for (int r = 0; r < nrows; ++r) {
                if (rc[r] != 1) FAIL("row %d of split %d copied %d times", r, s, rc[r]);
                cov[t0 + r]++;
            }
            // without a device length everything goes after the wait
            const PreWait ps = pre_wait_plan(false, T, t0, nrows, sr, ring);
            if (ps.pre || ps.post0 || ps.split_new) FAIL("static launch pre-wait copies");
        }
        for (int t = 0; t < T; ++t)
            if (cov[t] != 1) FAIL("row %d covered %d times", t, cov[t]);
    }
    printf("OK ctas=%lld split_stage=%lld late_new=%lld\n", ctas, split_stage, late_new);
    return 0;
}
'''


@pytest.mark.skipif(CXX is None, reason="no C++ compiler")
def test_decode_plan_enumerated(tmp_path):
    src = tmp_path / "check.cpp"
    src.write_text(CHECK)
    exe = tmp_path / "check"
    inc = os.path.join(ROOT, "streaming_attention_b200", "csrc")
    subprocess.run([CXX, "-std=c++17", "-O2", "-I", inc, str(src), "-o", str(exe)], check=True)
    r = subprocess.run([str(exe), "3000"], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert r.stdout.startswith("OK"), r.stdout
    # both schedules occur: the newest row's stage split around the wait, and
    # (in long splits) a newest-row stage past the ring issued after it
    counts = dict(kv.split("=") for kv in r.stdout.split()[1:])
    assert int(counts["split_stage"]) > 0 and int(counts["late_new"]) > 0, r.stdout
