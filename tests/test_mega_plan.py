"""The weight-copy schedule of the single-launch decode step
(streaming_attention_b200/csrc/sa_mega_plan.h), enumerated on the CPU for
every CTA: each copy lies inside its matrix, fits a ring slot and starts on a
16-byte boundary, the CTAs together cover every row of every matrix exactly
once, in phase order, and the O(1) job lookup the kernel uses (job_at) gives
exactly the job the step-by-step walk (next_job) gives.  CPU only (the header
compiles with g++)."""
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
#include "sa_mega_plan.h"
using namespace sa::mk;
int main(int argc, char** argv) {
    Plan p;
    p.n_cta = atoi(argv[1]); p.L = atoi(argv[2]); p.H = atoi(argv[3]); p.I = atoi(argv[4]);
    p.QD = atoi(argv[5]); p.NQKV = atoi(argv[6]); p.V = atoi(argv[7]); p.slot_bytes = atoi(argv[8]);
    p.max_rows = atoi(argv[9]);
    // coverage[layer][phase] counts per row
    std::vector<std::vector<std::vector<int>>> cov(p.L + 1, std::vector<std::vector<int>>(5));
    for (int l = 0; l <= p.L; ++l)
        for (int ph = 0; ph < 5; ++ph) cov[l][ph].assign(phase_rows(p, ph), 0);
    long long jobs = 0, max_jobs = 0;
    for (int c = 0; c < p.n_cta; ++c) {
        Iter it; Job j; long long n = 0; int last_key = -1;
        Sched sc; make_sched(p, c, sc);
        while (next_job(p, c, it, j)) {
            Job d;
            if (!job_at(p, sc, (int)n, d) || d.layer != j.layer || d.phase != j.phase || d.first != j.first ||
                d.n != j.n || d.src0 != j.src0 || d.src1 != j.src1 || d.bytes0 != j.bytes0 || d.bytes1 != j.bytes1) {
                printf("job_at %d %lld\n", c, n); return 1; }
            ++n;
            const int key = j.layer * 8 + j.phase;
            if (key < last_key) { printf("order %d\n", c); return 1; }
            last_key = key;
            const int rb = row_bytes(p, j.phase);
            const long long K = rb / 2;
            const long long rows = j.phase == PH_D ? 2LL * p.I : phase_rows(p, j.phase);
            if (j.n <= 0 || j.bytes0 + j.bytes1 > p.slot_bytes) { printf("size %d\n", c); return 1; }
            if ((j.phase == PH_D ? 2 * j.n : j.n) > p.max_rows) { printf("rows %d\n", c); return 1; }
            if (j.src0 < 0 || j.src0 * 2 + j.bytes0 > rows * K * 2) { printf("oob0 %d\n", c); return 1; }
            if (j.bytes1 && (j.src1 < 0 || j.src1 * 2 + j.bytes1 > rows * K * 2)) { printf("oob1 %d\n", c); return 1; }
            if ((j.src0 * 2) % 16 || (j.src1 * 2) % 16 || j.bytes0 % 16 || j.bytes1 % 16) { printf("align %d\n", c); return 1; }
            if (j.phase == PH_D && j.first / 32 != (j.first + j.n - 1) / 32) { printf("block %d\n", c); return 1; }
            if (j.phase == PH_D && j.src0 != (64LL * (j.first / 32) + j.first % 32) * K) { printf("gate %d\n", c); return 1; }
            if (j.phase != PH_D && j.src0 != (long long)j.first * K) { printf("row %d\n", c); return 1; }
            for (int r = j.first; r < j.first + j.n; ++r) cov[j.layer][j.phase][r]++;
        }
        if (sc.total != n) { printf("total %d\n", c); return 1; }
        { Job d; if (job_at(p, sc, (int)n, d)) { printf("past end %d\n", c); return 1; } }
        jobs += n;
        if (n > max_jobs) max_jobs = n;
    }
    for (int l = 0; l <= p.L; ++l)
        for (int ph = 0; ph < 5; ++ph) {
            const bool used = (l < p.L) != (ph == PH_F);
            for (int v : cov[l][ph])
                if (v != (used ? 1 : 0)) { printf("coverage l=%d ph=%d\n", l, ph); return 1; }
        }
    printf("OK jobs=%lld max_per_cta=%lld\n", jobs, max_jobs);
    return 0;
}
'''


@pytest.mark.skipif(CXX is None, reason="no C++ compiler")
@pytest.mark.parametrize("n_cta", [148, 132, 7, 1])
@pytest.mark.parametrize("dims", [
    (28, 1024, 3072, 2048, 4096, 151936),     # Qwen3-0.6B
    (2, 256, 512, 512, 1024, 1000),           # the tests' small models
    (2, 256, 768, 512, 1024, 2048),           # the golden tiny model
    (3, 512, 1536, 1024, 2048, 1000),
])
def test_mega_plan_covers_every_row_once(tmp_path, n_cta, dims):
    src = tmp_path / "plan.cpp"
    src.write_text(CHECK)
    exe = tmp_path / "plan"
    subprocess.run([CXX, "-std=c++17", "-O1", "-I", os.path.join(ROOT, "streaming_attention_b200", "csrc"),
                    str(src), "-o", str(exe)], check=True)
    L, H, I, QD, NQKV, V = dims
    # the kernel's geometry: 12 KB slots (one per warp), at most 6 rows per job
    r = subprocess.run([str(exe), str(n_cta), str(L), str(H), str(I), str(QD), str(NQKV), str(V), "12288", "6"],
                       capture_output=True, text=True, timeout=120)
    assert r.returncode == 0 and r.stdout.startswith("OK"), r.stdout + r.stderr
