"""The work split of the sequence-parallel causal prefill
(streaming_attention_b200/csrc/sa_spp_plan.h), enumerated on the CPU for
every rank of 1..8: each chunk's pieces cover its keys [0, start + C) exactly
once and in order (unmasked blocks before the chunk, every key of them
visible to every query row; then the causal diagonal), no chunk exceeds the
block cap, and every rank streams the same number of keys (the zig-zag
balance).  CPU only (the header compiles with g++)."""
import os
import shutil
import subprocess

import pytest

from conftest import ROOT

CXX = "/usr/bin/g++" if os.path.exists("/usr/bin/g++") else shutil.which("g++")

CHECK = r'''
#include <cstdio>
#include <cstdlib>
#include "sa_spp_plan.h"
using namespace sa::spp;
int main(int argc, char** argv) {
    const int world = atoi(argv[1]), C = atoi(argv[2]), min_keys = atoi(argv[3]), max_blocks = atoi(argv[4]);
    long long keys0 = -1;
    for (int r = 0; r < world; ++r) {
        PieceSpec p[64];
        int first[2], count[2];
        const int n = plan_pieces(r, world, C, min_keys, max_blocks, p, 64, first, count);
        if (n < 1) { printf("FAIL rank %d: no plan\n", r); return 1; }
        long long keys = 0;
        const int chunk[2] = {r, 2 * world - 1 - r};
        for (int h = 0; h < 2; ++h) {
            const int start = chunk[h] * C;
            if (first[h] != (h ? count[0] : 0) || count[h] < 1 || count[h] > max_blocks) {
                printf("FAIL rank %d chunk %d: first %d count %d\n", r, h, first[h], count[h]);
                return 1;
            }
            int next = 0;   // the next key the chunk's pieces must start at
            for (int i = first[h]; i < first[h] + count[h]; ++i) {
                const bool diag = i == first[h] + count[h] - 1;
                if (p[i].q_row0 != h * C || p[i].kv_row0 != next || p[i].Skv < 1) {
                    printf("FAIL rank %d piece %d: q_row0 %d kv_row0 %d (want %d) Skv %d\n", r, i, p[i].q_row0,
                           p[i].kv_row0, next, p[i].Skv);
                    return 1;
                }
                if (diag ? (p[i].kv_row0 != start || p[i].Skv != C || p[i].q_pos0 != 0)
                         : (p[i].kv_row0 + p[i].Skv > start || p[i].q_pos0 != start - p[i].kv_row0 ||
                            p[i].q_pos0 < p[i].Skv)) {
                    printf("FAIL rank %d piece %d: kv_row0 %d Skv %d q_pos0 %d start %d diag %d\n", r, i,
                           p[i].kv_row0, p[i].Skv, p[i].q_pos0, start, (int)diag);
                    return 1;
                }
                next = p[i].kv_row0 + p[i].Skv;
                keys += p[i].Skv;
            }
            if (next != start + C) { printf("FAIL rank %d chunk %d ends at %d\n", r, h, next); return 1; }
        }
        if (keys0 >= 0 && keys != keys0) { printf("FAIL rank %d streams %lld keys, rank 0 %lld\n", r, keys, keys0); return 1; }
        keys0 = keys;
        printf("rank %d pieces %d keys %lld\n", r, n, keys);
    }
    printf("OK\n");
    return 0;
}
'''


@pytest.fixture(scope="module")
def checker(tmp_path_factory):
    if not CXX:
        pytest.skip("no g++")
    d = tmp_path_factory.mktemp("spp_plan")
    src, exe = d / "check.cpp", d / "check"
    src.write_text(CHECK)
    subprocess.run([CXX, "-std=c++17", "-O1", "-I", os.path.join(ROOT, "streaming_attention_b200", "csrc"),
                    str(src), "-o", str(exe)], check=True)
    return str(exe)


@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
@pytest.mark.parametrize("C", [1, 7, 128, 512, 700, 1024, 4096, 16384])
def test_spp_plan_covers_every_key_once(checker, world, C):
    r = subprocess.run([checker, str(world), str(C), "1024", "16"], capture_output=True, text=True)
    assert r.returncode == 0 and r.stdout.strip().endswith("OK"), r.stdout


def test_spp_plan_configs2_piece_counts(checker):
    """configs[2] (S = 8192): 3 pieces per rank on one GPU, 5 on two, 9 on
    four, 10 on eight (blocks of at least 1024 keys)."""
    for world, want in ((1, 3), (2, 5), (4, 9), (8, 10)):
        r = subprocess.run([checker, str(world), str(8192 // (2 * world)), "1024", "16"], capture_output=True,
                           text=True)
        assert r.returncode == 0, r.stdout
        assert f"rank 0 pieces {want} " in r.stdout, (world, r.stdout)
