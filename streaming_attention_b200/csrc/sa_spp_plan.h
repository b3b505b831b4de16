// sa_spp_plan.h -- the work split of the sequence-parallel causal prefill
// (sa_sp_prefill.cu), shared by the library and a CPU test that enumerates it
// (tests/test_spp_plan.py compiles this header with g++).
//
// S tokens in 2P zig-zag chunks of C = S / 2P: rank r holds chunks r and
// 2P-1-r (local query rows [0, C) and [C, 2C)).  A chunk starting at key
// `start` attends keys [0, start + C): the keys before it in unmasked blocks
// of L keys (the last one shorter), then its causal diagonal block of C keys.
// L = max(C, min_keys, ceil((2P-1) C / (max_blocks - 1))): blocks long enough
// that a CTA's set-up is worth it, and at most max_blocks blocks per chunk.
#pragma once

namespace sa {
namespace spp {

struct PieceSpec {
    int q_row0;   // first local query row (0 or C)
    int kv_row0;  // first key of the block
    int Skv;      // keys in the block
    int q_pos0;   // query i sees key j of the block when j <= q_pos0 + i
};

// Fills pieces[0 .. returned count) for rank `rank` of `world`; first[h] /
// count[h] delimit chunk h's pieces (h = 0: chunk rank, h = 1: chunk
// 2 world - 1 - rank).  Returns -1 if a chunk would need more than
// max_blocks pieces or the table (cap entries) is too small.
inline int plan_pieces(int rank, int world, int C, int min_keys, int max_blocks, PieceSpec* pieces, int cap,
                       int first[2], int count[2]) {
    int L = C > min_keys ? C : min_keys;
    const int most = (2 * world - 1) * C;                      // keys before the last chunk
    const int need = (most + max_blocks - 2) / (max_blocks - 1);
    if (L < need) L = need;
    const int chunk[2] = {rank, 2 * world - 1 - rank};
    int n = 0;
    for (int half = 0; half < 2; ++half) {
        first[half] = n;
        const int start = chunk[half] * C;
        for (int kv0 = 0; kv0 < start; kv0 += L) {
            if (n - first[half] >= max_blocks - 1 || n >= cap) return -1;
            PieceSpec& p = pieces[n++];
            p.q_row0 = half * C;
            p.kv_row0 = kv0;
            p.Skv = kv0 + L < start ? L : start - kv0;
            p.q_pos0 = start - kv0;                             // past the block's last key: all visible
        }
        if (n >= cap) return -1;
        PieceSpec& d = pieces[n++];                             // the diagonal
        d.q_row0 = half * C;
        d.kv_row0 = start;
        d.Skv = C;
        d.q_pos0 = 0;
        count[half] = n - first[half];
    }
    return n;
}

}  // namespace spp
}  // namespace sa
