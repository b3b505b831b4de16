"""The arithmetic of two GPU methods, restated in numpy and checked against
float64 on the CPU (what the GPU parity tests' tolerances rest on).

1. Deferred RMSNorm of the prompt GEMMs (sa_gemm.cu, QW_EPI_RESID_NORM and
   the consumer's row scale): the producer writes A = hi/lo(g * x) (two bf16
   planes: hi = bf16(v), lo = bf16(v - hi)) and per-tile row sums of x^2; the
   consumer computes (A W^T) / rms(x) with rms from the tiles' sums.  This
   equals RMSNorm(x) W^T (qwen3_ops.cpp:450-456, ops.cpp rms_norm) to a few
   fp32 ulps of the output scale, also for activations spanning decades.
2. The sequence-parallel prefill's merge (sa_sp_prefill.cu): each key block
   gives bf16 output rows O_p and the log2-domain log-sum-exp lse_p of its
   scaled scores; out = sum_p 2^(lse_p - lse) O_p / sum_p 2^(lse_p - lse)
   equals the softmax over all keys within one bf16 rounding (2^-8
   relative)."""
import numpy as np

from oracle.oracle import bf16_round


def _hilo(v):
    hi = bf16_round(v.astype(np.float32))
    lo = bf16_round((v.astype(np.float32) - hi).astype(np.float32))
    return hi, lo


def test_deferred_rmsnorm_matches_rmsnorm_then_linear():
    rng = np.random.default_rng(5)
    M, K, N, eps, tiles = 64, 1024, 96, 1e-6, 4
    # residual rows with very different scales, some large outliers
    x = (rng.standard_normal((M, K)) * np.exp(rng.uniform(-3, 6, (M, 1)))).astype(np.float32)
    x[:, rng.integers(0, K, 8)] *= 50
    g = bf16_round((1 + 0.1 * rng.standard_normal(K)).astype(np.float32))
    W = bf16_round((0.02 * rng.standard_normal((N, K))).astype(np.float32))
    x64 = x.astype(np.float64)
    rms = np.sqrt((x64 ** 2).mean(axis=1, keepdims=True) + eps)
    ref = ((x64 / rms) * g) @ W.T.astype(np.float64)
    # the GPU method: per-tile row sums of x^2 (fp32), summed in tile order
    parts = [np.sum(x[:, t * K // tiles:(t + 1) * K // tiles] ** 2, axis=1, dtype=np.float32) for t in range(tiles)]
    ss = np.float32(0) + parts[0]
    for p in parts[1:]:
        ss = (ss + p).astype(np.float32)
    scale = (1.0 / np.sqrt(ss / np.float32(K) + np.float32(eps))).astype(np.float32)
    hi, lo = _hilo(g * x)
    acc = (hi.astype(np.float64) @ W.T.astype(np.float64) + lo.astype(np.float64) @ W.T.astype(np.float64))
    got = (acc.astype(np.float32) * scale[:, None]).astype(np.float64)
    err = np.abs(got - ref).max(axis=1) / np.abs(ref).max(axis=1)
    assert err.max() < 2e-5, err.max()
    # the plain bf16 operand (one plane) would be ~2^-9: the lo plane is what
    # keeps the prompt path at fp32-like accuracy
    one = (hi.astype(np.float64) @ W.T.astype(np.float64)).astype(np.float32) * scale[:, None]
    assert (np.abs(one - ref).max(axis=1) / np.abs(ref).max(axis=1)).max() > 10 * err.max()


def _blocks(S, L, start):
    """Key blocks of one chunk: [0, start) in blocks of L, then [start, S)."""
    b, k = [], 0
    while k < start:
        b.append((k, min(k + L, start)))
        k += L
    b.append((start, S))
    return b


def test_lse_merge_of_bf16_blocks_matches_full_softmax():
    rng = np.random.default_rng(7)
    d, S, L = 128, 3000, 512
    start = S - 200                              # the chunk's diagonal block: the last 200 keys
    q = rng.standard_normal((16, d))
    k = rng.standard_normal((S, d))
    v = rng.standard_normal((S, d))
    s2 = (q @ k.T) / np.sqrt(d) * np.log2(np.e)  # scaled scores, log2 domain
    p = np.exp2(s2 - s2.max(axis=1, keepdims=True))
    ref = (p @ v) / p.sum(axis=1, keepdims=True)
    lses, outs = [], []
    for a, b in _blocks(S, L, start):
        sb = s2[:, a:b]
        m = sb.max(axis=1, keepdims=True)
        l = np.exp2(sb - m).sum(axis=1, keepdims=True)
        o = (np.exp2(sb - m) @ v[a:b]) / l
        lses.append((m + np.log2(l))[:, 0].astype(np.float32))
        outs.append(bf16_round(o.astype(np.float32)))      # the pieces' bf16 outputs
    ls = np.stack(lses)                                     # [pieces, rows]
    mx = ls.max(axis=0)
    w = np.exp2(ls - mx)
    got = sum(w[i][:, None] * outs[i].astype(np.float64) for i in range(len(outs))) / w.sum(axis=0)[:, None]
    assert np.abs(got - ref).max() <= 2 ** -8 * np.abs(ref).max()
