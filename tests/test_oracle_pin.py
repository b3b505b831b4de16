"""Pin the CPU oracle (oracle/sa_oracle.c) to the reference.

The oracle is trusted as the parity checker for the CUDA path only because it
reproduces (a) the committed golden fixtures generated from the reference's
own functions and (b) the reference library compiled from its sources
(oracle/_ref), when present.  CPU only.
"""
import numpy as np
import pytest

import _inputs as I
from conftest import golden
from oracle.oracle import Qwen3Cfg, bf16_round, make_qwen3_weights

TOL = 1e-5  # reference's own naive-vs-streaming threshold (test_streaming_attention.cpp:100)


def test_single_query_golden(oracle):
    g = golden("single_query.npz")
    for i, (T, d) in enumerate(I.SINGLE_CASES):
        T_, d_, seed, block = g[f"c{i}_meta"]
        assert (T_, d_) == (T, d)
        q, k, v = I.single_query(T, d, int(seed))
        assert I.digest(q, k, v) == str(g[f"c{i}_digest"])
        s = oracle.streaming(q, k, v, int(block))
        n = oracle.naive(q, k, v)
        c = oracle.chunked(q, k, v, int(block), 4)
        np.testing.assert_allclose(s, g[f"c{i}_streaming"], atol=TOL, rtol=0)
        np.testing.assert_allclose(n, g[f"c{i}_naive"], atol=TOL, rtol=0)
        np.testing.assert_allclose(c, g[f"c{i}_omp4"], atol=TOL, rtol=0)


def test_gqa_golden(oracle):
    g = golden("gqa_decode.npz")
    for i, (hq, hkv, T, d) in enumerate(I.GQA_CASES):
        seed = int(g[f"c{i}_meta"][4])
        q, k, v = I.gqa(hq, hkv, T, d, seed)
        assert I.digest(q, k, v) == str(g[f"c{i}_digest"])
        out = oracle.gqa_decode(q, k, v, 64, 1.0 / np.sqrt(d))
        np.testing.assert_allclose(out, g[f"c{i}_out"], atol=TOL, rtol=0)
        outb = oracle.gqa_decode(bf16_round(q), bf16_round(k), bf16_round(v), 64, 1.0 / np.sqrt(d))
        np.testing.assert_allclose(outb, g[f"c{i}_out_bf16in"], atol=TOL, rtol=0)


def test_prefill_golden(oracle):
    g = golden("causal_prefill.npz")
    for i, (S, hq, hkv, d) in enumerate(I.PREFILL_CASES):
        seed = int(g[f"c{i}_meta"][4])
        q, k, v = I.prefill(S, hq, hkv, d, seed)
        q, k, v = bf16_round(q), bf16_round(k), bf16_round(v)
        assert I.digest(q, k, v) == str(g[f"c{i}_digest"])
        out = oracle.causal_prefill(q, k, v, 1.0 / np.sqrt(d))
        np.testing.assert_allclose(out, g[f"c{i}_blockwise"], atol=TOL, rtol=0)
        assert float(g[f"c{i}_standard_gap"]) < TOL


def _tiny():
    g = golden("qwen3_tiny.npz")
    V, H, L, hq, hkv, D, Iq = [int(x) for x in g["cfg"]]
    cfg = Qwen3Cfg(vocab=V, hidden=H, n_layers=L, hq=hq, hkv=hkv, head_dim=D, inter=Iq,
                   eps=1e-6, theta=1e6)
    w = make_qwen3_weights(cfg, int(g["seeds"][0]))
    assert I.digest(w["embed"], w["layers"]) == str(g["weights_digest"])
    return g, cfg, w


def test_qwen3_forward_golden(oracle):
    g, cfg, w = _tiny()
    logits = oracle.qwen3_forward(cfg, w, g["ids"])
    np.testing.assert_allclose(logits[-4:], g["logits_last4"], atol=1e-4, rtol=0)


def test_qwen3_cached_decode_golden(oracle):
    """Greedy decode through the oracle's KV cache reproduces the reference's tokens."""
    g, cfg, w = _tiny()
    ids = g["ids"]
    max_seq = 64
    kc = np.zeros((cfg.n_layers, cfg.hkv, max_seq, cfg.head_dim), np.float32)
    vc = np.zeros_like(kc)
    lg = oracle.qwen3_forward(cfg, w, ids, kc, vc, max_seq, 0, all_logits=False)
    pos = len(ids)
    toks = []
    nxt = int(np.argmax(lg[0]))
    for step in range(len(g["greedy_tokens"])):
        toks.append(nxt)
        lg = oracle.qwen3_forward(cfg, w, np.array([nxt]), kc, vc, max_seq, pos, all_logits=False)
        np.testing.assert_allclose(lg[0], g["decode_logits"][step], atol=1e-4, rtol=0)
        pos += 1
        nxt = int(np.argmax(lg[0]))
    assert toks == [int(t) for t in g["greedy_tokens"]]


def test_merge_is_associative(oracle):
    q, k, v = I.single_query(3000, 128, 7)
    full = oracle.streaming(q, k, v, 64)
    cuts = [0, 100, 1000, 1001, 2999, 3000]
    parts = [oracle.partial(q, k, v, a, b, 64) for a, b in zip(cuts[:-1], cuts[1:])]
    _, _, o = oracle.merge(parts)
    np.testing.assert_allclose(o, full, atol=TOL, rtol=0)
    _, _, o2 = oracle.merge(parts[::-1])
    np.testing.assert_allclose(o2, full, atol=TOL, rtol=0)


def test_empty_partial_is_identity(oracle):
    q, k, v = I.single_query(100, 64, 3)
    m, l, o = oracle.partial(q, k, v, 50, 50, 64)
    assert m == -np.inf and l == 1.0 and not o.any()


# ---- live pin against the reference library (when it was built here) ------

@pytest.mark.parametrize("T,d", [(4096, 128), (777, 64), (300, 256)])
def test_oracle_matches_reference_live(oracle, reference, T, d):
    q, k, v = I.single_query(T, d, 11)
    np.testing.assert_allclose(oracle.streaming(q, k, v, 64), reference.streaming_serial(q, k, v, 64),
                               atol=TOL, rtol=0)
    np.testing.assert_allclose(oracle.naive(q, k, v), reference.naive_serial(q, k, v), atol=TOL, rtol=0)


def test_oracle_qwen3_matches_reference_live(oracle, reference):
    cfg = Qwen3Cfg(vocab=512, hidden=128, n_layers=2, hq=4, hkv=2, head_dim=64, inter=256,
                   eps=1e-6, theta=1e6)
    w = make_qwen3_weights(cfg, 5, std=0.05)
    ids = I.rng(6).integers(0, cfg.vocab, 12)
    m = reference.qwen3(cfg, w)
    np.testing.assert_allclose(oracle.qwen3_forward(cfg, w, ids), m.forward(ids), atol=1e-4, rtol=0)
