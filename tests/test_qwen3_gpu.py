"""Parity of the Qwen3 forward (sa_qwen3_*) with the reference, through the C ABI.

Weights are random-init N(0, 0.02) rounded to bf16 (the reference loads bf16
checkpoints), so the GPU's bf16 weights are exact; activations, the residual
stream and the KV cache are fp32 on both sides.  Bars: logits within 2e-3 of
max |logit| (the prompt GEMMs carry ~16 bits of activation mantissa, the
decode GEMVs full fp32), greedy tokens identical to the reference's.
"""
import numpy as np

from oracle.oracle import bf16_round
import pytest

import _inputs as I
from conftest import golden
from oracle.oracle import Qwen3Cfg, make_qwen3_weights

pytestmark = pytest.mark.gpu
REL = 2e-3
# prompts of >= 256 tokens run their attention on bf16 tensor cores: the
# bf16 tensor-core bar (BASELINE's 2e-2 relative) applies to their logits
REL_BF16 = 2e-2


def _cfgdict(c: Qwen3Cfg) -> dict:
    return dict(vocab=c.vocab, hidden=c.hidden, n_layers=c.n_layers, hq=c.hq, hkv=c.hkv,
                head_dim=c.head_dim, inter=c.inter, eps=c.eps, theta=c.theta)


def _close(got, ref, what="", rel=REL):
    err = float(np.abs(got - ref).max())
    scale = float(np.abs(ref).max())
    assert err <= rel * max(scale, 1e-3), f"{what}: max|err| {err:.3e} vs max|ref| {scale:.3e}"


def _tiny():
    g = golden("qwen3_tiny.npz")
    V, H, L, hq, hkv, D, Iq = [int(x) for x in g["cfg"]]
    cfg = Qwen3Cfg(vocab=V, hidden=H, n_layers=L, hq=hq, hkv=hkv, head_dim=D, inter=Iq, eps=1e-6, theta=1e6)
    w = make_qwen3_weights(cfg, int(g["seeds"][0]))
    return g, cfg, w


def test_qwen3_tiny_forward_golden(ctx):
    from streaming_attention_b200 import Qwen3
    g, cfg, w = _tiny()
    m = Qwen3(_cfgdict(cfg), max_seq=64, ctx=ctx)
    m.load(w)
    logits = m.forward(g["ids"])
    _close(logits[-4:], g["logits_last4"], "prefill logits")
    assert m.cache_len == 0


def test_qwen3_tiny_greedy_decode_golden(ctx):
    """Cached greedy decode reproduces the reference's tokens and logits."""
    from streaming_attention_b200 import Qwen3
    g, cfg, w = _tiny()
    m = Qwen3(_cfgdict(cfg), max_seq=64, ctx=ctx)
    m.load(w)
    n = len(g["greedy_tokens"])
    toks = m.generate(g["ids"], n)
    assert [int(t) for t in toks] == [int(t) for t in g["greedy_tokens"]]
    assert m.cache_len == len(g["ids"]) + n - 1
    # step by step through forward(use_cache) with logits checked
    m.reset()
    lg = m.forward(g["ids"], use_cache=True, logits="last")
    nxt = int(np.argmax(lg[0]))
    for step in range(n):
        lg = m.forward(np.array([nxt]), use_cache=True, logits="last")
        _close(lg[0], g["decode_logits"][step], f"decode step {step}")
        nxt = int(np.argmax(lg[0]))


@pytest.mark.parametrize("S", [1, 7, 128, 200])
def test_qwen3_vs_oracle_shapes(ctx, oracle, S):
    """Prompt lengths around the 128-row GEMM tile and the single-token GEMV path."""
    from streaming_attention_b200 import Qwen3
    cfg = Qwen3Cfg(vocab=1000, hidden=512, n_layers=3, hq=8, hkv=4, head_dim=128, inter=1536,
                   eps=1e-6, theta=1e6)
    w = make_qwen3_weights(cfg, 17)
    ids = I.rng(S).integers(0, cfg.vocab, S)
    m = Qwen3(_cfgdict(cfg), max_seq=256, ctx=ctx)
    m.load(w)
    got = m.forward(ids)
    ref = oracle.qwen3_forward(cfg, w, ids)
    _close(got, ref, f"S={S}")


@pytest.mark.parametrize("hq,hkv,S", [(4, 4, 33), (8, 2, 47), (8, 4, 16), (4, 1, 5)])
def test_qwen3_prompt_gqa_ratios(ctx, oracle, hq, hkv, S):
    """Prompt attention blocks hold 16 / G prompt rows of all G query heads of
    a KV head: G = 1, 2, 4 and prompt lengths that leave ragged last blocks."""
    from streaming_attention_b200 import Qwen3
    cfg = Qwen3Cfg(vocab=700, hidden=256, n_layers=2, hq=hq, hkv=hkv, head_dim=128, inter=512,
                   eps=1e-6, theta=1e6)
    w = make_qwen3_weights(cfg, 29)
    ids = I.rng(S + hq).integers(0, cfg.vocab, S)
    m = Qwen3(_cfgdict(cfg), max_seq=128, ctx=ctx)
    m.load(w)
    _close(m.forward(ids), oracle.qwen3_forward(cfg, w, ids), f"hq={hq} hkv={hkv} S={S}")


def test_qwen3_long_prompt(ctx, oracle):
    """A 1000-token prompt: eight 128-row GEMM tiles (the last ragged), so the
    projections run unsplit with 256-wide tiles, and eight attention rounds."""
    from streaming_attention_b200 import Qwen3
    cfg = Qwen3Cfg(vocab=600, hidden=256, n_layers=2, hq=4, hkv=2, head_dim=128, inter=512,
                   eps=1e-6, theta=1e6)
    w = make_qwen3_weights(cfg, 53)
    ids = I.rng(9).integers(0, cfg.vocab, 1000)
    m = Qwen3(_cfgdict(cfg), max_seq=1024, ctx=ctx)
    m.load(w)
    _close(m.forward(ids, logits="all"), oracle.qwen3_forward(cfg, w, ids, all_logits=True), "S=1000")


@pytest.mark.parametrize("hq,hkv,S,cached", [(4, 2, 1100, 0), (8, 2, 1300, 200), (4, 4, 2048, 0)])
def test_qwen3_prompt_tensor_core_attention(ctx, oracle, hq, hkv, S, cached):
    """Prompts of >= 256 tokens run their attention on the tcgen05 prefill
    kernel (bf16 q / K / V, fp32 accumulation): logits of every position
    within the bar, and greedy tokens after the prompt identical to the
    oracle's; also a chunk of 1300 - 200 = 1100 tokens after a 200-token
    cached prefix (the tensor-core attention over prefix + chunk)."""
    from streaming_attention_b200 import Qwen3
    cfg = Qwen3Cfg(vocab=700, hidden=256, n_layers=2, hq=hq, hkv=hkv, head_dim=128, inter=512,
                   eps=1e-6, theta=1e6)
    w = make_qwen3_weights(cfg, 61)
    ids = I.rng(S).integers(0, cfg.vocab, S)
    m = Qwen3(_cfgdict(cfg), max_seq=S + 16, ctx=ctx)
    m.load(w)
    ref = oracle.qwen3_forward(cfg, w, ids, all_logits=True)
    if cached:
        m.forward(ids[:cached], use_cache=True, logits="none")
        got = m.forward(ids[cached:], use_cache=True, logits="all")
        _close(got, ref[cached:], f"S={S} after {cached} cached rows")
        return
    _close(m.forward(ids, logits="all"), ref, f"S={S}")
    toks = m.generate(ids, 6)
    L, D = cfg.n_layers, cfg.head_dim
    kc = np.zeros((L, hkv, S + 16, D), np.float32)
    vc = np.zeros_like(kc)
    lg = oracle.qwen3_forward(cfg, w, ids, kc, vc, S + 16, 0, all_logits=False)
    want, pos = [int(np.argmax(lg[0]))], S
    for _ in range(5):
        lg = oracle.qwen3_forward(cfg, w, np.array(want[-1:]), kc, vc, S + 16, pos, all_logits=False)
        pos += 1
        want.append(int(np.argmax(lg[0])))
    assert [int(t) for t in toks] == want


# The 0.6B layer shapes (hidden 1024, 16 / 8 heads, intermediate 3072) at a
# prompt long enough that all four projections run unsplit, so every fused
# GEMM epilogue runs: QKV with QK-norm + RoPE + cache append, o_proj and
# down_proj writing the next GEMM's operand with its RMSNorm deferred, gate/up
# and QKV scaling their rows by 1 / rms.
FUSED_CFG = dict(vocab=2000, hidden=1024, n_layers=2, hq=16, hkv=8, head_dim=128, inter=3072, eps=1e-6, theta=1e6)
FUSED_S = 3500

_FUSED_SCRIPT = """
import sys, numpy as np
sys.path.insert(0, sys.argv[1]); sys.path.insert(0, sys.argv[1] + "/tests")
import _inputs as I
from oracle.oracle import Qwen3Cfg, make_qwen3_weights
from streaming_attention_b200 import Context, Qwen3
cfg = dict(%s)
w = make_qwen3_weights(Qwen3Cfg(**cfg), 71)
ids = I.rng(%d).integers(0, cfg["vocab"], %d)
ctx = Context(0)
m = Qwen3(cfg, max_seq=%d + 16, ctx=ctx)
m.load(w)
np.save(sys.argv[2], m.forward(ids, logits="all"))
m.close(); ctx.close()
"""


def _fused_ref(oracle):
    cfg = Qwen3Cfg(**FUSED_CFG)
    w = make_qwen3_weights(cfg, 71)
    ids = I.rng(FUSED_S).integers(0, cfg.vocab, FUSED_S)
    return cfg, w, ids


def test_qwen3_fused_epilogues_fp32_attention(oracle, tmp_path):
    """Fused prompt GEMM epilogues with the fp32 prompt attention (the
    tensor-core crossover raised past the prompt, in a child process since
    the crossover is read once per process): every position's logits within
    the fp32 bar (2e-3 of max |logit|)."""
    import os
    import subprocess
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    cfg_src = ", ".join(f"{k}={v!r}" for k, v in FUSED_CFG.items())
    out = tmp_path / "logits.npy"
    env = dict(os.environ, SA_QWEN3_TC_ATTN_MIN="1000000")
    r = subprocess.run([sys.executable, "-c", _FUSED_SCRIPT % (cfg_src, FUSED_S, FUSED_S, FUSED_S), root, str(out)],
                       env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout + r.stderr
    cfg, w, ids = _fused_ref(oracle)
    ref = oracle.qwen3_forward(cfg, w, ids, all_logits=True)
    got = np.load(out)
    for r0 in range(0, FUSED_S, 500):
        _close(got[r0:r0 + 500], ref[r0:r0 + 500], f"fused epilogues, fp32 attention, rows {r0}..")


def test_qwen3_fused_epilogues_tensor_core_attention(ctx, oracle):
    """The same prompt with its attention on the tensor cores (q / K / V
    written in bf16 by the QKV epilogue, the output as the o_proj operand's
    hi / lo planes): logits within the bf16 bar, then greedy tokens equal to
    the oracle's."""
    from streaming_attention_b200 import Qwen3
    cfg, w, ids = _fused_ref(oracle)
    S, n_new = FUSED_S, 4
    m = Qwen3(FUSED_CFG, max_seq=S + 16, ctx=ctx)
    m.load(w)
    ref = oracle.qwen3_forward(cfg, w, ids, all_logits=True)
    _close(m.forward(ids, logits="all"), ref, "fused epilogues, tensor-core attention", REL_BF16)
    ref_toks, gaps, _ = _oracle_greedy(oracle, cfg, w, ids, n_new, S + 16)
    _same_tokens(m.generate(ids, n_new), ref_toks, gaps, "fused epilogues, 4 new tokens")
    m.close()


def test_qwen3_long_prefix_continuation(ctx, oracle):
    """A 40-token prompt continued after 300 cached tokens: its attention runs
    over several 128-row rounds of the cache."""
    from streaming_attention_b200 import Qwen3
    cfg = Qwen3Cfg(vocab=500, hidden=256, n_layers=2, hq=4, hkv=2, head_dim=128, inter=512,
                   eps=1e-6, theta=1e6)
    w = make_qwen3_weights(cfg, 41)
    ids = I.rng(8).integers(0, cfg.vocab, 340)
    m = Qwen3(_cfgdict(cfg), max_seq=400, ctx=ctx)
    m.load(w)
    m.forward(ids[:300], use_cache=True, logits="none")
    part = m.forward(ids[300:], use_cache=True, logits="all")
    ref = oracle.qwen3_forward(cfg, w, ids, all_logits=True)[300:]
    _close(part, ref, "continuation after 300 cached rows")


def test_qwen3_cache_continuation_matches_full_prompt(ctx, oracle):
    """A prompt fed in two chunks through the cache equals one pass over the
    whole prompt (the KVCache append/advance contract)."""
    from streaming_attention_b200 import Qwen3
    cfg = Qwen3Cfg(vocab=500, hidden=256, n_layers=2, hq=4, hkv=2, head_dim=128, inter=512,
                   eps=1e-6, theta=1e6)
    w = make_qwen3_weights(cfg, 3)
    ids = I.rng(4).integers(0, cfg.vocab, 150)
    m = Qwen3(_cfgdict(cfg), max_seq=200, ctx=ctx)
    m.load(w)
    full = m.forward(ids, logits="last")
    m.reset()
    m.forward(ids[:100], use_cache=True, logits="none")
    part = m.forward(ids[100:], use_cache=True, logits="last")
    assert m.cache_len == 150
    _close(part, full, "chunked")
    _close(full[0], oracle.qwen3_forward(cfg, w, ids, all_logits=False)[0], "oracle")


def test_qwen3_kv_mirror_read_write(ctx, oracle):
    """The device cache read back after a cached prefill equals the oracle's
    KVCache contents; a second model that adopts it (write_kv + set_cache_len,
    the path for a host KVCache filled elsewhere) continues bit-identically."""
    from streaming_attention_b200 import Qwen3
    cfg = Qwen3Cfg(vocab=500, hidden=256, n_layers=2, hq=4, hkv=2, head_dim=128, inter=512,
                   eps=1e-6, theta=1e6)
    w = make_qwen3_weights(cfg, 5)
    S, MS = 40, 64
    ids = I.rng(9).integers(0, cfg.vocab, S)
    m = Qwen3(_cfgdict(cfg), max_seq=MS, ctx=ctx)
    m.load(w)
    m.forward(ids, use_cache=True, logits="none")
    kc = np.zeros((cfg.n_layers, cfg.hkv, MS, cfg.head_dim), np.float32)
    vc = np.zeros_like(kc)
    oracle.qwen3_forward(cfg, w, ids, kc=kc, vc=vc, max_seq=MS, all_logits=False)
    m2 = Qwen3(_cfgdict(cfg), max_seq=MS, ctx=ctx)
    m2.load(w)
    for layer in range(cfg.n_layers):
        k, v = m.read_kv(layer, seq_stride=MS)
        assert not k[:, S:].any() and not v[:, S:].any()
        _close(k[:, :S], kc[layer, :, :S], f"K layer {layer}")
        _close(v[:, :S], vc[layer, :, :S], f"V layer {layer}")
        k, v = m.read_kv(layer)
        assert k.shape == (cfg.hkv, S, cfg.head_dim)
        m2.write_kv(layer, k, v)
    m2.set_cache_len(S)
    a = m.forward(np.array([7]), use_cache=True, logits="last")
    b = m2.forward(np.array([7]), use_cache=True, logits="last")
    np.testing.assert_array_equal(a, b)
    assert m.cache_len == m2.cache_len == S + 1


@pytest.mark.parametrize("dtype,tied", [("BF16", True), ("BF16", False), ("F32", True), ("F16", True)])
def test_qwen3_from_safetensors_equals_load(ctx, tmp_path, dtype, tied):
    """A model uploaded straight from a safetensors checkpoint (bf16 bytes to
    the GPU) computes exactly what the same weights uploaded through
    sa_qwen3_set_layer compute; F16 checkpoints hold the weights rounded to
    fp16, so they agree within the logits bar."""
    from streaming_attention_b200 import Qwen3
    from streaming_attention_b200.checkpoint import write_qwen3_safetensors
    from streaming_attention_b200.qwen3 import random_weights
    cfg = dict(vocab=600, hidden=256, n_layers=2, hq=4, hkv=2, head_dim=128, inter=512, eps=1e-6, theta=1e6)
    w = random_weights(cfg, 21)
    w["final_norm"] = bf16_round(np.linspace(0.5, 1.5, cfg["hidden"], dtype=np.float32))
    if not tied:
        w["lm_head"] = random_weights(cfg, 22)["embed"]
    path = str(tmp_path / "m.safetensors")
    write_qwen3_safetensors(path, cfg, w, dtype=dtype, tied=tied)
    a = Qwen3(cfg, max_seq=64, ctx=ctx)
    a.load(w)
    b = Qwen3.from_safetensors(path, max_seq=64, ctx=ctx)
    assert b.cfg["n_layers"] == 2 and b.cfg["hq"] == 4
    ids = I.rng(5).integers(0, cfg["vocab"], 20)
    la, lb = a.forward(ids), b.forward(ids)
    if dtype == "F16":
        _close(lb, la, "f16 checkpoint")
    else:
        np.testing.assert_array_equal(lb, la)
    assert [int(t) for t in a.generate(ids, 5)] == [int(t) for t in b.generate(ids, 5)]


@pytest.mark.parametrize("prompt_len,n_new", [(5, 40), (300, 24)])
def test_qwen3_single_launch_step_matches_kernel_graph(ctx, monkeypatch, prompt_len, n_new):
    """Greedy decode through the single-launch step (one cooperative kernel per
    token, SA_QWEN3_MEGA=1) yields the tokens of the multi-kernel CUDA-graph
    step (the default) on a model with Qwen3-0.6B's layer shapes, and leaves
    the same KV cache."""
    from streaming_attention_b200 import Qwen3
    from streaming_attention_b200.qwen3 import random_weights
    cfg = dict(vocab=32000, hidden=1024, n_layers=4, hq=16, hkv=8, head_dim=128, inter=3072, eps=1e-6, theta=1e6)
    w = random_weights(cfg, 31)
    ids = I.rng(prompt_len).integers(0, cfg["vocab"], prompt_len)
    monkeypatch.setenv("SA_QWEN3_MEGA", "1")
    a = Qwen3(cfg, max_seq=512, ctx=ctx)
    a.load(w)
    ta = [int(t) for t in a.generate(ids, n_new)]
    monkeypatch.delenv("SA_QWEN3_MEGA")
    b = Qwen3(cfg, max_seq=512, ctx=ctx)
    b.load(w)
    tb = [int(t) for t in b.generate(ids, n_new)]
    assert ta == tb
    assert a.cache_len == b.cache_len == prompt_len + n_new - 1
    for layer in (0, cfg["n_layers"] - 1):
        ka, va = a.read_kv(layer)
        kb, vb = b.read_kv(layer)
        _close(ka, kb, f"K cache layer {layer}")
        _close(va, vb, f"V cache layer {layer}")
    # and a second generate on the same model continues from its cache
    monkeypatch.setenv("SA_QWEN3_MEGA", "1")
    more = [int(t) for t in a.generate(np.array([ta[-1]]), 4)]
    monkeypatch.delenv("SA_QWEN3_MEGA")
    assert len(more) == 4 and a.cache_len == prompt_len + n_new - 1 + 4


def test_qwen3_errors(ctx):
    from streaming_attention_b200 import Qwen3, SAError
    cfg = dict(vocab=300, hidden=256, n_layers=1, hq=2, hkv=1, head_dim=128, inter=256)
    m = Qwen3(cfg, max_seq=8, ctx=ctx)
    with pytest.raises(SAError):           # weights not loaded
        m.forward([1, 2])
    w = make_qwen3_weights(Qwen3Cfg(vocab=300, hidden=256, n_layers=1, hq=2, hkv=1, head_dim=128,
                                    inter=256, eps=1e-6, theta=1e6), 1)
    m.load(w)
    with pytest.raises(SAError) as e:      # embedding index out of range (ops.cpp:296)
        m.forward([1, 300])
    assert e.value.code == -6
    m.forward(list(range(8)), use_cache=True, logits="none")
    with pytest.raises(SAError) as e:      # KV cache full (kv_cache.h:109-111)
        m.forward([1], use_cache=True)
    assert e.value.code == -7


@pytest.fixture(scope="module")
def q06():
    """The real Qwen3-0.6B architecture with seeded random-init weights
    (BASELINE configs[3] / [4]), generated once for the module."""
    from streaming_attention_b200 import QWEN3_0_6B
    cfg = Qwen3Cfg(**{k: QWEN3_0_6B[k] for k in ("vocab", "hidden", "n_layers", "hq", "hkv", "head_dim",
                                                   "inter", "eps", "theta")})
    return cfg, make_qwen3_weights(cfg, 2026)


@pytest.fixture(scope="module")
def q06_model(q06, ctx):
    from streaming_attention_b200 import QWEN3_0_6B, Qwen3
    m = Qwen3(QWEN3_0_6B, max_seq=Q06_MAX_SEQ, ctx=ctx)
    m.load(q06[1])
    yield m
    m.close()


Q06_MAX_SEQ = 4096 + 16


def _oracle_greedy(oracle, cfg, w, prompt, n, max_seq):
    """The oracle's cached greedy decode (qwen3_forward_with_cache STANDARD,
    qwen3_ops.cpp:936-1014, then ops::argmax): the prompt, then n-1 one-token
    steps.  Returns the n tokens, the top-1 minus top-2 logit gap at each
    choice, and the prompt's last-token logits."""
    kc = np.zeros((cfg.n_layers, cfg.hkv, max_seq, cfg.head_dim), np.float32)
    vc = np.zeros_like(kc)
    lg = oracle.qwen3_forward(cfg, w, prompt, kc, vc, max_seq, 0, all_logits=False)[0]
    first = lg.copy()
    toks, gaps, pos = [], [], len(prompt)
    for i in range(n):
        top2 = np.partition(lg, -2)[-2:]
        gaps.append(float(top2[1] - top2[0]))
        nxt = int(np.argmax(lg))
        toks.append(nxt)
        if i + 1 < n:
            lg = oracle.qwen3_forward(cfg, w, np.array([nxt]), kc, vc, max_seq, pos, all_logits=False)[0]
            pos += 1
    return toks, gaps, first


def _same_tokens(got, ref, gaps, what):
    got = [int(t) for t in got]
    if got != ref:
        i = next(j for j in range(len(ref)) if got[j] != ref[j])
        pytest.fail(f"{what}: greedy token {i} differs (GPU {got[i]}, oracle {ref[i]}); the oracle's "
                    f"top-1 minus top-2 logit gap there is {gaps[i]:.3e}")


def test_qwen3_0_6b_prefill_and_100_greedy_tokens(q06, q06_model, oracle):
    """logits of all 128 prompt positions (qwen3_forward) within
    the bar; configs[4] first run: the 100 greedy tokens after the 128-token
    prompt identical to the oracle's cached decode."""
    cfg, w = q06
    m = q06_model
    ids = I.rng(42).integers(0, cfg.vocab, 128)
    m.reset()
    got = m.forward(ids, logits="all")
    ref = oracle.qwen3_forward(cfg, w, ids)
    for r in range(0, 128, 16):
        _close(got[r:r + 16], ref[r:r + 16], f"prefill logits rows {r}..{r + 15}")
    toks = m.generate(ids, 100)
    ref_toks, gaps, last = _oracle_greedy(oracle, cfg, w, ids, 100, 128 + 100)
    _close(got[-1], last, "last-token logits (cached forward)")
    _same_tokens(toks, ref_toks, gaps, "128-token prompt, 100 new tokens")


def test_qwen3_0_6b_4096_token_prompt(q06, q06_model, oracle):
    """configs[4] second run: a 4096-token prompt, then long-KV decode: the
    prompt's last-token logits within the bf16 tensor-core bar (its attention
    runs on the tcgen05 prefill kernel; measured 2.8e-3 of max |logit|) and
    the greedy tokens identical to the oracle's (8 new tokens keep the
    oracle's CPU time bounded)."""
    cfg, w = q06
    m = q06_model
    ids = I.rng(4096).integers(0, cfg.vocab, 4096)
    n_new = 8
    ref_toks, gaps, last = _oracle_greedy(oracle, cfg, w, ids, n_new, 4096 + n_new)
    m.reset()
    lg = m.forward(ids, use_cache=True, logits="last")
    assert m.cache_len == 4096
    _close(lg[0], last, "4096-token prompt, last-token logits", REL_BF16)
    m.reset()
    toks = m.generate(ids, n_new)
    _same_tokens(toks, ref_toks, gaps, "4096-token prompt, 8 new tokens")


def test_qwen3_graph_replay_and_cache_isolation(ctx):
    """Cache-free forwards of one shape run eagerly, then captured, then
    replayed (CUDA graph): identical logits each time; a cache-free forward
    leaves a live KV cache untouched (qwen3_forward never touches KVCache);
    a second generate() reuses the captured decode step."""
    from streaming_attention_b200 import Qwen3
    cfg = Qwen3Cfg(vocab=700, hidden=256, n_layers=2, hq=4, hkv=2, head_dim=128, inter=512,
                   eps=1e-6, theta=1e6)
    w = make_qwen3_weights(cfg, 8)
    m = Qwen3(_cfgdict(cfg), max_seq=256, ctx=ctx)
    m.load(w)
    ids = I.rng(1).integers(0, cfg.vocab, 40)
    outs = [m.forward(ids) for _ in range(3)]
    assert np.array_equal(outs[0], outs[1]) and np.array_equal(outs[1], outs[2])
    # live cache + an interleaved cache-free forward
    prompt = I.rng(2).integers(0, cfg.vocab, 30)
    a = m.generate(prompt, 5)
    m.reset()
    m.forward(prompt, use_cache=True, logits="none")
    m.forward(ids, logits="last")                       # must not disturb the cache
    assert m.cache_len == 30
    lg = m.forward(np.array([a[0]]), use_cache=True, logits="last")
    assert int(np.argmax(lg[0])) == int(a[1])
    m.reset()
    b = m.generate(prompt, 5)
    assert [int(x) for x in a] == [int(x) for x in b]
