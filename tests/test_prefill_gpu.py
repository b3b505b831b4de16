"""Parity of the tcgen05 causal prefill attention (sa_attn_prefill) with the
reference, through the C ABI.

The kernel multiplies bf16 operands (P is rounded to bf16 before P.V) with fp32
accumulation, so the bar is the one BASELINE.json sets for bf16 tensor-core
paths: max |err| <= 2e-2 x max |ref| (relative), with inputs that are exactly
representable in bf16 so the fp32 oracle sees the same values.
"""
import numpy as np
import pytest

import _inputs as I
from conftest import golden
from oracle.oracle import bf16_round

pytestmark = pytest.mark.gpu
REL = 2e-2


def _bf(x):
    import torch
    return torch.from_numpy(np.ascontiguousarray(x)).cuda().to(torch.bfloat16)


def _check(got, ref, what=""):
    err = float(np.abs(got - ref).max())
    scale = float(np.abs(ref).max())
    assert err <= REL * scale, f"{what}: max|err| {err:.3e} vs max|ref| {scale:.3e}"


def test_prefill_golden(ctx):
    import torch
    from streaming_attention_b200 import attn_prefill
    g = golden("causal_prefill.npz")
    for i, (S, hq, hkv, d) in enumerate(I.PREFILL_CASES):
        seed = int(g[f"c{i}_meta"][4])
        q, k, v = I.prefill(S, hq, hkv, d, seed)
        q, k, v = bf16_round(q), bf16_round(k), bf16_round(v)
        out = attn_prefill(_bf(q), _bf(k), _bf(v), 1.0 / np.sqrt(d), ctx=ctx)
        torch.cuda.synchronize()
        _check(out.cpu().numpy(), g[f"c{i}_blockwise"], f"case {i}")


@pytest.mark.parametrize("S", [1, 63, 64, 65, 127, 128, 129, 300, 777])
@pytest.mark.parametrize("hq,hkv", [(2, 1), (4, 2), (2, 2), (16, 8), (8, 2), (3, 1), (1, 1)])
def test_prefill_vs_oracle(ctx, oracle, S, hq, hkv):
    import torch
    from streaming_attention_b200 import attn_prefill
    q, k, v = I.prefill(S, hq, hkv, 128, seed=S * 31 + hq)
    q, k, v = bf16_round(q), bf16_round(k), bf16_round(v)
    s = 1.0 / np.sqrt(128)
    out = attn_prefill(_bf(q), _bf(k), _bf(v), s, ctx=ctx)
    outb = attn_prefill(_bf(q), _bf(k), _bf(v), s, out_dtype="bfloat16", ctx=ctx)
    torch.cuda.synchronize()
    ref = oracle.causal_prefill(q, k, v, s)
    _check(out.cpu().numpy(), ref, "fp32 out")
    _check(outb.float().cpu().numpy(), ref, "bf16 out")


@pytest.mark.parametrize("Sq,q_pos0", [(128, 128), (100, 37), (256, 512), (1, 999)])
def test_prefill_query_offset(ctx, oracle, Sq, q_pos0):
    """A chunk of queries at positions q_pos0.. against all earlier keys (the
    shape one rank of sequence-parallel prefill or a chunked prefill computes)."""
    import torch
    from streaming_attention_b200 import attn_prefill
    Skv = q_pos0 + Sq
    q, k, v = I.prefill(Skv, 4, 2, 128, seed=Sq + q_pos0)
    q, k, v = bf16_round(q), bf16_round(k), bf16_round(v)
    s = 1.0 / np.sqrt(128)
    out = attn_prefill(_bf(q[q_pos0:]), _bf(k), _bf(v), s, q_pos0=q_pos0, ctx=ctx)
    torch.cuda.synchronize()
    ref = oracle.causal_prefill(q[q_pos0:], k, v, s, q_pos0=q_pos0)
    _check(out.cpu().numpy(), ref, f"offset {q_pos0}")


@pytest.mark.parametrize("kind", ["wide", "negative", "ramp"])
def test_prefill_extreme_logits(ctx, oracle, kind):
    """Score ranges that exercise the running-max logic: logits with a spread
    of hundreds (the max moves many times, O is rescaled), rows whose logits
    are all far below zero (the first tile's max must replace the initial
    running max), and keys whose logits grow along the sequence."""
    import torch
    from streaming_attention_b200 import attn_prefill
    S, hq, hkv, d = 400, 4, 2, 128
    rs = np.random.default_rng(11)
    q = rs.standard_normal((S, hq, d)).astype(np.float32)
    k = rs.standard_normal((S, hkv, d)).astype(np.float32)
    v = rs.standard_normal((S, hkv, d)).astype(np.float32)
    scale = 1.0 / np.sqrt(d)
    if kind == "wide":
        scale = 1.0                                   # logits ~ N(0, 128)
    elif kind == "negative":
        k = np.abs(k) + 1.0
        q = -np.abs(q) - 2.0                          # every logit << 0
        scale = 1.0
    else:
        k = k + np.linspace(0.0, 4.0, S, dtype=np.float32)[:, None, None]
        q = np.abs(q)
        scale = 0.25
    q, k, v = bf16_round(q), bf16_round(k), bf16_round(v)
    out = attn_prefill(_bf(q), _bf(k), _bf(v), scale, ctx=ctx)
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    assert np.isfinite(got).all()
    _check(got, oracle.causal_prefill(q, k, v, scale), kind)


def test_prefill_strided_qkv_from_one_buffer(ctx, oracle):
    """Q, K, V as column slices of one fused [S, (hq+2*hkv)*d] projection output
    (the QKV GEMM's layout), read in place through their token strides."""
    import torch
    from streaming_attention_b200 import attn_prefill
    S, hq, hkv, d = 300, 16, 8, 128
    q, k, v = I.prefill(S, hq, hkv, d, seed=5)
    q, k, v = bf16_round(q), bf16_round(k), bf16_round(v)
    fused = np.concatenate([q.reshape(S, -1), k.reshape(S, -1), v.reshape(S, -1)], axis=1)
    ft = _bf(fused)
    qt = ft[:, :hq * d].view(S, hq, d)
    kt = ft[:, hq * d:(hq + hkv) * d].view(S, hkv, d)
    vt = ft[:, (hq + hkv) * d:].view(S, hkv, d)
    out = attn_prefill(qt, kt, vt, 1 / np.sqrt(d), ctx=ctx)
    torch.cuda.synchronize()
    _check(out.cpu().numpy(), oracle.causal_prefill(q, k, v, 1 / np.sqrt(d)), "strided")


def test_config3_full_size_vs_torch_fp32(ctx):
    """Q [8192, 16, 128], K/V [8192, 8, 128] bf16 N(0,1),
    causal, scale 1/sqrt(128), against torch fp32 attention on the same values."""
    import torch
    import torch.nn.functional as F
    from streaming_attention_b200 import attn_prefill
    S, hq, hkv, d = 8192, 16, 8, 128
    g = torch.Generator(device="cuda").manual_seed(3)
    q = torch.randn(S, hq, d, device="cuda", generator=g).to(torch.bfloat16)
    k = torch.randn(S, hkv, d, device="cuda", generator=g).to(torch.bfloat16)
    v = torch.randn(S, hkv, d, device="cuda", generator=g).to(torch.bfloat16)
    out = attn_prefill(q, k, v, 1 / np.sqrt(d), ctx=ctx)
    qf = q.float().transpose(0, 1)
    kf = k.float().transpose(0, 1).repeat_interleave(hq // hkv, dim=0)
    vf = v.float().transpose(0, 1).repeat_interleave(hq // hkv, dim=0)
    worst, scale = 0.0, 0.0
    for h0 in range(0, hq, 4):      # a few heads at a time keeps the S x S scores small
        ref = F.scaled_dot_product_attention(qf[h0:h0 + 4], kf[h0:h0 + 4], vf[h0:h0 + 4],
                                             is_causal=True).transpose(0, 1)
        worst = max(worst, (out[:, h0:h0 + 4] - ref).abs().max().item())
        scale = max(scale, ref.abs().max().item())
    torch.cuda.synchronize()
    assert worst <= REL * scale, (worst, scale)


def test_prefill_argument_errors(ctx):
    import torch
    from streaming_attention_b200 import SAError, attn_prefill
    q = torch.zeros(10, 3, 64, device="cuda", dtype=torch.bfloat16)
    k = torch.zeros(10, 1, 64, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(SAError):
        attn_prefill(q, k, k, 1.0, ctx=ctx)            # d = 64
    q = torch.zeros(10, 3, 128, device="cuda", dtype=torch.bfloat16)
    k = torch.zeros(10, 2, 128, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(SAError):
        attn_prefill(q, k, k, 1.0, ctx=ctx)            # hq % hkv != 0
    q = torch.zeros(10, 2, 128, device="cuda", dtype=torch.bfloat16)
    k = torch.zeros(10, 1, 128, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(SAError):
        attn_prefill(q, k[:5], k[:5], 1.0, ctx=ctx)    # Sq > Skv
