"""Parity of the CUDA decode attention (sa_attn_decode / _partial / sa_attn_merge)
with the reference, through the C ABI.

Tolerances: 1e-4 max-abs for fp32 paths (the bar BASELINE.json sets for fp32;
the reference's own OMP-vs-serial threshold, test_streaming_attention.cpp:178-251).
bf16 inputs here are exactly representable in bf16 and the kernel computes in
fp32, so the same 1e-4 applies to them.
"""
import ctypes as C

import numpy as np
import pytest

import _inputs as I
from conftest import golden
from oracle.oracle import bf16_round

pytestmark = pytest.mark.gpu
TOL = 1e-4


def _t(x, dtype="float32"):
    import torch
    t = torch.from_numpy(np.ascontiguousarray(x)).cuda()
    return t.to(getattr(torch, dtype))


def test_single_query_golden_host_ptrs(ctx):
    """attention.h drop-in: host buffers in, d-vector out, unscaled."""
    from streaming_attention_b200 import naive_attention_cuda, streaming_attention_cuda
    g = golden("single_query.npz")
    for i, (T, d) in enumerate(I.SINGLE_CASES):
        seed = int(g[f"c{i}_meta"][2])
        q, k, v = I.single_query(T, d, seed)
        out = streaming_attention_cuda(q, k, v, T, d, 64, ctx=ctx)
        np.testing.assert_allclose(out, g[f"c{i}_streaming"], atol=TOL, rtol=0, err_msg=f"T={T} d={d}")
        np.testing.assert_allclose(out, g[f"c{i}_naive"], atol=TOL, rtol=0)
        out2 = naive_attention_cuda(q, k, v, T, d, ctx=ctx)
        np.testing.assert_array_equal(out, out2)


def test_gqa_golden_device_ptrs(ctx):
    import torch
    from streaming_attention_b200 import attn_decode
    g = golden("gqa_decode.npz")
    for i, (hq, hkv, T, d) in enumerate(I.GQA_CASES):
        seed = int(g[f"c{i}_meta"][4])
        q, k, v = I.gqa(hq, hkv, T, d, seed)
        s = 1.0 / np.sqrt(d)
        out = attn_decode(_t(q), _t(k), _t(v), s, 64, ctx)
        torch.cuda.synchronize()
        np.testing.assert_allclose(out.cpu().numpy(), g[f"c{i}_out"], atol=TOL, rtol=0,
                                   err_msg=f"case {i}")
        outb = attn_decode(_t(q, "bfloat16"), _t(k, "bfloat16"), _t(v, "bfloat16"), s, 64, ctx)
        torch.cuda.synchronize()
        np.testing.assert_allclose(outb.cpu().numpy(), g[f"c{i}_out_bf16in"], atol=TOL, rtol=0,
                                   err_msg=f"bf16 case {i}")


@pytest.mark.parametrize("d", [64, 128, 256])
@pytest.mark.parametrize("hq,hkv", [(1, 1), (2, 1), (4, 1), (16, 8)])
@pytest.mark.parametrize("T", [1, 31, 32, 33, 500, 4097])
@pytest.mark.parametrize("dtype", ["float32", "bfloat16"])
def test_decode_vs_oracle_ragged(ctx, oracle, d, hq, hkv, T, dtype):
    import torch
    from streaming_attention_b200 import attn_decode
    if hq // hkv == 4 and d == 256:
        pytest.skip("G=4 is built for d <= 128")
    q, k, v = I.gqa(hq, hkv, T, d, seed=T * 7 + d + hq)
    if dtype == "bfloat16":
        q, k, v = bf16_round(q), bf16_round(k), bf16_round(v)
    s = 1.0 / np.sqrt(d)
    out = attn_decode(_t(q, dtype), _t(k, dtype), _t(v, dtype), s, 64, ctx)
    torch.cuda.synchronize()
    ref = oracle.gqa_decode(q, k, v, 64, s)
    np.testing.assert_allclose(out.cpu().numpy(), ref, atol=TOL, rtol=0)


def test_empty_sequence_gives_zeros(ctx):
    import torch
    from streaming_attention_b200 import attn_decode, attn_decode_partial
    q = torch.randn(4, 128, device="cuda")
    k = torch.empty(2, 0, 128, device="cuda")
    out = attn_decode(q, k, k, 1.0, 64, ctx)
    m, l, o = attn_decode_partial(q, k, k, 1.0, 64, ctx)
    torch.cuda.synchronize()
    assert not out.any() and not o.any()
    assert torch.isinf(m).all() and (m < 0).all() and (l == 1).all()


def test_partial_merge_equals_full_sequence_parallel(ctx, oracle):
    """KV split into shards (as streaming_attention_mpi_simple splits it over
    ranks), each reduced to a partial, then merged: equals the unsplit result."""
    import torch
    from streaming_attention_b200 import attn_decode, attn_decode_partial, attn_merge
    hq, hkv, T, d = 16, 8, 10000, 128
    q, k, v = I.gqa(hq, hkv, T, d, 42)
    s = 1 / np.sqrt(d)
    qt, kt, vt = _t(q), _t(k), _t(v)
    full = attn_decode(qt, kt, vt, s, 64, ctx)
    cuts = [0, 2500, 2501, 7000, 10000]
    ms, ls, os_ = [], [], []
    for a, b in zip(cuts[:-1], cuts[1:]):
        m, l, o = attn_decode_partial(qt, kt[:, a:b].contiguous(), vt[:, a:b].contiguous(), s, 64, ctx)
        ms.append(m.clone()); ls.append(l.clone()); os_.append(o.clone())
    merged, mm, lm = attn_merge(torch.stack(ms), torch.stack(ls), torch.stack(os_), ctx, with_state=True)
    mfull, lfull, _ = attn_decode_partial(qt, kt, vt, s, 64, ctx)
    torch.cuda.synchronize()
    np.testing.assert_allclose(merged.cpu().numpy(), full.cpu().numpy(), atol=TOL, rtol=0)
    np.testing.assert_allclose(merged.cpu().numpy(), oracle.gqa_decode(q, k, v, 64, s), atol=TOL, rtol=0)
    np.testing.assert_allclose(mm.cpu().numpy(), mfull.cpu().numpy(), rtol=1e-5)
    np.testing.assert_allclose(lm.cpu().numpy(), lfull.cpu().numpy(), rtol=1e-4)


def test_partial_state_matches_oracle(ctx, oracle):
    from streaming_attention_b200 import attn_decode_partial
    q, k, v = I.single_query(3000, 128, 5)
    m, l, o = attn_decode_partial(q.reshape(1, -1), k.reshape(1, 3000, 128), v.reshape(1, 3000, 128),
                                  1.0, 64, ctx)
    rm, rl, ro = oracle.partial(q, k, v, 0, 3000, 64)
    np.testing.assert_allclose(o[0], ro, atol=TOL, rtol=0)
    assert abs(m[0] - rm) <= 1e-4 * max(1.0, abs(rm))
    np.testing.assert_allclose(l[0], rl, rtol=1e-4)


def test_host_merge_matches_oracle_merge(ctx, oracle):
    from streaming_attention_b200 import attn_merge
    q, k, v = I.single_query(2000, 64, 9)
    parts = [oracle.partial(q, k, v, a, b, 64) for a, b in [(0, 10), (10, 10), (10, 1999), (1999, 2000)]]
    m = np.array([[p[0]] for p in parts], np.float32)
    l = np.array([[p[1]] for p in parts], np.float32)
    o = np.stack([p[2][None] for p in parts])
    out = attn_merge(m, l, o, ctx)
    np.testing.assert_allclose(out[0], oracle.merge(parts)[2], atol=TOL, rtol=0)


def test_config1_full_size(ctx, oracle):
    """q in R^128 over K, V in R^{8192x128}, N(0,1), scale
    1/sqrt(128), block 64, vs the naive serial softmax."""
    from streaming_attention_b200 import attn_decode
    q, k, v = I.single_query(8192, 128, 1)
    s = 1 / np.sqrt(128)
    out = attn_decode(q.reshape(1, 128), k.reshape(1, 8192, 128), v.reshape(1, 8192, 128), s, 64, ctx)
    np.testing.assert_allclose(out[0], oracle.naive(q, k, v, s), atol=TOL, rtol=0)
    # unscaled, as attention.h computes it
    out1 = attn_decode(q.reshape(1, 128), k.reshape(1, 8192, 128), v.reshape(1, 8192, 128), 1.0, 64, ctx)
    np.testing.assert_allclose(out1[0], oracle.naive(q, k, v, 1.0), atol=TOL, rtol=0)


@pytest.mark.parametrize("T", [65536, 262144])
@pytest.mark.parametrize("dtype", ["float32", "bfloat16"])
def test_config2_full_size_vs_fp64(ctx, T, dtype):
    """BASELINE config 2 sizes (hq 16, hkv 8, d 128) against a float64 torch
    evaluation of softmax(s*qK^T)V on the same (bf16-representable) values."""
    import torch
    from streaming_attention_b200 import attn_decode
    g = torch.Generator(device="cuda").manual_seed(T)
    hq, hkv, d = 16, 8, 128
    q = torch.randn(hq, d, device="cuda", generator=g).to(getattr(torch, dtype))
    k = torch.randn(hkv, T, d, device="cuda", generator=g).to(getattr(torch, dtype))
    v = torch.randn(hkv, T, d, device="cuda", generator=g).to(getattr(torch, dtype))
    s = 1 / np.sqrt(d)
    out = attn_decode(q, k, v, s, 64, ctx)
    kk = k.double().repeat_interleave(hq // hkv, dim=0)
    vv = v.double().repeat_interleave(hq // hkv, dim=0)
    sc = torch.einsum("hd,htd->ht", q.double(), kk) * s
    ref = torch.einsum("ht,htd->hd", torch.softmax(sc, dim=-1), vv)
    torch.cuda.synchronize()
    assert (out.double() - ref).abs().max().item() < TOL


def test_deterministic_and_host_equals_device(ctx):
    import torch
    from streaming_attention_b200 import attn_decode
    q, k, v = I.gqa(16, 8, 20000, 128, 3)
    a = attn_decode(_t(q), _t(k), _t(v), 0.1, 64, ctx)
    b = attn_decode(_t(q), _t(k), _t(v), 0.1, 64, ctx)
    c = attn_decode(q, k, v, 0.1, 64, ctx)
    torch.cuda.synchronize()
    assert torch.equal(a, b)
    np.testing.assert_array_equal(a.cpu().numpy(), c)


def test_argument_errors(ctx):
    import torch
    from streaming_attention_b200 import SAError, attn_decode, lib
    q = torch.randn(2, 96, device="cuda")
    k = torch.randn(1, 10, 96, device="cuda")
    with pytest.raises(SAError) as e:
        attn_decode(q, k, k, 1.0, 64, ctx)
    assert e.value.code == -1 and "d = 96" in str(e.value)
    q = torch.randn(3, 128, device="cuda")
    k = torch.randn(2, 10, 128, device="cuda")
    with pytest.raises(SAError):
        attn_decode(q, k, k, 1.0, 64, ctx)      # hq % hkv != 0
    buf = torch.randn(4 * 10 * 128 + 1, device="cuda")
    kk = buf[1:]                                # misaligned by 4 bytes
    out = torch.empty(4, 128, device="cuda")
    qq = torch.randn(4, 128, device="cuda")
    rc = lib().sa_attn_decode(ctx.h, 0, C.c_void_p(qq.data_ptr()), C.c_void_p(kk.data_ptr()),
                              C.c_void_p(kk.data_ptr()), 10 * 128, 10, 128, 4, 4, 64, 1.0,
                              C.c_void_p(out.data_ptr()), 0)
    assert rc == -1 and b"aligned" in lib().sa_last_error()
    ctx.synchronize()


def test_decode_step_appends_and_attends(ctx, oracle):
    """KV-cache decode step: the new row lands at `pos` and attention covers
    rows [0, pos] (kv_cache.h:94-130 + qwen3_ops.cpp:876-885)."""
    import torch
    from streaming_attention_b200 import attn_decode_step
    hq, hkv, d, max_seq, pos = 16, 8, 128, 5000, 4000
    q, k, v = I.gqa(hq, hkv, max_seq, d, 77)
    kc, vc = _t(k), _t(v)
    kn, vn = k[:, pos].copy() + 1.0, v[:, pos].copy() - 1.0
    s = 1 / np.sqrt(d)
    out = attn_decode_step(q, kn, vn, kc, vc, pos, s, 64, ctx)       # host q/k/v/out
    k2, v2 = k.copy(), v.copy()
    k2[:, pos], v2[:, pos] = kn, vn
    ref = oracle.gqa_decode(q, np.ascontiguousarray(k2[:, :pos + 1]), np.ascontiguousarray(v2[:, :pos + 1]), 64, s)
    np.testing.assert_allclose(out, ref, atol=TOL, rtol=0)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(kc[:, pos].cpu().numpy(), kn)
    # device-pointer variant on the next position
    out2 = attn_decode_step(_t(q), _t(kn), _t(vn), kc, vc, pos + 1, s, 64, ctx)
    torch.cuda.synchronize()
    k2[:, pos + 1], v2[:, pos + 1] = kn, vn
    ref2 = oracle.gqa_decode(q, np.ascontiguousarray(k2[:, :pos + 2]), np.ascontiguousarray(v2[:, :pos + 2]), 64, s)
    np.testing.assert_allclose(out2.cpu().numpy(), ref2, atol=TOL, rtol=0)


def test_decode_step_cache_full(ctx):
    import torch
    from streaming_attention_b200 import SAError, attn_decode_step
    kc = torch.zeros(2, 8, 64, device="cuda")
    q = np.zeros((2, 64), np.float32)
    kn = np.zeros((2, 64), np.float32)
    with pytest.raises(SAError) as e:
        attn_decode_step(q, kn, kn, kc, kc.clone(), 8, 1.0, 64, ctx)
    assert e.value.code == -7 and "full" in str(e.value)


@pytest.mark.parametrize("dtype", ["float32", "bfloat16"])
def test_decode_kv_static_back_to_back(ctx, oracle, dtype):
    """SA_KV_STATIC: each call launches as a programmatic dependent of the
    kernel before it and streams K/V early; q is written by that kernel (a
    copy) right before every call, and every output must still be the
    oracle's for its own q -- the early start may not read q or reuse the
    split scratch before the previous kernel (here also the previous decode
    call) is done."""
    import torch
    from oracle.oracle import bf16_round
    from streaming_attention_b200 import attn_decode
    hq, hkv, T, d = 16, 8, 9001, 128
    _, k, v = I.gqa(hq, hkv, T, d, 31)
    qs = [I.gqa(hq, hkv, 1, d, 100 + i)[0] for i in range(6)]
    if dtype == "bfloat16":
        k, v, qs = bf16_round(k), bf16_round(v), [bf16_round(x) for x in qs]
    tdt = getattr(torch, dtype)
    kt, vt = torch.from_numpy(k).cuda().to(tdt), torch.from_numpy(v).cuda().to(tdt)
    qsrc = [torch.from_numpy(x).cuda().to(tdt) for x in qs]
    q = torch.empty_like(qsrc[0])
    outs = [torch.empty(hq, d, device="cuda") for _ in qs]
    torch.cuda.synchronize()
    for i in range(len(qs)):
        q.copy_(qsrc[i])                     # the kernel right before the call writes q
        attn_decode(q, kt, vt, 1 / np.sqrt(d), 64, ctx, outs[i], kv_static=True)
        attn_decode(q, kt, vt, 1 / np.sqrt(d), 64, ctx, kv_static=True)   # back to back, same scratch
    torch.cuda.synchronize()
    for i, x in enumerate(qs):
        ref = oracle.gqa_decode(x, k, v, 64, 1 / np.sqrt(d))
        assert np.abs(outs[i].cpu().numpy() - ref).max() < 1e-4
