"""fp32 multi-query attention (sa_attn_prompt_f32), the GPU side of the
tensor_cpp operators ops::self_attention (no mask / causal mask,
tensor_cpp/src/ops.cpp:514-641) and self_attention_streaming_blockwise
(ops.cpp:1383-1450): causal rows on the prompt-attention kernel, full rows,
saturated rows and other head sizes on the decode kernel's multi-query launch.
Causal cases are checked against the oracle's block-wise causal attention
(oracle/sa_oracle.c), full ones against float64 numpy; fp32 bar 1e-4 max-abs."""
import numpy as np
import pytest

import _inputs as I

pytestmark = pytest.mark.gpu
TOL = 1e-4

CASES = [  # (Sq, Skv, q_pos0, causal, d, hq, hkv)
    (200, 200, 0, True, 128, 16, 8),      # prompt kernel, a whole prompt
    (77, 300, 223, True, 128, 8, 2),      # a query block after a cached prefix
    (300, 250, 0, True, 128, 4, 4),       # queries past the last key see every key (block-wise form)
    (130, 130, 0, True, 128, 32, 2),      # 16 query heads per KV head
    (5, 1000, 10, True, 256, 4, 2),       # head_dim 256: multi-query decode launch
    (129, 129, 0, True, 64, 8, 8),        # head_dim 64, causal
    (33, 500, 0, False, 64, 8, 2),        # no mask
    (1, 4097, 0, False, 128, 16, 8),      # one decode query
    (66000, 16, 0, False, 64, 1, 1),      # more queries than one launch's grid.z
]


def _full_ref(q, k, v, scale):
    Sq, hq, d = q.shape
    hkv = k.shape[0]
    G = hq // hkv
    kr = np.repeat(k, G, axis=0).astype(np.float64)
    vr = np.repeat(v, G, axis=0).astype(np.float64)
    s = np.einsum("ihd,htd->iht", q.astype(np.float64), kr) * scale
    p = np.exp(s - s.max(axis=2, keepdims=True))
    p /= p.sum(axis=2, keepdims=True)
    return np.einsum("iht,htd->ihd", p, vr)


@pytest.mark.parametrize("Sq,Skv,q_pos0,causal,d,hq,hkv", CASES)
def test_prompt_f32_vs_reference(ctx, oracle, Sq, Skv, q_pos0, causal, d, hq, hkv):
    import torch
    from streaming_attention_b200 import attn_prompt_f32
    g = I.rng(Sq * 7 + Skv)
    q = g.standard_normal((Sq, hq, d), dtype=np.float32)
    k = g.standard_normal((hkv, Skv, d), dtype=np.float32)
    v = g.standard_normal((hkv, Skv, d), dtype=np.float32)
    scale = 1.0 / np.sqrt(d)
    out = attn_prompt_f32(torch.from_numpy(q).cuda(), torch.from_numpy(k).cuda(), torch.from_numpy(v).cuda(),
                          scale, q_pos0, causal, ctx)
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    if causal:
        ref = oracle.causal_prefill(q, np.ascontiguousarray(k.transpose(1, 0, 2)),
                                    np.ascontiguousarray(v.transpose(1, 0, 2)), scale, q_pos0)
    else:
        ref = _full_ref(q, k, v, scale)
    assert np.abs(got - ref).max() < TOL


def test_prompt_f32_host_pointers_and_errors(ctx, oracle):
    """Host (numpy) buffers through SA_HOST_PTRS; argument errors."""
    from streaming_attention_b200 import SAError, attn_prompt_f32
    g = I.rng(3)
    q = g.standard_normal((50, 8, 128), dtype=np.float32)
    k = g.standard_normal((4, 90, 128), dtype=np.float32)
    v = g.standard_normal((4, 90, 128), dtype=np.float32)
    got = attn_prompt_f32(q, k, v, 0.1, 40, True, ctx)
    ref = oracle.causal_prefill(q, np.ascontiguousarray(k.transpose(1, 0, 2)),
                                np.ascontiguousarray(v.transpose(1, 0, 2)), 0.1, 40)
    assert np.abs(got - ref).max() < TOL
    with pytest.raises(SAError):
        attn_prompt_f32(q, k, v, 0.1, 90, True, ctx)          # query 0 would see no key
    with pytest.raises(SAError):
        attn_prompt_f32(q[:, :6], k[:4], v[:4], 0.1, 0, True, ctx)   # 6 query heads over 4 KV heads
