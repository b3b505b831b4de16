"""Attention entry points, mirroring the reference's operator interface.

``streaming_attention_cuda`` / ``naive_attention_cuda`` take the arguments of
``streaming_attention_serial`` / ``naive_attention_serial``
(attention/src/attention.h:27-44, 118-125): a query row, row-major K and V of
T x d, unscaled scores, and return the d-vector.  ``streaming_attention_mpi_cuda``
is ``streaming_attention_mpi_simple`` (attention.h:191-208) over
torch.distributed ranks, one GPU per rank.

Arrays may be numpy (host memory: the library copies them in and the result
out) or CUDA torch tensors (device memory: the call runs on torch's current
stream, asynchronously).
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from ._capi import SA_BF16, SA_F32, SA_HOST_PTRS, SA_KV_STATIC, Context, check, default_context, lib


def _is_torch(x) -> bool:
    return type(x).__module__.startswith("torch")


def _dtype_code(x) -> int:
    if _is_torch(x):
        import torch
        if x.dtype == torch.float32:
            return SA_F32
        if x.dtype == torch.bfloat16:
            return SA_BF16
        raise TypeError(f"unsupported dtype {x.dtype}")
    if x.dtype == np.float32:
        return SA_F32
    raise TypeError(f"host arrays must be float32 (got {x.dtype}); pass bf16 as torch tensors")


def _ctx_for(x, ctx: Context | None) -> Context:
    if ctx is not None:
        return ctx
    if _is_torch(x):
        return default_context(x.device.index or 0)
    return default_context(0)


def _bind_stream(ctx: Context, x) -> None:
    if _is_torch(x):
        import torch
        ctx.set_stream(torch.cuda.current_stream(x.device).cuda_stream)


def _ptr(x):
    if _is_torch(x):
        return C.c_void_p(x.data_ptr())
    return x.ctypes.data_as(C.c_void_p)


def _prep(x):
    if _is_torch(x):
        return x.contiguous()
    return np.ascontiguousarray(x)


def _out_like(x, shape):
    if _is_torch(x):
        import torch
        return torch.empty(shape, dtype=torch.float32, device=x.device)
    return np.empty(shape, np.float32)


def attn_decode(q, k, v, scale: float = 1.0, block: int = 64, ctx: Context | None = None,
                out=None, kv_static: bool = False):
    """GQA decode attention (sa_attn_decode).

    q [hq, d]; k, v [hkv, T, d] (same dtype: fp32, or bf16 torch tensors);
    returns out [hq, d] fp32.  ``scale`` multiplies the scores (1.0 reproduces
    the unscaled attention.h kernels; 1/sqrt(d) the Qwen3 attention).
    ``kv_static`` (device tensors): K and V are not written by a kernel still
    running, so the call may stream them while the previous kernel finishes
    (SA_KV_STATIC).
    """
    q, k, v = _prep(q), _prep(k), _prep(v)
    hq, d = q.shape
    hkv, T, d2 = k.shape
    assert d2 == d and tuple(v.shape) == tuple(k.shape)
    ctx = _ctx_for(q, ctx)
    dt = _dtype_code(q)
    flags = (SA_KV_STATIC if kv_static else 0) if _is_torch(q) else SA_HOST_PTRS
    if out is None:
        out = _out_like(q, (hq, d))
    _bind_stream(ctx, q)
    check(lib().sa_attn_decode(ctx.h, dt, _ptr(q), _ptr(k), _ptr(v), T * d, T, d, hq, hkv, block,
                               scale, _ptr(out), flags))
    return out


def attn_decode_partial(q, k, v, scale: float = 1.0, block: int = 64, ctx: Context | None = None):
    """Un-finalised state (m [hq], l [hq], o [hq, d]) of attn_decode (sa_attn_decode_partial)."""
    q, k, v = _prep(q), _prep(k), _prep(v)
    hq, d = q.shape
    hkv, T, _ = k.shape
    ctx = _ctx_for(q, ctx)
    flags = 0 if _is_torch(q) else SA_HOST_PTRS
    m, l, o = _out_like(q, (hq,)), _out_like(q, (hq,)), _out_like(q, (hq, d))
    _bind_stream(ctx, q)
    check(lib().sa_attn_decode_partial(ctx.h, _dtype_code(q), _ptr(q), _ptr(k), _ptr(v), T * d, T,
                                       d, hq, hkv, block, scale, _ptr(m), _ptr(l), _ptr(o), flags))
    return m, l, o


def attn_merge(m, l, o, ctx: Context | None = None, with_state: bool = False):
    """Merge part-major partials m, l [n, hq], o [n, hq, d] (sa_attn_merge)."""
    m, l, o = _prep(m), _prep(l), _prep(o)
    n, hq, d = o.shape
    ctx = _ctx_for(o, ctx)
    flags = 0 if _is_torch(o) else SA_HOST_PTRS
    out = _out_like(o, (hq, d))
    mo = _out_like(o, (hq,)) if with_state else None
    lo = _out_like(o, (hq,)) if with_state else None
    _bind_stream(ctx, o)
    check(lib().sa_attn_merge(ctx.h, n, hq, d, _ptr(m), _ptr(l), _ptr(o), _ptr(out),
                              _ptr(mo) if with_state else None, _ptr(lo) if with_state else None,
                              flags))
    return (out, mo, lo) if with_state else out


def attn_decode_step(q, k_new, v_new, k_cache, v_cache, pos: int, scale: float = 1.0,
                     block: int = 64, ctx: Context | None = None, out=None):
    """One decode step over a device KV cache (sa_attn_decode_step).

    k_cache, v_cache: CUDA torch tensors [hkv, max_seq, d]; the new token's
    k_new, v_new [hkv, d] are written at row ``pos`` and q [hq, d] attends over
    rows [0, pos].  q / k_new / v_new may be numpy (host; the call then copies
    them in, and returns the output on the host) or CUDA tensors.
    """
    hkv, max_seq, d = k_cache.shape
    hq = q.shape[0]
    host = not _is_torch(q)
    q, k_new, v_new = _prep(q), _prep(k_new), _prep(v_new)
    ctx = _ctx_for(k_cache, ctx)
    if out is None:
        out = np.empty((hq, d), np.float32) if host else _out_like(q, (hq, d))
    _bind_stream(ctx, k_cache)
    dt = _dtype_code(k_cache)
    check(lib().sa_attn_decode_step(ctx.h, dt, _ptr(q), _ptr(k_new), _ptr(v_new), _ptr(k_cache),
                                    _ptr(v_cache), max_seq, pos, d, hq, hkv, block, scale, _ptr(out),
                                    SA_HOST_PTRS if host else 0))
    return out


def attn_prefill(q, k, v, scale: float, q_pos0: int = 0, out_dtype: str = "float32",
                 ctx: Context | None = None, out=None):
    """Causal GQA prefill attention on tensor cores (sa_attn_prefill).

    q [Sq, hq, 128], k, v [Skv, hkv, 128]: bf16 CUDA tensors (token-major; any
    token stride).  Query i sits at position q_pos0 + i and sees keys
    0 .. q_pos0 + i.  Returns out [Sq, hq, 128] in ``out_dtype``.
    """
    import torch
    Sq, hq, d = q.shape
    Skv, hkv, _ = k.shape
    for t in (q, k, v):
        assert t.dtype == torch.bfloat16 and t.is_cuda and t.stride(2) == 1 and t.stride(1) == d
    odt = torch.float32 if out_dtype == "float32" else torch.bfloat16
    if out is None:
        out = torch.empty(Sq, hq, d, dtype=odt, device=q.device)
    ctx = _ctx_for(q, ctx)
    _bind_stream(ctx, q)
    check(lib().sa_attn_prefill(ctx.h, _ptr(q), _ptr(k), _ptr(v), Sq, Skv, q_pos0, d, hq, hkv,
                                q.stride(0), k.stride(0), scale, _ptr(out),
                                SA_F32 if odt == torch.float32 else SA_BF16, out.stride(0), 0))
    return out


def attn_prompt_f32(q, k, v, scale: float, q_pos0: int = 0, causal: bool = True, ctx: Context | None = None,
                    out=None):
    """fp32 attention of several query rows (sa_attn_prompt_f32).

    q [Sq, hq, d] token-major; k, v [hkv, Skv, d] head-major (one batch row
    of the reference's [B, H, S, D] tensors); fp32, numpy (host) or CUDA
    torch tensors.  causal: query i sees keys 0 .. min(q_pos0 + i, Skv - 1);
    else every key.  Returns out [Sq, hq, d] fp32.
    """
    q, k, v = _prep(q), _prep(k), _prep(v)
    Sq, hq, d = q.shape
    hkv, Skv, _ = k.shape
    ctx = _ctx_for(q, ctx)
    flags = 0 if _is_torch(q) else SA_HOST_PTRS
    if out is None:
        out = _out_like(q, (Sq, hq, d))
    _bind_stream(ctx, q)
    check(lib().sa_attn_prompt_f32(ctx.h, _ptr(q), _ptr(k), _ptr(v), Sq, Skv, q_pos0, 1 if causal else 0, d, hq,
                                   hkv, hq * d, Skv * d, scale, _ptr(out), hq * d, flags))
    return out


# ---- attention.h mirror ---------------------------------------------------

def streaming_attention_cuda(Q, K, V, T: int, d: int, block_size: int, ctx: Context | None = None):
    """streaming_attention_serial/_omp (attention.h:118-125, 159-167) on the GPU."""
    q = _prep(Q).reshape(1, d)
    k = _prep(K).reshape(1, T, d)
    v = _prep(V).reshape(1, T, d)
    return attn_decode(q, k, v, 1.0, block_size, ctx).reshape(d)


def naive_attention_cuda(Q, K, V, T: int, d: int, ctx: Context | None = None):
    """naive_attention_serial (attention.h:27-33): the same softmax(qK^T)V."""
    return streaming_attention_cuda(Q, K, V, T, d, 64, ctx)


def streaming_attention_mpi_cuda(Q_local, K_local, V_local, T_local: int, T_global: int, d: int,
                                 block_size: int, group=None, ctx: Context | None = None):
    """streaming_attention_mpi_simple (attention/src/streaming_mpi.cpp:252-309).

    One rank per GPU under torch.distributed; Q (meaningful on rank 0) and the
    rank's K/V slice are CUDA torch tensors.  Unscaled scores, as attention.h.
    Rank 0 returns the d-vector, the other ranks zeros.
    """
    from .sequence_parallel import sp_decode
    q = Q_local.reshape(1, d)
    if q.dtype != K_local.dtype:
        q = q.to(K_local.dtype)
    k = K_local.reshape(1, T_local, d)
    v = V_local.reshape(1, T_local, d)
    pf = lambda q_, k_, v_, s_, b_: attn_decode_partial(q_, k_, v_, s_, b_, ctx)
    mf = lambda m_, l_, o_: attn_merge(m_, l_, o_, ctx)
    return sp_decode(q, k, v, 1.0, block_size, group, pf, mf).reshape(d)
