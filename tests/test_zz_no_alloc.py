"""The allocation-free decode entry point, sa_attn_decode_noalloc.

Some callers of this library cannot call cudaMalloc: serving runtimes that
reserve nearly all device memory for their own pools at start-up, and
latency-critical loops that cannot afford cudaMalloc's implicit device
synchronisation.  sa_attn_decode_noalloc serves them from a fixed-size static
device array instead of allocated scratch.  These tests call it through the C
ABI and check it against sa_attn_decode on two calls in a row, that a third
call allocates no device memory, and that shapes needing more scratch than the
array holds are rejected.

The file name makes pytest collect it last, so a failure here does not keep
a run that stops at the first failure from running the other tests.
"""
import ctypes as C

import numpy as np
import pytest

import _inputs as I

pytestmark = pytest.mark.gpu
TOL = 1e-4   # the fp32 decode tolerance used by tests/test_decode_gpu.py


def _noalloc(q, k, v, scale, out):
    import torch
    from streaming_attention_b200 import SA_BF16, SA_F32, lib
    hq, d = q.shape
    hkv, T, _ = k.shape
    dt = SA_F32 if q.dtype == torch.float32 else SA_BF16
    P = lambda t: C.c_void_p(t.data_ptr())
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    return lib().sa_attn_decode_noalloc(stream, dt, P(q), P(k), P(v), T * d, T, d, hq, hkv, 64,
                                        scale, P(out))


def _case(hq, hkv, T, d, seed, dtype):
    import torch
    q, k, v = I.gqa(hq, hkv, T, d, seed)
    t = lambda x: torch.from_numpy(x).cuda().to(getattr(torch, dtype))
    return t(q), t(k), t(v)


def test_noalloc_matches_decode_on_consecutive_calls(ctx):
    import torch
    from streaming_attention_b200 import attn_decode, lib

    cases = [(16, 8, 20000, 128, 1, "float32"),    # the bench's GQA shape
             (4, 2, 3333, 64, 2, "bfloat16")]      # another shape reusing the same array
    for hq, hkv, T, d, seed, dtype in cases:
        q, k, v = _case(hq, hkv, T, d, seed, dtype)
        s = 1.0 / np.sqrt(d)
        ref = attn_decode(q, k, v, s, 64, ctx)
        out = torch.full((hq, d), float("nan"), device="cuda")
        rc = _noalloc(q, k, v, s, out)
        assert rc == 0, lib().sa_last_error()
        torch.cuda.synchronize()
        assert torch.isfinite(out).all()
        assert (out - ref).abs().max().item() < TOL


def test_noalloc_allocates_no_device_memory(ctx):
    import torch
    from streaming_attention_b200 import attn_decode, lib
    q, k, v = _case(16, 8, 5000, 128, 3, "float32")
    ref = attn_decode(q, k, v, 0.125, 64, ctx)
    out = torch.empty(16, 128, device="cuda")
    assert _noalloc(q, k, v, 0.125, out) == 0, lib().sa_last_error()   # set-up call
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    for _ in range(3):
        assert _noalloc(q, k, v, 0.125, out) == 0
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0
    assert (out - ref).abs().max().item() < TOL


def test_noalloc_rejects_shapes_beyond_static_scratch():
    import torch
    from streaming_attention_b200 import lib
    hq, hkv, T, d = 4096, 1024, 16, 128     # 4096 heads x (128 + 2) floats > 2 MiB
    q = torch.zeros(hq, d, device="cuda")
    k = torch.zeros(hkv, T, d, device="cuda")
    out = torch.empty(hq, d, device="cuda")
    assert _noalloc(q, k, k, 1.0, out) == -1
    assert b"static maximum" in lib().sa_last_error()
