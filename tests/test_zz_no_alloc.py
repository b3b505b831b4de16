"""The allocation-free decode entry point, sa_attn_decode_noalloc.

Some callers of this library cannot call cudaMalloc: serving runtimes that
reserve nearly all device memory for their own pools at start-up, and
latency-critical loops that cannot afford cudaMalloc's implicit device
synchronisation.  sa_attn_decode_noalloc serves them from a fixed-size static
device array instead of allocated scratch.  These tests call it through the C
ABI and check it against the oracle's GQA decode (oracle/sa_oracle.c, the
reference's streaming attention per head) on two calls in a row, on a side
stream, with T = 0 and with the output on a second GPU; that a third call
allocates no device memory; and that shapes needing more scratch than the
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


def _case(hq, hkv, T, d, seed, dtype, device="cuda"):
    """Seeded inputs as device tensors, and the same values as float32 numpy
    arrays for the oracle (bf16 inputs rounded once, so both see the same)."""
    import torch
    from oracle.oracle import bf16_round
    q, k, v = I.gqa(hq, hkv, T, d, seed)
    if dtype == "bfloat16":
        q, k, v = bf16_round(q), bf16_round(k), bf16_round(v)
    t = lambda x: torch.from_numpy(x).to(device).to(getattr(torch, dtype))
    return (t(q), t(k), t(v)), (q, k, v)


def test_noalloc_matches_oracle_on_consecutive_calls(oracle):
    import torch
    from streaming_attention_b200 import lib

    cases = [(16, 8, 20000, 128, 1, "float32"),    # the bench's GQA shape
             (4, 2, 3333, 64, 2, "bfloat16")]      # another shape reusing the same array
    for hq, hkv, T, d, seed, dtype in cases:
        (q, k, v), host = _case(hq, hkv, T, d, seed, dtype)
        s = 1.0 / np.sqrt(d)
        ref = oracle.gqa_decode(*host, 64, s)
        for _ in range(2):                          # two calls in a row share the array
            out = torch.full((hq, d), float("nan"), device="cuda")
            rc = _noalloc(q, k, v, s, out)
            assert rc == 0, lib().sa_last_error()
            torch.cuda.synchronize()
            got = out.cpu().numpy()
            assert np.isfinite(got).all()
            assert np.abs(got - ref).max() < TOL


def test_noalloc_side_stream_and_empty_sequence(oracle):
    """A caller's own non-default stream, and T = 0 (zeros, as the reference's
    serial path returns for an empty sequence)."""
    import torch
    from streaming_attention_b200 import lib
    (q, k, v), host = _case(16, 8, 7777, 128, 4, "float32")
    ref = oracle.gqa_decode(*host, 64, 0.125)
    side = torch.cuda.Stream()
    out = torch.full((16, 128), float("nan"), device="cuda")
    with torch.cuda.stream(side):
        assert _noalloc(q, k, v, 0.125, out) == 0, lib().sa_last_error()
    side.synchronize()
    assert np.abs(out.cpu().numpy() - ref).max() < TOL
    empty = torch.empty(8, 0, 128, device="cuda")
    out0 = torch.full((16, 128), float("nan"), device="cuda")
    assert _noalloc(q, empty, empty, 0.125, out0) == 0, lib().sa_last_error()
    torch.cuda.synchronize()
    assert (out0 == 0).all()


def test_noalloc_on_second_gpu(oracle):
    """Inputs and output on GPU 1 while GPU 0 is current: the call runs on the
    GPU that holds `out`, with that GPU's own copy of the array."""
    import torch
    from streaming_attention_b200 import lib
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    torch.cuda.set_device(0)
    (q, k, v), host = _case(16, 8, 9000, 128, 5, "float32", device="cuda:1")
    ref = oracle.gqa_decode(*host, 64, 0.125)
    out = torch.full((16, 128), float("nan"), device="cuda:1")
    stream = torch.cuda.current_stream(1)
    P = lambda t: C.c_void_p(t.data_ptr())
    for _ in range(2):
        rc = lib().sa_attn_decode_noalloc(C.c_void_p(stream.cuda_stream), 0, P(q), P(k), P(v), 9000 * 128, 9000,
                                          128, 16, 8, 64, 0.125, P(out))
        assert rc == 0, lib().sa_last_error()
        torch.cuda.synchronize(1)
        assert np.abs(out.cpu().numpy() - ref).max() < TOL
    assert torch.cuda.current_device() == 0


def test_noalloc_allocates_no_device_memory(oracle):
    import torch
    from streaming_attention_b200 import lib
    (q, k, v), host = _case(16, 8, 5000, 128, 3, "float32")
    ref = torch.from_numpy(oracle.gqa_decode(*host, 64, 0.125)).cuda()
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
