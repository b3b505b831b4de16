"""Fused sequence-parallel decode (sa_sp_* / sa_attn_decode_sp): the KV
sequence split over GPUs as streaming_attention_mpi_simple splits it over MPI
ranks (attention/src/streaming_mpi.cpp:252-309), one launch per rank that
exchanges the (m, l, O) states over NVLink and merges them.  Every rank's
output is checked against the oracle's unsharded GQA decode at the fp32
tolerance (1e-4 max-abs), over consecutive calls (the exchange slots
alternate), uneven and empty slices, bf16 K/V and the merged (m, l) state.
The argument checks (one GPU per rank) run on one GPU; the exchange itself
needs 2 or 4."""
import os

import numpy as np
import pytest

import _inputs as I

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
pytestmark = pytest.mark.gpu
TOL = 1e-4

# (hq, hkv, T, d, dtype, seed, how the sequence is cut over the ranks)
CASES = [
    (16, 8, 20001, 128, "float32", 11, None),       # configs[1] heads, uneven slices
    (16, 8, 4099, 128, "float32", 12, "first"),     # every row on rank 0, the rest empty
    (4, 2, 3001, 256, "bfloat16", 13, None),
    (8, 8, 777, 64, "float32", 14, None),
    (16, 8, 65536, 128, "float32", 15, None),
]


def _cuts(T, world, mode):
    if mode == "first":
        return [0] + [T] * world
    return [int(x) for x in np.linspace(0, T, world + 1)]


def _inputs(hq, hkv, T, d, dtype, seed):
    from oracle.oracle import bf16_round
    q, k, v = I.gqa(hq, hkv, T, d, seed)
    if dtype == "bfloat16":
        q, k, v = bf16_round(q), bf16_round(k), bf16_round(v)
    return q, k, v


def _state_ref(q, k, scale):
    """Merged (m, l) of the whole sequence in float64: m = max score, l = sum exp(score - m)."""
    hq, d = q.shape
    hkv = k.shape[0]
    G = hq // hkv
    s = np.einsum("hd,htd->ht", q.astype(np.float64), np.repeat(k, G, axis=0).astype(np.float64)) * scale
    m = s.max(axis=1)
    return m, np.exp(s - m[:, None]).sum(axis=1)


def _worker(rank, world, port, out_dir):
    import sys
    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    from datetime import timedelta
    import torch
    import torch.distributed as dist
    import streaming_attention_b200 as sa
    from streaming_attention_b200.sequence_parallel import SpDecoder
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    # gloo only carries the exchange-buffer handles and a barrier
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    ctx = sa.Context(rank)
    sp = SpDecoder(ctx, rank, world, max_hq=16, max_d=256)
    sp.connect_dist()
    for ci, (hq, hkv, T, d, dtype, seed, mode) in enumerate(CASES):
        q, k, v = _inputs(hq, hkv, T, d, dtype, seed)
        c = _cuts(T, world, mode)
        tdt = getattr(torch, dtype)
        qt = torch.from_numpy(q).to(dev).to(tdt)
        kt = torch.from_numpy(np.ascontiguousarray(k[:, c[rank]:c[rank + 1]])).to(dev).to(tdt)
        vt = torch.from_numpy(np.ascontiguousarray(v[:, c[rank]:c[rank + 1]])).to(dev).to(tdt)
        # two calls in a row on the same inputs, then the state-returning form
        a = sp.decode(qt, kt, vt, 1 / np.sqrt(d), 64)
        b = sp.decode(qt, kt, vt, 1 / np.sqrt(d), 64)
        o, m, l = sp.decode(qt, kt, vt, 1 / np.sqrt(d), 64, with_state=True)
        # SA_KV_STATIC: launched as a programmatic dependent of the copy that
        # writes q, then of the previous decode (same scratch, next exchange slot)
        q2 = torch.empty_like(qt)
        q2.copy_(qt)
        e = sp.decode(q2, kt, vt, 1 / np.sqrt(d), 64, kv_static=True)
        f = sp.decode(q2, kt, vt, 1 / np.sqrt(d), 64, kv_static=True)
        ctx.synchronize()
        np.savez(os.path.join(out_dir, f"r{rank}_c{ci}.npz"), a=a.cpu().numpy(), b=b.cpu().numpy(),
                 o=o.cpu().numpy(), m=m.cpu().numpy(), l=l.cpu().numpy(), e=e.cpu().numpy(),
                 f=f.cpu().numpy())
    dist.barrier()
    sp.close()
    ctx.close()
    dist.destroy_process_group()


def _check(out_dir, world, oracle):
    for ci, (hq, hkv, T, d, dtype, seed, mode) in enumerate(CASES):
        q, k, v = _inputs(hq, hkv, T, d, dtype, seed)
        ref = oracle.gqa_decode(q, k, v, 64, 1 / np.sqrt(d))
        m_ref, l_ref = _state_ref(q, k, 1 / np.sqrt(d))
        first = None
        for r in range(world):
            z = np.load(os.path.join(out_dir, f"r{r}_c{ci}.npz"))
            for key in ("a", "b", "o", "e", "f"):
                err = np.abs(z[key] - ref).max()
                assert err < TOL, (ci, r, key, err)
            for key in ("b", "o", "e", "f"):
                assert np.array_equal(z["a"], z[key]), key
            np.testing.assert_allclose(z["m"], m_ref, rtol=1e-5, atol=1e-5)
            np.testing.assert_allclose(z["l"], l_ref, rtol=1e-4)
            if first is None:
                first = z["o"]
            assert np.array_equal(z["o"], first), "ranks disagree"   # same merge order everywhere


@pytest.mark.parametrize("world", [2, 4])
def test_sp_fused_decode_matches_oracle(tmp_path, oracle, world):
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    mp.spawn(_worker, args=(world, 29400 + world * 40 + os.getpid() % 40, str(tmp_path)), nprocs=world,
             join=True)
    _check(str(tmp_path), world, oracle)


def test_sp_fused_decode_one_process_two_gpus(oracle):
    """sa_sp_connect_local: both ranks in this process (peer pointers instead
    of IPC mappings), launched one after the other from one thread."""
    import torch
    import streaming_attention_b200 as sa
    from streaming_attention_b200.sequence_parallel import SpDecoder
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    ctxs = [sa.Context(i) for i in range(2)]
    sps = [SpDecoder(ctxs[i], i, 2, max_hq=16, max_d=128) for i in range(2)]
    SpDecoder.connect_local(sps)
    hq, hkv, T, d = 16, 8, 12345, 128
    q, k, v = I.gqa(hq, hkv, T, d, 21)
    ref = oracle.gqa_decode(q, k, v, 64, 1 / np.sqrt(d))
    c = _cuts(T, 2, None)
    ins = []
    for i in range(2):
        dev = torch.device("cuda", i)
        ins.append((torch.from_numpy(q).to(dev), torch.from_numpy(np.ascontiguousarray(k[:, c[i]:c[i + 1]])).to(dev),
                    torch.from_numpy(np.ascontiguousarray(v[:, c[i]:c[i + 1]])).to(dev)))
    for _ in range(3):
        outs = []
        for i in range(2):
            with torch.cuda.device(i):
                outs.append(sps[i].decode(*ins[i], 1 / np.sqrt(d), 64))
        for i in range(2):
            ctxs[i].synchronize()
            assert np.abs(outs[i].cpu().numpy() - ref).max() < TOL
    for s in sps:
        s.close()
    for cx in ctxs:
        cx.close()


def test_sp_rejects_two_ranks_on_one_gpu():
    """The ranks' launches wait for one another, so they must run on different
    GPUs: both connection paths refuse two ranks on one GPU (nothing runs)."""
    import ctypes as C
    import torch
    import streaming_attention_b200 as sa
    from streaming_attention_b200 import SAError, lib
    from streaming_attention_b200.sequence_parallel import SpDecoder
    c0, c1 = sa.Context(0), sa.Context(0)
    a, b = SpDecoder(c0, 0, 2), SpDecoder(c1, 1, 2)
    with pytest.raises(SAError) as e:
        SpDecoder.connect_local([a, b])
    assert e.value.code == -1 and "share GPU" in str(e.value)
    with pytest.raises(SAError) as e:
        a.connect([a.handle(), b.handle()])
    assert e.value.code == -1 and "this rank's GPU" in str(e.value)
    # an unconnected rank refuses to launch
    q = torch.zeros(16, 128, device="cuda")
    out = torch.empty(16, 128, device="cuda")
    rc = lib().sa_attn_decode_sp(a.h, 0, C.c_void_p(q.data_ptr()), None, None, 0, 0, 128, 16, 8, 64, 1.0,
                                 C.c_void_p(out.data_ptr()), None, None, 0)
    assert rc == -1 and b"not connected" in lib().sa_last_error()
    # handles that are not sa_sp handles, or name the wrong rank
    with pytest.raises(SAError):
        a.connect([b"\0" * 128, b.handle()])
    with pytest.raises(SAError):
        a.connect([b.handle(), a.handle()])
    for x in (a, b):
        x.close()
    c0.close()
    c1.close()
