"""Sequence-parallel causal prefill (sa_spp_* / SpPrefill): zig-zag chunks,
K/V stored by each rank straight into every rank's buffer over NVLink, one
tensor-core launch over a table of key-block pieces per rank, pieces merged
by their log-sum-exp.

The target is the oracle's causal prefill (oracle/sa_oracle.c, the
reference's block-wise online softmax, ops.cpp:1027-1112) on the same
bf16-valued inputs, within the bf16 tensor-core bar (2e-2 of max |out|);
the pieces' merge is also checked against the single-launch prefill of the
whole sequence (same kernel, different key blocking, bf16 piece outputs) at
5e-3.  World 1 runs on one GPU (the piece table and the merge); 2 and 4
ranks need that many."""
import os

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
pytestmark = pytest.mark.gpu
BAR = 2e-2


def _inputs(S, hq, hkv, seed):
    import torch
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(S, hq, 128, generator=g).to(torch.bfloat16)
    k = torch.randn(S, hkv, 128, generator=g).to(torch.bfloat16)
    v = torch.randn(S, hkv, 128, generator=g).to(torch.bfloat16)
    return q, k, v


def _ref(oracle, q, k, v):
    return oracle.causal_prefill(q.float().numpy(), k.float().numpy(), v.float().numpy(), 1 / np.sqrt(128))


def _assemble(parts, world, S):
    from streaming_attention_b200.sequence_parallel import zigzag_chunks
    out = np.empty((S,) + parts[0].shape[1:], np.float32)
    for r in range(world):
        (a0, a1), (b0, b1) = zigzag_chunks(r, world, S)
        out[a0:a1], out[b0:b1] = parts[r][:a1 - a0], parts[r][a1 - a0:]
    return out


@pytest.mark.parametrize("S,hq,hkv", [(2048, 16, 8), (1400, 16, 8), (1024, 8, 8), (1536, 12, 4)])
def test_spp_one_gpu(ctx, oracle, S, hq, hkv):
    """World 1: chunks 0 and 1 of C = S / 2 rows; three pieces (the first
    chunk's diagonal, the second chunk's unmasked block and diagonal), also
    with chunks that are not whole 128-row tiles (C = 700) and odd GQA
    groups.  Three calls in a row (the buffer slots alternate) agree."""
    import torch
    import streaming_attention_b200 as sa
    from streaming_attention_b200.sequence_parallel import SpPrefill, zigzag_shard
    q, k, v = _inputs(S, hq, hkv, S + hq)
    dev = torch.device("cuda", 0)
    sp = SpPrefill(ctx, 0, 1, max_seq=S, hkv=hkv)
    ql, kl, vl = (zigzag_shard(t, 0, 1).to(dev) for t in (q, k, v))
    outs = [sp.prefill(ql, kl, vl, 1 / np.sqrt(128), out_dtype=torch.float32) for _ in range(3)]
    full = sa.attn_prefill(q.to(dev), k.to(dev), v.to(dev), 1 / np.sqrt(128), 0, "float32", ctx)
    ctx.synchronize()
    got = _assemble([outs[0].cpu().numpy()], 1, S)
    for o in outs[1:]:
        assert torch.equal(o, outs[0])
    ref = _ref(oracle, q, k, v)
    scale = np.abs(ref).max()
    assert np.abs(got - ref).max() <= BAR * scale
    # the pieces' outputs are bf16: one bf16 rounding (2^-8 relative) apart
    assert np.abs(got - full.cpu().numpy()).max() <= 5e-3 * scale
    # bf16 output: the fp32 result rounded
    ob = sp.prefill(ql, kl, vl, 1 / np.sqrt(128))
    ctx.synchronize()
    assert ob.dtype == torch.bfloat16
    assert np.abs(ob.float().cpu().numpy() - outs[0].cpu().numpy()).max() <= 1e-2 * scale
    sp.close()


def _worker(rank, world, port, out_dir, S):
    import sys
    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    from datetime import timedelta
    import torch
    import torch.distributed as dist
    import streaming_attention_b200 as sa
    from streaming_attention_b200.sequence_parallel import SpPrefill, zigzag_shard
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    # gloo only carries the buffer handles and a barrier
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    ctx = sa.Context(rank)
    q, k, v = _inputs(S, 16, 8, 77)
    sp = SpPrefill(ctx, rank, world, max_seq=S, hkv=8)
    sp.connect_dist()
    ql, kl, vl = (zigzag_shard(t, rank, world).to(dev) for t in (q, k, v))
    a = sp.prefill(ql, kl, vl, 1 / np.sqrt(128), out_dtype=torch.float32)
    b = sp.prefill(ql, kl, vl, 1 / np.sqrt(128), out_dtype=torch.float32)   # the other slot
    ctx.synchronize()
    np.save(os.path.join(out_dir, f"r{rank}.npy"), a.cpu().numpy())
    np.save(os.path.join(out_dir, f"r{rank}b.npy"), b.cpu().numpy())
    dist.barrier()
    sp.close()
    ctx.close()
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_spp_multi_gpu(tmp_path, oracle, world):
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    S = 4096
    mp.spawn(_worker, args=(world, 29900 + world * 10 + os.getpid() % 50, str(tmp_path), S), nprocs=world,
             join=True)
    parts = [np.load(tmp_path / f"r{r}.npy") for r in range(world)]
    for r in range(world):
        np.testing.assert_array_equal(np.load(tmp_path / f"r{r}b.npy"), parts[r])
    got = _assemble(parts, world, S)
    q, k, v = _inputs(S, 16, 8, 77)
    ref = _ref(oracle, q, k, v)
    assert np.abs(got - ref).max() <= BAR * np.abs(ref).max()


def test_spp_one_process_two_gpus(oracle):
    """sa_spp_connect_local: both ranks in this process (peer pointers),
    launched one after the other from one thread."""
    import torch
    import streaming_attention_b200 as sa
    from streaming_attention_b200.sequence_parallel import SpPrefill, zigzag_shard
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    S = 2048
    q, k, v = _inputs(S, 16, 8, 78)
    ctxs = [sa.Context(i) for i in range(2)]
    sps = [SpPrefill(ctxs[i], i, 2, max_seq=S, hkv=8) for i in range(2)]
    SpPrefill.connect_local(sps)
    ins = [[zigzag_shard(t, i, 2).to(torch.device("cuda", i)) for t in (q, k, v)] for i in range(2)]
    outs = []
    for i in range(2):
        with torch.cuda.device(i):
            outs.append(sps[i].prefill(*ins[i], 1 / np.sqrt(128), out_dtype=torch.float32))
    for c in ctxs:
        c.synchronize()
    got = _assemble([o.cpu().numpy() for o in outs], 2, S)
    ref = _ref(oracle, q, k, v)
    assert np.abs(got - ref).max() <= BAR * np.abs(ref).max()
    for s in sps:
        s.close()
    for c in ctxs:
        c.close()


def test_spp_rejects_bad_use():
    """Two ranks on one GPU are refused by both connection paths, an
    unconnected rank refuses to run, and S must split into 2 x world chunks
    within max_seq (nothing runs)."""
    import torch
    import streaming_attention_b200 as sa
    from streaming_attention_b200 import SAError
    from streaming_attention_b200.sequence_parallel import SpPrefill
    c0, c1 = sa.Context(0), sa.Context(0)
    a, b = SpPrefill(c0, 0, 2, max_seq=1024, hkv=8), SpPrefill(c1, 1, 2, max_seq=1024, hkv=8)
    with pytest.raises(SAError) as e:
        SpPrefill.connect_local([a, b])
    assert e.value.code == -1 and "share GPU" in str(e.value)
    with pytest.raises(SAError) as e:
        a.connect([a.handle(), b.handle()])
    assert e.value.code == -1 and "this rank's GPU" in str(e.value)
    q = torch.zeros(512, 16, 128, dtype=torch.bfloat16, device="cuda")
    kv = torch.zeros(512, 8, 128, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(SAError) as e:
        a.prefill(q, kv, kv, 1.0)
    assert "not connected" in str(e.value)
    one = SpPrefill(c0, 0, 1, max_seq=1024, hkv=8)
    with pytest.raises(SAError):                     # S = 2 x 600 > max_seq
        one.prefill(torch.zeros(1200, 16, 128, dtype=torch.bfloat16, device="cuda"),
                    torch.zeros(1200, 8, 128, dtype=torch.bfloat16, device="cuda"),
                    torch.zeros(1200, 8, 128, dtype=torch.bfloat16, device="cuda"), 1.0)
    with pytest.raises(SAError):                     # created for hkv = 8
        one.prefill(q, q, q, 1.0)
    for x in (a, b, one):
        x.close()
    c0.close()
    c1.close()
