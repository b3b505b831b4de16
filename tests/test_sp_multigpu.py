"""Sequence parallelism across 2 GPUs (NCCL), through the C ABI on each rank.
Decode: the KV sequence is split over the ranks, partials are all-gathered and
merged on the device; rank 0's result must equal the unsharded attention.
Causal prefill: zig-zag query chunks, K/V all-gathered; the ranks' outputs in
sequence order must match the oracle's causal prefill (oracle/sa_oracle.c,
the reference's block-wise online softmax) on the same bf16-valued inputs
within the bf16 tensor-core bar (2e-2 of max |out|), and equal the
single-GPU prefill.  Skipped on boxes with fewer than 2 GPUs."""
import os

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
pytestmark = pytest.mark.gpu


def _worker(rank, world, port, res):
    import sys
    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    from datetime import timedelta
    import torch
    import torch.distributed as dist
    import _inputs as I
    import streaming_attention_b200 as sa
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    hq, hkv, d, T = 16, 8, 128, 20001
    q, k, v = I.gqa(hq, hkv, T, d, 9)
    cuts = np.linspace(0, T, world + 1).astype(int)
    a, b = cuts[rank], cuts[rank + 1]
    dev = torch.device("cuda", rank)
    kt = torch.from_numpy(np.ascontiguousarray(k[:, a:b])).to(dev)
    vt = torch.from_numpy(np.ascontiguousarray(v[:, a:b])).to(dev)
    qt = torch.from_numpy(q).to(dev) if rank == 0 else torch.zeros(hq, d, device=dev)
    ctx = sa.Context(rank)
    from streaming_attention_b200.sequence_parallel import sp_decode
    pf = lambda q_, k_, v_, s_, b_: sa.attn_decode_partial(q_, k_, v_, s_, b_, ctx)
    mf = lambda m_, l_, o_: sa.attn_merge(m_, l_, o_, ctx)
    out = sp_decode(qt, kt, vt, 1 / np.sqrt(d), 64, None, pf, mf)
    torch.cuda.synchronize(dev)
    if rank == 0:
        np.save(res, out.cpu().numpy())
    dist.barrier(device_ids=[rank])
    ctx.close()
    dist.destroy_process_group()


def test_sp_decode_two_gpus(tmp_path, oracle):
    import torch
    import torch.multiprocessing as mp
    import _inputs as I
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    res = str(tmp_path / "out.npy")
    mp.spawn(_worker, args=(2, 29600 + os.getpid() % 200, res), nprocs=2, join=True)
    q, k, v = I.gqa(16, 8, 20001, 128, 9)
    ref = oracle.gqa_decode(q, k, v, 64, 1 / np.sqrt(128))
    np.testing.assert_allclose(np.load(res), ref, atol=1e-4, rtol=0)


def _prefill_worker(rank, world, port, out_dir):
    import sys
    sys.path.insert(0, ROOT)
    from datetime import timedelta
    import torch
    import torch.distributed as dist
    import streaming_attention_b200 as sa
    from streaming_attention_b200.sequence_parallel import sp_prefill, zigzag_shard
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60), device_id=dev)
    S, hq, hkv, d = 2048, 16, 8, 128
    g = torch.Generator(device=dev).manual_seed(5)
    q = torch.randn(S, hq, d, device=dev, generator=g).to(torch.bfloat16)
    k = torch.randn(S, hkv, d, device=dev, generator=g).to(torch.bfloat16)
    v = torch.randn(S, hkv, d, device=dev, generator=g).to(torch.bfloat16)
    ctx = sa.Context(rank)
    pf = lambda q_, k_, v_, s_, p0, o_: sa.attn_prefill(q_, k_, v_, s_, p0, "float32", ctx, o_)
    streams = [torch.cuda.Stream(dev), torch.cuda.Stream(dev)]
    out = sp_prefill(zigzag_shard(q, rank, world), zigzag_shard(k, rank, world), zigzag_shard(v, rank, world),
                     1 / np.sqrt(d), None, pf, streams, torch.float32)
    torch.cuda.synchronize(dev)
    np.save(os.path.join(out_dir, f"r{rank}.npy"), out.cpu().numpy())
    if rank == 0:
        full = sa.attn_prefill(q, k, v, 1 / np.sqrt(d), 0, "float32", ctx)
        torch.cuda.synchronize(dev)
        np.save(os.path.join(out_dir, "full.npy"), full.cpu().numpy())
        for name, t in (("q", q), ("k", k), ("v", v)):      # the bf16 values, for the oracle
            np.save(os.path.join(out_dir, f"{name}.npy"), t.float().cpu().numpy())
    dist.barrier(device_ids=[rank])
    ctx.close()
    dist.destroy_process_group()


def test_sp_prefill_two_gpus(tmp_path, oracle):
    import torch
    import torch.multiprocessing as mp
    from streaming_attention_b200.sequence_parallel import zigzag_chunks
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    mp.spawn(_prefill_worker, args=(2, 29800 + os.getpid() % 200, str(tmp_path)), nprocs=2, join=True)
    full = np.load(tmp_path / "full.npy")
    got = np.empty_like(full)
    for r in range(2):
        part = np.load(tmp_path / f"r{r}.npy")
        (a0, a1), (b0, b1) = zigzag_chunks(r, 2, full.shape[0])
        got[a0:a1], got[b0:b1] = part[:a1 - a0], part[a1 - a0:]
    q, k, v = (np.load(tmp_path / f"{n}.npy") for n in ("q", "k", "v"))
    ref = oracle.causal_prefill(q, k, v, 1 / np.sqrt(q.shape[2]))
    assert np.abs(got - ref).max() <= 2e-2 * np.abs(ref).max()
    # the chunks start on 128-row tiles, so each query row sees the same tiles
    np.testing.assert_allclose(got, full, atol=1e-6, rtol=0)
