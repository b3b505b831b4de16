"""Sequence-parallel causal prefill (zig-zag chunks) over gloo ranks on CPU.

sp_prefill's host logic -- which query chunks a rank owns, the all-gather of
K and V, their reassembly in sequence order, the global query offset and key
extent of each chunk -- with the oracle's causal prefill standing in for the
GPU kernel, so the test needs no GPU.  The ranks' outputs, put back in
sequence order, must equal the unsharded causal prefill.
"""
import os

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
S, HQ, HKV, D = 256, 4, 2, 128


def _worker(rank, world, port, out_dir):
    import sys
    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    import _inputs as I
    from oracle.oracle import Oracle
    from streaming_attention_b200.sequence_parallel import sp_prefill, zigzag_shard

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    O = Oracle()
    q, k, v = (torch.from_numpy(x) for x in I.prefill(S, HQ, HKV, D, 77))
    scale = 1 / np.sqrt(D)

    def prefill_fn(qc, kc, vc, s, q_pos0, out):
        assert kc.shape[0] == q_pos0 + qc.shape[0]          # keys end at the chunk's last query
        out.copy_(torch.from_numpy(O.causal_prefill(qc.numpy(), kc.numpy(), vc.numpy(), s,
                                                    q_pos0=q_pos0)))

    out = sp_prefill(zigzag_shard(q, rank, world), zigzag_shard(k, rank, world),
                     zigzag_shard(v, rank, world), scale, None, prefill_fn)
    np.save(os.path.join(out_dir, f"r{rank}.npy"), out.numpy())
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [1, 2, 4])
def test_sp_prefill_zigzag_gloo(tmp_path, world):
    import _inputs as I
    from oracle.oracle import Oracle
    from streaming_attention_b200.sequence_parallel import zigzag_chunks
    port = 29700 + (os.getpid() % 500) + world
    mp.spawn(_worker, args=(world, port, str(tmp_path)), nprocs=world, join=True)
    q, k, v = I.prefill(S, HQ, HKV, D, 77)
    ref = Oracle().causal_prefill(q, k, v, 1 / np.sqrt(D))
    got = np.empty_like(ref)
    for r in range(world):
        part = np.load(tmp_path / f"r{r}.npy")
        (a0, a1), (b0, b1) = zigzag_chunks(r, world, S)
        got[a0:a1], got[b0:b1] = part[:a1 - a0], part[a1 - a0:]
    np.testing.assert_allclose(got, ref, atol=1e-5, rtol=0)


def test_zigzag_balances_causal_work():
    from streaming_attention_b200.sequence_parallel import zigzag_chunks
    for world in (2, 4, 8):
        work = []
        for r in range(world):
            # causal key-query pairs of the rank's queries
            work.append(sum((q + 1) for a, b in zigzag_chunks(r, world, 8192) for q in range(a, b)))
        assert max(work) - min(work) <= 0.001 * max(work)
    with pytest.raises(ValueError):
        zigzag_chunks(0, 3, 100)
