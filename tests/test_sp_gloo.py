"""Sequence-parallel decode orchestration over world-size-2 gloo ranks on CPU.

The collective sequence of sp_decode (broadcast q from rank 0, per-rank
partial, all-gather, merge, rank-0 result) is the host logic of the multi-GPU
path; here the partial and merge steps are the CPU oracle, so the test needs no
GPU and checks that ranks are merged in sequence order into exactly the
unsharded attention.
"""
import os

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _worker(rank, world, port, T_cuts, result_path):
    import sys
    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    import _inputs as I
    from oracle.oracle import Oracle
    from streaming_attention_b200.sequence_parallel import sp_decode

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    O = Oracle()
    hq, hkv, d = 4, 2, 64
    T = T_cuts[-1]
    q, k, v = I.gqa(hq, hkv, T, d, 123)
    a, b = T_cuts[rank], T_cuts[rank + 1]
    scale = 1 / np.sqrt(d)

    def partial_fn(qt, kt, vt, s, blk):
        qn, kn, vn = qt.numpy(), kt.numpy(), vt.numpy()
        G = hq // hkv
        ms, ls, os_ = [], [], []
        for h in range(hq):
            m_, l_, o_ = O.partial(qn[h], kn[h // G], vn[h // G], 0, kn.shape[1], blk, s)
            ms.append(m_); ls.append(l_); os_.append(o_)
        return torch.tensor(ms), torch.tensor(ls), torch.tensor(np.stack(os_))

    def merge_fn(m, l, o):
        out = np.empty((hq, d), np.float32)
        for h in range(hq):
            parts = [(float(m[r, h]), float(l[r, h]), o[r, h].numpy()) for r in range(m.shape[0])]
            out[h] = O.merge(parts)[2]
        return torch.from_numpy(out)

    q_rank = torch.from_numpy(q) if rank == 0 else torch.zeros(hq, d)   # only rank 0 holds q
    out = sp_decode(q_rank, torch.from_numpy(np.ascontiguousarray(k[:, a:b])),
                    torch.from_numpy(np.ascontiguousarray(v[:, a:b])), scale, 64, None,
                    partial_fn, merge_fn)
    if rank == 0:
        np.save(result_path, out.numpy())
    else:
        assert not out.any()
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("cuts", [[0, 700, 1500], [0, 1, 1500], [0, 1499, 1500]])
def test_sp_decode_gloo_two_ranks(tmp_path, cuts):
    import _inputs as I
    from oracle.oracle import Oracle
    port = 29500 + (os.getpid() % 1000) + cuts[1] % 97
    res = str(tmp_path / "out.npy")
    mp.spawn(_worker, args=(2, port, cuts, res), nprocs=2, join=True)
    hq, hkv, d, T = 4, 2, 64, cuts[-1]
    q, k, v = I.gqa(hq, hkv, T, d, 123)
    ref = Oracle().gqa_decode(q, k, v, 64, 1 / np.sqrt(d))
    np.testing.assert_allclose(np.load(res), ref, atol=1e-5, rtol=0)
