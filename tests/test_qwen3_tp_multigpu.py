"""Head-parallel Qwen3 (sa_qwen3_create_tp) over 2 and 4 GPUs, one process per
GPU, exchange buffers connected through handles passed over a gloo group.

Every rank must return the same logits and tokens; those must match the CPU
oracle within the logits bar of the single-GPU tests (the ranks sum the
o_proj / down_proj partial products in a different order than one GPU does)
and reproduce its greedy tokens; each rank's KV cache must hold the oracle's
cache rows of its own KV heads.  Skipped on boxes with too few GPUs."""
import os

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
pytestmark = pytest.mark.gpu

CFG = dict(vocab=1000, hidden=512, n_layers=3, hq=8, hkv=4, head_dim=128, inter=1536, eps=1e-6, theta=1e6)
SEED, PROMPT, N_NEW, STEPS, MAX_SEQ = 17, 37, 12, 4, 256
REL = 2e-3


def _prompt():
    import _inputs as I
    return I.rng(11).integers(0, CFG["vocab"], PROMPT)


def _worker(rank, world, port, out_dir):
    import sys
    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    from datetime import timedelta
    import torch.distributed as dist
    from oracle.oracle import Qwen3Cfg, make_qwen3_weights
    from streaming_attention_b200 import Context, Qwen3
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=120))
    ctx = Context(rank)
    m = Qwen3(CFG, max_seq=MAX_SEQ, ctx=ctx, rank=rank, world=world)
    m.load(make_qwen3_weights(Qwen3Cfg(**CFG), SEED))
    m.connect()
    ids = _prompt()
    res = {"logits": m.forward(ids)}                  # cache-free, every position
    res["tokens"] = m.generate(ids, N_NEW)            # prompt + graph-replayed decode steps
    res["cache_len"] = np.array(m.cache_len)
    m.reset()
    lg = m.forward(ids, use_cache=True, logits="last")
    steps, nxt = [], int(np.argmax(lg[0]))
    for _ in range(STEPS):                            # single-token forwards with logits
        lg = m.forward(np.array([nxt]), use_cache=True, logits="last")
        steps.append(lg[0])
        nxt = int(np.argmax(lg[0]))
    res["steps"] = np.stack(steps)
    res["k0"], res["v0"] = m.read_kv(0)
    np.savez(os.path.join(out_dir, f"r{rank}.npz"), **res)
    dist.barrier()
    m.close()
    ctx.close()
    dist.destroy_process_group()


def _close(got, ref, what):
    err = float(np.abs(got - ref).max())
    scale = float(np.abs(ref).max())
    assert err <= REL * max(scale, 1e-3), f"{what}: max|err| {err:.3e} vs max|ref| {scale:.3e}"


@pytest.mark.parametrize("world", [2, 4])
def test_qwen3_head_parallel(tmp_path, oracle, world):
    import torch
    import torch.multiprocessing as mp
    from oracle.oracle import Qwen3Cfg, make_qwen3_weights
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    mp.spawn(_worker, args=(world, 29400 + world + os.getpid() % 100, str(tmp_path)), nprocs=world, join=True)
    res = [np.load(tmp_path / f"r{r}.npz") for r in range(world)]
    for r in range(1, world):     # identical results on every rank
        for key in ("logits", "tokens", "steps", "cache_len"):
            np.testing.assert_array_equal(res[r][key], res[0][key], err_msg=f"rank {r} {key}")
    cfg = Qwen3Cfg(**CFG)
    w = make_qwen3_weights(cfg, SEED)
    ids = _prompt()
    _close(res[0]["logits"], oracle.qwen3_forward(cfg, w, ids), "prompt logits")
    # greedy decode through the oracle's KV cache
    L, hkv, D = CFG["n_layers"], CFG["hkv"], CFG["head_dim"]
    kc = np.zeros((L, hkv, MAX_SEQ, D), np.float32)
    vc = np.zeros_like(kc)
    lg = oracle.qwen3_forward(cfg, w, ids, kc=kc, vc=vc, max_seq=MAX_SEQ, all_logits=False)
    toks, pos = [int(np.argmax(lg[0]))], PROMPT
    for _ in range(N_NEW - 1):
        lg = oracle.qwen3_forward(cfg, w, np.array(toks[-1:]), kc=kc, vc=vc, max_seq=MAX_SEQ, pos0=pos,
                                  all_logits=False)
        pos += 1
        toks.append(int(np.argmax(lg[0])))
    assert [int(t) for t in res[0]["tokens"]] == toks
    assert int(res[0]["cache_len"]) == PROMPT + N_NEW - 1
    # the single-token forwards' logits follow the same tokens (first STEPS of them)
    for s in range(STEPS):
        assert int(np.argmax(res[0]["steps"][s])) == toks[s + 1]
    # rank r holds KV heads [r * hkv / world, (r + 1) * hkv / world) of the cache;
    # its length after the step-by-step run is PROMPT + STEPS
    hl, n = hkv // world, PROMPT + STEPS
    kc2 = np.zeros_like(kc)
    vc2 = np.zeros_like(vc)
    seq = list(ids) + toks[:STEPS]
    oracle.qwen3_forward(cfg, w, np.array(seq), kc=kc2, vc=vc2, max_seq=MAX_SEQ, all_logits=False)
    for r in range(world):
        assert res[r]["k0"].shape == (hl, n, D)
        _close(res[r]["k0"], kc2[0, r * hl:(r + 1) * hl, :n], f"rank {r} K cache")
        _close(res[r]["v0"], vc2[0, r * hl:(r + 1) * hl, :n], f"rank {r} V cache")
