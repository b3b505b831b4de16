"""Sequence-parallel Qwen3 (sa_qwen3_create_sp) over 2 and 4 GPUs, one process
per GPU, buffers connected through handles passed over a gloo group.

The reference's SEQUENCE strategy (qwen3_forward_mpi_omp,
tensor_cpp/src/qwen3_ops_mpi.cpp:498-642) splits the prompt's tokens over the
ranks; its outputs are wrong there, so the target is the single-GPU forward:
every rank must return the same logits and tokens, within the logits bar of
the single-GPU tests of the CPU oracle and with its greedy tokens, and every
rank's KV cache must hold the oracle's cache rows (the ranks exchange theirs
each layer).  Covered: a split prompt (cache-free, three times, so the third
replays the captured graph), a prompt too short to split (run whole on every
rank), a cached prompt continued by a second split chunk at an offset, and
greedy decode after a split prompt.  Skipped on boxes with too few GPUs."""
import os

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
pytestmark = pytest.mark.gpu

CFG = dict(vocab=1000, hidden=512, n_layers=3, hq=8, hkv=4, head_dim=128, inter=1536, eps=1e-6, theta=1e6)
SEED, PROMPT, CONT, N_NEW, MAX_SEQ = 23, 37, 50, 10, 256
REL = 2e-3


def _ids(seed, n):
    import _inputs as I
    return I.rng(seed).integers(0, CFG["vocab"], n)


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
    m = Qwen3(CFG, max_seq=MAX_SEQ, ctx=ctx, rank=rank, world=world, strategy="sequence")
    m.load(make_qwen3_weights(Qwen3Cfg(**CFG), SEED))
    m.connect()
    ids = _ids(11, PROMPT)
    res = {}
    runs = [m.forward(ids) for _ in range(3)]         # split prompt, cache-free; the third replays a graph
    res["logits"] = runs[0]
    res["replay_same"] = np.array(all(np.array_equal(r, runs[0]) for r in runs))
    res["short"] = m.forward(_ids(12, 3), logits="last")   # too short to split: whole on every rank
    res["tokens"] = m.generate(ids, N_NEW)            # split prompt + replicated graph-replayed decode
    res["cache_len"] = np.array(m.cache_len)
    m.reset()
    m.forward(ids, use_cache=True, logits="none")     # cached split prompt ...
    res["cont"] = m.forward(_ids(13, CONT), use_cache=True, logits="all")   # ... continued by a split chunk
    res["cont_len"] = np.array(m.cache_len)
    res["k0"], res["v0"] = m.read_kv(0)
    res["k2"], res["v2"] = m.read_kv(2)
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
def test_qwen3_sequence_parallel(tmp_path, oracle, world):
    import torch
    import torch.multiprocessing as mp
    from oracle.oracle import Qwen3Cfg, make_qwen3_weights
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    mp.spawn(_worker, args=(world, 29700 + world + os.getpid() % 100, str(tmp_path)), nprocs=world, join=True)
    res = [np.load(tmp_path / f"r{r}.npz") for r in range(world)]
    for r in range(world):
        assert bool(res[r]["replay_same"]), f"rank {r}: graph replay changed the logits"
    for r in range(1, world):     # identical results on every rank
        for key in ("logits", "short", "tokens", "cache_len", "cont", "cont_len"):
            np.testing.assert_array_equal(res[r][key], res[0][key], err_msg=f"rank {r} {key}")
    cfg = Qwen3Cfg(**CFG)
    w = make_qwen3_weights(cfg, SEED)
    ids = _ids(11, PROMPT)
    _close(res[0]["logits"], oracle.qwen3_forward(cfg, w, ids), "split prompt logits")
    _close(res[0]["short"][0], oracle.qwen3_forward(cfg, w, _ids(12, 3))[-1], "short prompt logits")
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
    # cached prompt + continuation chunk, and the whole cache on every rank
    kc2 = np.zeros_like(kc)
    vc2 = np.zeros_like(vc)
    oracle.qwen3_forward(cfg, w, ids, kc=kc2, vc=vc2, max_seq=MAX_SEQ, all_logits=False)
    ref_cont = oracle.qwen3_forward(cfg, w, _ids(13, CONT), kc=kc2, vc=vc2, max_seq=MAX_SEQ, pos0=PROMPT)
    _close(res[0]["cont"], ref_cont, "continuation logits")
    n = PROMPT + CONT
    assert int(res[0]["cont_len"]) == n
    for r in range(world):
        for layer, key in ((0, "0"), (2, "2")):
            assert res[r]["k" + key].shape == (hkv, n, D)
            _close(res[r]["k" + key], kc2[layer, :, :n], f"rank {r} layer {layer} K cache")
            _close(res[r]["v" + key], vc2[layer, :, :n], f"rank {r} layer {layer} V cache")


def test_qwen3_sp_rejects_two_ranks_on_one_gpu():
    """The ranks wait for one another, so they must be on different GPUs: a
    handle naming this rank's own GPU is refused (nothing runs)."""
    from streaming_attention_b200 import Context, Qwen3, SAError
    c0, c1 = Context(0), Context(0)
    a = Qwen3(CFG, max_seq=64, ctx=c0, rank=0, world=2, strategy="sequence")
    b = Qwen3(CFG, max_seq=64, ctx=c1, rank=1, world=2, strategy="sequence")
    with pytest.raises(SAError) as e:
        a.sp_connect([a.sp_handle(), b.sp_handle()])
    assert e.value.code == -1 and "this rank's GPU" in str(e.value)
    with pytest.raises(SAError):
        a.forward(_ids(1, 8))                     # not connected
    for x in (a, b):
        x.close()
    c0.close()
    c1.close()
