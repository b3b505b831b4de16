"""The C++ host layer on a GPU: the command-line drivers (the reference test
drivers' arguments and "Time: <ms>" line) and the side-by-side check of the
reference's own C++ API against this repository's CUDA method
(oracle/_ref/cuda_method_check, built where the reference tree exists)."""
import os
import re
import subprocess

import pytest

from conftest import ROOT

pytestmark = pytest.mark.gpu
BIN = os.path.join(ROOT, "streaming_attention_b200", "bin")
CHECK = os.path.join(ROOT, "oracle", "_ref", "cuda_method_check")


def _run(args, timeout=300):
    r = subprocess.run(args, capture_output=True, text=True, timeout=timeout)
    assert r.returncode == 0, r.stdout + r.stderr
    return r.stdout


def _time_ms(out):
    m = re.search(r"^Time: (\S+) ms", out, flags=re.M)
    assert m, out
    assert float(out.split("Time:")[1].split()[0]) == float(m.group(1))   # 2nd token = ms
    return float(m.group(1))


def _err(out):
    return float(re.search(r"Max error vs fp64 softmax: (\S+)", out).group(1))


@pytest.mark.parametrize("args", [
    ["test_streaming_cuda", "8192", "128", "64"],
    ["test_streaming_cuda", "1000", "64", "128"],
    ["test_naive_cuda", "8192", "128"],
    ["test_streaming_cuda_multi", "8192", "128", "64", "1"],
    ["test_mpi_cuda", "--T", "8192", "--d", "128", "--block", "64"],
])
def test_attention_drivers(args):
    out = _run([os.path.join(BIN, args[0])] + args[1:] + ["--iters", "3"])
    assert _time_ms(out) > 0
    assert _err(out) <= 1e-4


def test_multi_gpu_driver_on_two_gpus():
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    out = _run([os.path.join(BIN, "test_streaming_cuda_multi"), "65536", "128", "64", "2", "--iters", "3"])
    assert _err(out) <= 1e-4


def test_reference_api_side_by_side():
    if not os.path.exists(CHECK):
        pytest.skip("oracle/_ref/cuda_method_check not built (needs the reference tree at build time)")
    out = _run([CHECK], timeout=600)
    assert "CUDA METHOD CHECK OK" in out, out


def _ckpt(tmp_path):
    from oracle.oracle import Qwen3Cfg, make_qwen3_weights
    from streaming_attention_b200.checkpoint import write_qwen3_safetensors
    cfg = dict(vocab=800, hidden=256, n_layers=2, hq=4, hkv=2, head_dim=128, inter=512, eps=1e-6, theta=1e6)
    w = make_qwen3_weights(Qwen3Cfg(**cfg), 5)
    path = str(tmp_path / "q.safetensors")
    write_qwen3_safetensors(path, cfg, w)
    return path, cfg, w


def _field(out, label):
    m = re.search(label + r"\s*(\S+)", out)
    assert m, out
    return float(m.group(1))


def _tokens(out):
    line = [x for x in out.splitlines() if x.startswith("生成tokens:")][0]
    return [int(t) for t in line.split(":", 1)[1].split()]


def test_qwen3_benchmark_driver(tmp_path, oracle):
    """bin/benchmark_qwen3_cuda (the CUDA method of benchmark_qwen3) on a
    synthetic checkpoint: the results block of both phases, and the decode
    phase's greedy tokens equal to the oracle's; with 2 GPUs the head-wise and
    the sequence strategy (both selectable: the legacy --attention no longer
    overrides them) give the same tokens."""
    import numpy as np
    import torch
    from oracle.oracle import Qwen3Cfg
    path, cfg, w = _ckpt(tmp_path)
    exe = os.path.join(BIN, "benchmark_qwen3_cuda")
    out = _run([exe, "--model", path, "--phase", "prefill", "--prompt-len", "64", "--iters", "3"])
    assert _field(out, "处理token数:") == 192 and _field(out, "吞吐量:") > 0
    out = _run([exe, "--model", path, "--phase", "decode", "--prompt-len", "40", "--gen-len", "12", "--iters", "2",
                "--attention", "streaming"])
    toks = _tokens(out)
    assert len(toks) == 12 and _field(out, "处理token数:") == 12
    # the oracle's greedy decode of the same prompt (mt19937(42) ids, as the driver draws them)
    ids = _mt19937_tokens(40, cfg["vocab"])
    c = Qwen3Cfg(**cfg)
    kc = np.zeros((c.n_layers, c.hkv, 64, c.head_dim), np.float32)
    vc = np.zeros_like(kc)
    lg = oracle.qwen3_forward(c, w, np.array(ids), kc, vc, 64, 0, all_logits=False)
    want, pos = [int(np.argmax(lg[0]))], 40
    for _ in range(11):
        lg = oracle.qwen3_forward(c, w, np.array(want[-1:]), kc, vc, 64, pos, all_logits=False)
        pos += 1
        want.append(int(np.argmax(lg[0])))
    assert toks == want
    if torch.cuda.device_count() < 2:
        return
    for strategy in ("headwise", "sequence"):
        out = _run([exe, "--model", path, "--phase", "decode", "--prompt-len", "40", "--gen-len", "12", "--iters",
                    "2", "--gpus", "2", "--parallel-strategy", strategy, "--attention", "standard"])
        assert "并行策略:       " + strategy in out
        assert _tokens(out) == want, strategy
        out = _run([exe, "--model", path, "--phase", "prefill", "--prompt-len", "64", "--iters", "2", "--gpus", "2",
                    "--parallel-strategy", strategy])
        assert _field(out, "处理token数:") == 128


def _mt19937_tokens(n, vocab):
    """std::mt19937(42) + uniform_int_distribution<long>(0, vocab - 1), as the
    reference's generate_random_tokens (benchmark_qwen3.cpp:223-234) and the
    driver draw prompt ids -- computed by a small C++ program."""
    import shutil
    import tempfile
    cxx = "/usr/bin/g++" if os.path.exists("/usr/bin/g++") else shutil.which("g++")
    d = tempfile.mkdtemp()
    src = os.path.join(d, "ids.cpp")
    with open(src, "w") as f:
        f.write("#include <random>\n#include <cstdio>\nint main(){std::mt19937 g(42);"
                f"std::uniform_int_distribution<long> u(0,{vocab - 1});for(int i=0;i<{n};++i)"
                "std::printf(\"%ld\\n\",u(g));}\n")
    subprocess.run([cxx, "-O1", src, "-o", os.path.join(d, "ids")], check=True)
    out = subprocess.run([os.path.join(d, "ids")], capture_output=True, text=True, check=True).stdout
    return [int(x) for x in out.split()]
