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
