"""The C++ host layer over the C ABI (CPU only): libsa_host.so provides every
function include/sa_attention_cuda.h declares, the command-line drivers parse
the reference drivers' argument forms, and the header-only Qwen3 adapter
compiles against the reference's own headers when that tree is present."""
import os
import re
import shutil
import subprocess

import pytest

from conftest import ROOT

PKG = os.path.join(ROOT, "streaming_attention_b200")
BIN = os.path.join(PKG, "bin")
# the reference tree: $SA_REFERENCE_DIR, else a checkout named `reference` beside this repository
REF = os.environ.get("SA_REFERENCE_DIR", os.path.join(os.path.dirname(ROOT), "reference"))
CXX = "/usr/bin/g++" if os.path.exists("/usr/bin/g++") else shutil.which("g++")
DRIVERS = ["test_naive_cuda", "test_streaming_cuda", "test_streaming_cuda_multi", "test_mpi_cuda",
           "benchmark_qwen3_cuda"]


def _declared_cpp():
    src = open(os.path.join(ROOT, "include", "sa_attention_cuda.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return re.findall(r"^[\w:<>]+\s+\**(\w+)\s*\(", src, flags=re.M)


def test_host_library_links_every_declared_function(tmp_path):
    names = _declared_cpp()
    assert {"naive_attention_cuda", "streaming_attention_cuda", "streaming_attention_cuda_multi"} <= set(names)
    if CXX is None:
        pytest.skip("no C++ compiler")
    # a program that takes the address of each declared function links only if
    # libsa_host.so defines all of them
    prog = tmp_path / "link.cpp"
    prog.write_text('#include "sa_attention_cuda.h"\n#include <cstdio>\nint main() {\n' +
                    "".join(f'  std::printf("%p\\n", (void*)&{n});\n' for n in names) + "  return 0;\n}\n")
    exe = tmp_path / "link"
    subprocess.run([CXX, "-std=c++17", "-I", os.path.join(ROOT, "include"), str(prog), "-o", str(exe),
                    "-L", PKG, "-lsa_host", "-lsa_cuda", f"-Wl,-rpath,{PKG}"], check=True)


@pytest.mark.parametrize("name", DRIVERS)
def test_driver_usage(name):
    exe = os.path.join(BIN, name)
    assert os.path.exists(exe), f"{exe} not built (make -C streaming_attention_b200)"
    r = subprocess.run([exe, "--help"], capture_output=True, text=True, timeout=30)
    assert r.returncode == 2 and "usage:" in r.stderr


@pytest.mark.skipif(not os.path.isdir(os.path.join(REF, "tensor_cpp", "include")),
                    reason="reference headers not present")
def test_qwen3_adapter_compiles_against_reference_headers(tmp_path):
    src = tmp_path / "use.cpp"
    src.write_text(
        '#include "tensor_cpp/qwen3_ops.h"\n#include "sa_qwen3_tensorcpp.hpp"\n'
        "using namespace tensor_cpp;\n"
        "Tensor f(const TensorL& ids, qwen3::KVCache* kv, const qwen3::Qwen3Weights* w) {\n"
        "  return qwen3::cuda::qwen3_forward_cuda_with_cache(ids, kv, w->embed_tokens, w->layers,\n"
        "      w->norm_weight, w->lm_head, w->num_layers, w->num_attention_heads, w->num_key_value_heads,\n"
        "      w->head_dim, 1e-6f, qwen3::AttentionType::STREAMING);\n}\n"
        "Tensor g(const TensorL& ids, const qwen3::Qwen3Weights& w) {\n"
        "  return qwen3::cuda::qwen3_forward_cuda(ids, w.embed_tokens, w.layers, w.norm_weight, w.lm_head,\n"
        "      w.num_layers, w.num_attention_heads, w.num_key_value_heads, w.head_dim, 1e-6f);\n}\n")
    r = subprocess.run([CXX, "-std=c++17", "-fsyntax-only", "-w", "-I", os.path.join(REF, "tensor_cpp", "include"),
                        "-I", os.path.join(ROOT, "include"), '-include', "tensor_cpp/qwen3_loader.h", str(src)],
                       capture_output=True, text=True)
    assert r.returncode == 0, r.stderr[-2000:]


@pytest.mark.skipif(not os.path.isdir(os.path.join(REF, "tensor_cpp", "include")),
                    reason="reference headers not present")
def test_ops_adapter_compiles_against_reference_headers(tmp_path):
    """include/sa_ops_tensorcpp.hpp: the CUDA method of ops::self_attention,
    self_attention_streaming[_blockwise] and the ops::mpi head-wise / sequence
    operators, called with the reference's Tensor types."""
    src = tmp_path / "use_ops.cpp"
    src.write_text(
        '#include "tensor_cpp/ops.h"\n#include "sa_ops_tensorcpp.hpp"\n'
        "using namespace tensor_cpp;\n"
        "Tensor f(const Tensor& q, const Tensor& k, const Tensor& v, const Tensor* m) {\n"
        "  Tensor a = ops::cuda::self_attention(q, k, v, m, 0.1f);\n"
        "  Tensor b = ops::cuda::self_attention_streaming(q, k, v, 0.1f, 64);\n"
        "  Tensor c = ops::cuda::self_attention_streaming_blockwise(q, k, v, 0.1f, 32, 64);\n"
        "  Tensor d = ops::mpi::cuda::attention_headwise_standard(q, k, v, m, 0.1f, 16, 8);\n"
        "  Tensor e = ops::mpi::cuda::attention_headwise_online_softmax(q, k, v, m, 0.1f, 16, 8, 2);\n"
        "  return ops::mpi::cuda::attention_sequence_online_softmax(q, k, v, m, 0.1f, 16, 8, 128, 4);\n}\n")
    r = subprocess.run([CXX, "-std=c++17", "-fsyntax-only", "-Wall", "-Wextra", "-I",
                        os.path.join(REF, "tensor_cpp", "include"), "-I", os.path.join(ROOT, "include"), str(src)],
                       capture_output=True, text=True)
    assert r.returncode == 0, r.stderr[-2000:]
    assert "sa_ops_tensorcpp.hpp" not in r.stderr, r.stderr[-2000:]    # no warnings from the header itself


def test_qwen3_driver_rejects_other_methods_and_bad_options():
    """benchmark_qwen3_cuda takes the reference driver's options; it runs the
    CUDA method only and refuses what that method does not do (no GPU needed:
    the options are checked before any CUDA call)."""
    exe = os.path.join(BIN, "benchmark_qwen3_cuda")
    r = subprocess.run([exe, "--model", "x.safetensors", "--method", "avx2"], capture_output=True, text=True)
    assert r.returncode == 2 and "--method cuda" in r.stderr
    r = subprocess.run([exe, "--model", "x.safetensors", "--batch-size", "4"], capture_output=True, text=True)
    assert r.returncode == 2 and "batch 1" in r.stderr
    r = subprocess.run([exe, "--model", "x.safetensors", "--parallel-strategy", "pipeline"], capture_output=True,
                       text=True)
    assert r.returncode == 2 and "usage:" in r.stderr
