"""Safetensors checkpoints (CPU only): the synthetic-checkpoint writer produces
files the official safetensors reader reads back bit-exactly, files written by
the official writer pass this library's validation, the configuration is
inferred from the shapes, and malformed files are rejected with the tensor
named (sa_safetensors_inspect needs no GPU)."""
import json
import os
import struct

import numpy as np

from oracle.oracle import bf16_round
import pytest

CFG = dict(vocab=500, hidden=256, n_layers=2, hq=4, hkv=2, head_dim=128, inter=512, eps=1e-6, theta=1e6)


def _weights(seed=3):
    from streaming_attention_b200.qwen3 import random_weights
    w = random_weights(CFG, seed)
    w["final_norm"] = bf16_round(np.linspace(0.5, 1.5, CFG["hidden"], dtype=np.float32))   # not all ones
    return w


@pytest.mark.parametrize("dtype", ["BF16", "F16", "F32"])
@pytest.mark.parametrize("tied", [True, False])
def test_writer_roundtrip_with_official_reader(tmp_path, dtype, tied):
    import torch
    from safetensors.torch import load_file
    from streaming_attention_b200.checkpoint import qwen3_tensors, write_qwen3_safetensors
    from streaming_attention_b200.qwen3 import inspect_safetensors
    w = _weights()
    p = str(tmp_path / "m.safetensors")
    write_qwen3_safetensors(p, CFG, w, dtype=dtype, tied=tied)
    got = load_file(p)
    want = qwen3_tensors(CFG, w, tied)
    assert set(got) == set(want)
    tdt = {"BF16": torch.bfloat16, "F16": torch.float16, "F32": torch.float32}[dtype]
    for name, arr in want.items():
        assert got[name].dtype == tdt and tuple(got[name].shape) == arr.shape
        np.testing.assert_array_equal(got[name].float().numpy(), torch.from_numpy(arr).to(tdt).float().numpy())
    cfg = inspect_safetensors(p)
    assert {k: cfg[k] for k in ("vocab", "hidden", "n_layers", "hq", "hkv", "head_dim", "inter")} == \
        {k: CFG[k] for k in ("vocab", "hidden", "n_layers", "hq", "hkv", "head_dim", "inter")}


def test_official_writer_file_is_accepted(tmp_path):
    import torch
    from safetensors.torch import save_file
    from streaming_attention_b200.checkpoint import qwen3_tensors
    from streaming_attention_b200.qwen3 import inspect_safetensors
    t = {k: torch.from_numpy(np.ascontiguousarray(v)).to(torch.bfloat16)
         for k, v in qwen3_tensors(CFG, _weights(), tied=True).items()}
    p = str(tmp_path / "hf.safetensors")
    save_file(t, p, metadata={"format": "pt"})
    assert inspect_safetensors(p)["n_layers"] == 2


def _rewrite_header(src, dst, edit):
    raw = open(src, "rb").read()
    n = struct.unpack("<Q", raw[:8])[0]
    h = json.loads(raw[8:8 + n])
    edit(h)
    hb = json.dumps(h).encode()
    hb += b" " * (-len(hb) % 8)
    open(dst, "wb").write(struct.pack("<Q", len(hb)) + hb + raw[8 + n:])


@pytest.mark.parametrize("case,needle", [
    ("missing", "model.layers.1.mlp.down_proj.weight"),
    ("shape", "model.layers.0.self_attn.k_proj.weight"),
    ("dtype", "model.layers.0.mlp.up_proj.weight"),
    ("offsets", "model.norm.weight"),
    ("truncated", "outside"),
    ("notjson", "JSON"),
    ("hugelen", "header length"),
    ("noembed", "embed_tokens"),
])
def test_malformed_files_are_rejected(tmp_path, case, needle):
    from streaming_attention_b200 import SAError
    from streaming_attention_b200.checkpoint import write_qwen3_safetensors
    from streaming_attention_b200.qwen3 import inspect_safetensors
    good = str(tmp_path / "good.safetensors")
    write_qwen3_safetensors(good, CFG, _weights())
    bad = str(tmp_path / "bad.safetensors")
    if case == "missing":
        _rewrite_header(good, bad, lambda h: h.pop("model.layers.1.mlp.down_proj.weight"))
    elif case == "shape":
        _rewrite_header(good, bad, lambda h: h["model.layers.0.self_attn.k_proj.weight"].update(
            shape=[128, 512]))
    elif case == "dtype":
        def f(h):
            e = h["model.layers.0.mlp.up_proj.weight"]
            e["dtype"] = "I16"
        _rewrite_header(good, bad, f)
    elif case == "offsets":
        _rewrite_header(good, bad, lambda h: h["model.norm.weight"].update(data_offsets=[0, 10]))
    elif case == "truncated":
        raw = open(good, "rb").read()
        open(bad, "wb").write(raw[:len(raw) // 2])
    elif case == "notjson":
        raw = open(good, "rb").read()
        n = struct.unpack("<Q", raw[:8])[0]
        open(bad, "wb").write(raw[:8] + b"{" + b"x" * (n - 1) + raw[8 + n:])
    elif case == "hugelen":
        raw = open(good, "rb").read()
        open(bad, "wb").write(struct.pack("<Q", 1 << 62) + raw[8:])
    elif case == "noembed":
        _rewrite_header(good, bad, lambda h: h.pop("model.embed_tokens.weight"))
    with pytest.raises(SAError) as e:
        inspect_safetensors(bad)
    assert e.value.code == -1 and needle in str(e.value), str(e.value)


def test_missing_file_is_an_argument_error(tmp_path):
    from streaming_attention_b200 import SAError
    from streaming_attention_b200.qwen3 import inspect_safetensors
    with pytest.raises(SAError):
        inspect_safetensors(str(tmp_path / "absent.safetensors"))


def test_reference_loader_reads_the_synthetic_checkpoint(tmp_path):
    """The reference's own load_qwen3_weights (compiled from its sources) reads
    a checkpoint written here and computes the logits the oracle computes on
    the original weights.  Its loader fixes 28 layers and 16/8 heads of 128,
    so the checkpoint keeps those and shrinks hidden / inter / vocab."""
    from oracle.oracle import Oracle, Qwen3Cfg, RefQwen3, Reference
    from streaming_attention_b200.checkpoint import write_qwen3_safetensors
    from streaming_attention_b200.qwen3 import inspect_safetensors, random_weights
    try:
        ref = Reference()
    except FileNotFoundError as e:
        pytest.skip(str(e))
    cfg = dict(vocab=300, hidden=256, n_layers=28, hq=16, hkv=8, head_dim=128, inter=256, eps=1e-6, theta=1e6)
    w = random_weights(cfg, 7)
    w["final_norm"] = bf16_round(np.linspace(0.5, 1.5, cfg["hidden"], dtype=np.float32))
    p = str(tmp_path / "ref.safetensors")
    write_qwen3_safetensors(p, cfg, w, tied=False)      # this loader needs lm_head.weight
    r = RefQwen3.from_safetensors(ref, p)
    assert (r.cfg.vocab, r.cfg.hidden, r.cfg.n_layers, r.cfg.inter) == (300, 256, 28, 256)
    assert inspect_safetensors(p)["n_layers"] == 28
    ids = np.array([3, 141, 59, 26, 299])
    got = r.forward(ids)
    want = Oracle().qwen3_forward(Qwen3Cfg(**cfg), w, ids)
    assert np.abs(got - want).max() <= 1e-4 * np.abs(want).max()
    r.close()
