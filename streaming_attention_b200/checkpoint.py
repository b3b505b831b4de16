"""Qwen3 checkpoints in the safetensors format.

``write_qwen3_safetensors`` writes a weights dict (the layout ``Qwen3.load``
takes) as a single safetensors file with the Hugging Face Qwen3 tensor names
that the reference's loader reads (tensor_cpp/src/qwen3_loader.cpp:140-297)
and ``sa_qwen3_load_safetensors`` uploads.  With no checkpoint available
offline, this is how a synthetic random-init Qwen3-0.6B checkpoint is made for
the loader tests and for loading the same weights on both sides of a
comparison.

File layout: 8-byte little-endian header length, a JSON header (padded with
spaces to a multiple of 8 bytes) mapping each name to its dtype, shape and
[begin, end) byte offsets in the data section, then the data.
"""
from __future__ import annotations

import json
import struct

import numpy as np

from .qwen3 import LAYER_FIELDS, unpack_layer

_HF_LAYER = {
    "in_norm": "input_layernorm.weight", "q": "self_attn.q_proj.weight", "k": "self_attn.k_proj.weight",
    "v": "self_attn.v_proj.weight", "q_norm": "self_attn.q_norm.weight", "k_norm": "self_attn.k_norm.weight",
    "o": "self_attn.o_proj.weight", "post_norm": "post_attention_layernorm.weight",
    "gate": "mlp.gate_proj.weight", "up": "mlp.up_proj.weight", "down": "mlp.down_proj.weight",
}


def to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even bf16 bit patterns (uint16) of float32 values."""
    u = np.ascontiguousarray(x, np.float32).view(np.uint32)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def qwen3_tensors(cfg: dict, weights: dict, tied: bool = True) -> dict:
    """name -> float32 array in the Hugging Face Qwen3 naming."""
    out = {"model.embed_tokens.weight": weights["embed"], "model.norm.weight": weights["final_norm"]}
    if not tied:
        out["lm_head.weight"] = weights.get("lm_head", weights["embed"])
    flat = np.ascontiguousarray(weights["layers"], np.float32)
    per = flat.size // cfg["n_layers"]
    for i in range(cfg["n_layers"]):
        parts = unpack_layer(cfg, flat[i * per:(i + 1) * per])
        for f in LAYER_FIELDS:
            out[f"model.layers.{i}.{_HF_LAYER[f]}"] = parts[f]
    return out


def write_safetensors(path: str, tensors: dict, dtype: str = "BF16", metadata: dict | None = None) -> None:
    """Write name -> array (float32 values) as a safetensors file in BF16, F16 or F32."""
    conv = {"BF16": to_bf16_bits, "F16": lambda a: np.asarray(a, np.float16),
            "F32": lambda a: np.asarray(a, np.float32)}[dtype]
    header, blobs, off = {}, [], 0
    if metadata:
        header["__metadata__"] = {str(k): str(v) for k, v in metadata.items()}
    for name, arr in tensors.items():
        data = np.ascontiguousarray(conv(arr)).tobytes()
        header[name] = {"dtype": dtype, "shape": list(np.shape(arr)), "data_offsets": [off, off + len(data)]}
        blobs.append(data)
        off += len(data)
    h = json.dumps(header, separators=(",", ":")).encode()
    h += b" " * (-len(h) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)


def write_qwen3_safetensors(path: str, cfg: dict, weights: dict, dtype: str = "BF16", tied: bool = True) -> None:
    """A Qwen3 checkpoint of ``weights`` (the ``Qwen3.load`` dict) at ``path``;
    with ``tied`` the file has no lm_head.weight (Qwen3-0.6B's tied embeddings)."""
    write_safetensors(path, qwen3_tensors(cfg, weights, tied), dtype,
                      {"format": "pt", "producer": "streaming_attention_b200.checkpoint"})
