"""Qwen3 forward on the GPU (sa_qwen3_* of include/sa_cuda.h).

Mirrors the reference's model API: ``forward`` is ``qwen3_forward`` /
``qwen3_forward_with_cache`` (tensor_cpp/include/tensor_cpp/qwen3_ops.h:242-333),
``reset`` / ``cache_len`` are the ``KVCache`` calls (kv_cache.h), ``generate``
is the greedy decode loop of benchmark_qwen3 with the argmax on the device.
Weights come as fp32 host arrays in the reference's shapes.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

from ._capi import SA_HOST_PTRS, Context, check, default_context, lib


class Qwen3Config(C.Structure):
    """sa_qwen3_config."""
    _fields_ = [("vocab", C.c_int), ("hidden", C.c_int), ("n_layers", C.c_int), ("hq", C.c_int),
                ("hkv", C.c_int), ("head_dim", C.c_int), ("inter", C.c_int), ("eps", C.c_float),
                ("theta", C.c_float), ("max_seq", C.c_int)]


# Qwen3-0.6B: the model of the benchmark configurations configs[3] and configs[4]
QWEN3_0_6B = dict(vocab=151936, hidden=1024, n_layers=28, hq=16, hkv=8, head_dim=128, inter=3072,
                  eps=1e-6, theta=1e6)

# order of one layer's tensors in a packed per-layer fp32 block
LAYER_FIELDS = ("in_norm", "q", "k", "v", "q_norm", "k_norm", "o", "post_norm", "gate", "up", "down")


def layer_shapes(cfg: dict) -> list:
    H, D, I = cfg["hidden"], cfg["head_dim"], cfg["inter"]
    QD, KD = cfg["hq"] * D, cfg["hkv"] * D
    return [(H,), (QD, H), (KD, H), (KD, H), (D,), (D,), (H, QD), (H,), (I, H), (I, H), (H, I)]


def unpack_layer(cfg: dict, flat: np.ndarray) -> dict:
    """Split one packed layer block into named arrays (views)."""
    out, off = {}, 0
    for name, shp in zip(LAYER_FIELDS, layer_shapes(cfg)):
        n = int(np.prod(shp))
        out[name] = flat[off:off + n].reshape(shp)
        off += n
    assert off == flat.size, (off, flat.size)
    return out


def _fp(a: np.ndarray):
    return a.ctypes.data_as(C.POINTER(C.c_float))


_CFG_FIELDS = ("vocab", "hidden", "n_layers", "hq", "hkv", "head_dim", "inter", "eps", "theta")


def inspect_safetensors(path: str) -> dict:
    """The Qwen3 configuration a safetensors checkpoint implies (no GPU needed;
    sa_safetensors_inspect).  Raises SAError for malformed files."""
    c = Qwen3Config()
    check(lib().sa_safetensors_inspect(os.fsencode(path), C.byref(c)))
    return {f: getattr(c, f) for f in _CFG_FIELDS}


SA_TP_HANDLE_BYTES = 64
SA_QWEN3_SP_HANDLE_BYTES = 256


class Qwen3:
    """One Qwen3 model on one GPU, or (rank, world) of a model over `world`
    GPUs: ``strategy="head"`` is head-parallel (sa_qwen3_create_tp: every rank
    keeps its share of the heads and MLP features), ``strategy="sequence"``
    sequence-parallel (sa_qwen3_create_sp: every rank holds the whole model,
    prompts are split over the ranks by tokens).  Every rank is given the
    same full weights; after ``connect`` every rank calls ``forward`` /
    ``generate`` with the same arguments and gets the same results."""

    @classmethod
    def from_safetensors(cls, path: str, max_seq: int = 4096, ctx: Context | None = None,
                         eps: float = 0.0, theta: float = 0.0, rank: int = 0, world: int = 1) -> "Qwen3":
        """A model whose weights are uploaded straight from a safetensors
        checkpoint (sa_qwen3_load_safetensors: bf16 bytes to the GPU, no fp32
        round trip).  eps / theta <= 0 select Qwen3's 1e-6 / 1e6."""
        self = cls.__new__(cls)
        self.cfg = inspect_safetensors(path)
        if eps > 0:
            self.cfg["eps"] = eps
        if theta > 0:
            self.cfg["theta"] = theta
        self.ctx = ctx or default_context(0)
        self.rank, self.world = rank, world
        h = C.c_void_p()
        check(lib().sa_qwen3_load_safetensors_tp(self.ctx.h, os.fsencode(path), max_seq, eps, theta, rank, world,
                                                 C.byref(h)))
        self.h = h
        self.max_seq = max_seq
        return self

    def __init__(self, cfg: dict, max_seq: int = 4096, ctx: Context | None = None, rank: int = 0, world: int = 1,
                 strategy: str = "head"):
        if strategy not in ("head", "sequence"):
            raise ValueError(f"strategy {strategy!r}: 'head' or 'sequence'")
        self.cfg = dict(cfg)
        self.ctx = ctx or default_context(0)
        self.rank, self.world, self.strategy = rank, world, strategy
        c = Qwen3Config(vocab=cfg["vocab"], hidden=cfg["hidden"], n_layers=cfg["n_layers"],
                        hq=cfg["hq"], hkv=cfg["hkv"], head_dim=cfg["head_dim"], inter=cfg["inter"],
                        eps=cfg.get("eps", 1e-6), theta=cfg.get("theta", 1e6), max_seq=max_seq)
        h = C.c_void_p()
        if world == 1:
            check(lib().sa_qwen3_create(self.ctx.h, C.byref(c), C.byref(h)))
        elif strategy == "sequence":
            check(lib().sa_qwen3_create_sp(self.ctx.h, C.byref(c), rank, world, C.byref(h)))
        else:
            check(lib().sa_qwen3_create_tp(self.ctx.h, C.byref(c), rank, world, C.byref(h)))
        self.h = h
        self.max_seq = max_seq

    # -- head-parallel ranks ------------------------------------------------
    def tp_handle(self) -> bytes:
        """This rank's exchange-buffer handle (sa_qwen3_tp_handle)."""
        buf = C.create_string_buffer(SA_TP_HANDLE_BYTES)
        check(lib().sa_qwen3_tp_handle(self.h, buf))
        return buf.raw

    def tp_connect(self, handles) -> None:
        """Map the other ranks' exchange buffers: `handles` in rank order."""
        assert len(handles) == self.world and all(len(x) == SA_TP_HANDLE_BYTES for x in handles)
        blob = b"".join(handles)
        check(lib().sa_qwen3_tp_connect(self.h, C.create_string_buffer(blob, len(blob))))

    @property
    def local_kv_heads(self) -> int:
        """KV heads this rank's cache holds: its share under the head-parallel
        strategy, all of them otherwise."""
        if self.world > 1 and getattr(self, "strategy", "head") == "head":
            return self.cfg["hkv"] // self.world
        return self.cfg["hkv"]

    # -- sequence-parallel ranks --------------------------------------------
    def sp_handle(self) -> bytes:
        """This rank's row-buffer and K/V-cache handles (sa_qwen3_sp_handle)."""
        buf = C.create_string_buffer(SA_QWEN3_SP_HANDLE_BYTES)
        check(lib().sa_qwen3_sp_handle(self.h, buf))
        return buf.raw

    def sp_connect(self, handles) -> None:
        """Map the other ranks' buffers and caches: `handles` in rank order."""
        assert len(handles) == self.world and all(len(x) == SA_QWEN3_SP_HANDLE_BYTES for x in handles)
        blob = b"".join(handles)
        check(lib().sa_qwen3_sp_connect(self.h, C.create_string_buffer(blob, len(blob))))

    def connect(self, group=None) -> None:
        """Exchange handles over a torch.distributed group (one rank per
        process, ranks in group order) and connect."""
        import torch.distributed as dist
        mine = self.sp_handle() if getattr(self, "strategy", "head") == "sequence" else self.tp_handle()
        handles = [None] * self.world
        dist.all_gather_object(handles, mine, group=group)
        if getattr(self, "strategy", "head") == "sequence":
            self.sp_connect(handles)
        else:
            self.tp_connect(handles)

    def close(self):
        if getattr(self, "h", None):
            lib().sa_qwen3_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # -- weights ------------------------------------------------------------
    def set_embed(self, embed, final_norm, lm_head=None):
        e = np.ascontiguousarray(embed, np.float32)
        n = np.ascontiguousarray(final_norm, np.float32)
        lm = None if lm_head is None or lm_head is embed else np.ascontiguousarray(lm_head, np.float32)
        check(lib().sa_qwen3_set_embed(self.h, _fp(e), _fp(n), _fp(lm) if lm is not None else None))

    def set_layer(self, i: int, w: dict):
        a = [np.ascontiguousarray(w[k], np.float32) for k in LAYER_FIELDS]
        check(lib().sa_qwen3_set_layer(self.h, i, *[_fp(x) for x in a]))

    def load(self, weights: dict):
        """weights: {"embed", "final_norm", "lm_head", "layers"} with "layers" the
        packed per-layer fp32 blocks (LAYER_FIELDS order) concatenated."""
        self.set_embed(weights["embed"], weights["final_norm"], weights.get("lm_head"))
        flat = np.ascontiguousarray(weights["layers"], np.float32)
        per = flat.size // self.cfg["n_layers"]
        for i in range(self.cfg["n_layers"]):
            self.set_layer(i, unpack_layer(self.cfg, flat[i * per:(i + 1) * per]))

    # -- forward ------------------------------------------------------------
    def reset(self):
        check(lib().sa_qwen3_reset(self.h))

    @property
    def cache_len(self) -> int:
        return lib().sa_qwen3_cache_len(self.h)

    def read_kv(self, layer: int, seq_stride: int | None = None):
        """(K, V) of one layer's live cache rows: float32 [hkv, seq_stride, head_dim]
        (rows past cache_len are zero), the layout of KVCache's layer tensors."""
        L = self.cache_len
        stride = L if seq_stride is None else seq_stride
        shape = (self.local_kv_heads, stride, self.cfg["head_dim"])
        k, v = np.zeros(shape, np.float32), np.zeros(shape, np.float32)
        check(lib().sa_qwen3_read_kv(self.h, layer, k.ctypes.data, v.ctypes.data, stride))
        return k, v

    def write_kv(self, layer: int, k, v):
        """Upload rows 0..len-1 of one layer's cache from float32 [hkv, len, head_dim]."""
        k = np.ascontiguousarray(k, np.float32)
        v = np.ascontiguousarray(v, np.float32)
        assert k.shape == v.shape and k.shape[0] == self.local_kv_heads and k.shape[2] == self.cfg["head_dim"]
        check(lib().sa_qwen3_write_kv(self.h, layer, k.ctypes.data, v.ctypes.data, k.shape[1], k.shape[1]))

    def set_cache_len(self, n: int):
        check(lib().sa_qwen3_set_cache_len(self.h, n))

    def forward(self, ids, use_cache: bool = False, logits: str = "all"):
        ids = np.ascontiguousarray(ids, np.int64).ravel()
        S = ids.size
        mode = {"all": 0, "last": 1, "none": 2}[logits]
        out = None if mode == 2 else np.empty((S if mode == 0 else 1, self.cfg["vocab"]), np.float32)
        check(lib().sa_qwen3_forward(self.h, ids.ctypes.data_as(C.POINTER(C.c_int64)), S,
                                     1 if use_cache else 0,
                                     _fp(out) if out is not None else None, mode, SA_HOST_PTRS))
        return out

    def generate(self, prompt, n_new: int) -> np.ndarray:
        prompt = np.ascontiguousarray(prompt, np.int64).ravel()
        out = np.empty(max(n_new, 1), np.int64)
        check(lib().sa_qwen3_generate(self.h, prompt.ctypes.data_as(C.POINTER(C.c_int64)), prompt.size,
                                      n_new, out.ctypes.data_as(C.POINTER(C.c_int64)), SA_HOST_PTRS))
        return out[:n_new]


def bf16_round(x: np.ndarray) -> np.ndarray:
    """Round fp32 values to the nearest bf16 (ties to even), kept as fp32
    (finite inputs; 32-bit arithmetic, u + 0x7FFF + lsb < 2^32 for them)."""
    x = np.ascontiguousarray(x, np.float32)
    u = x.view(np.uint32)
    r = (u >> 16) & np.uint32(1)
    r += np.uint32(0x7FFF)
    r += u
    r &= np.uint32(0xFFFF0000)
    return r.view(np.float32).reshape(x.shape)


def random_weights(cfg: dict, seed: int, std: float = 0.02) -> dict:
    """Synthetic random-init weights for benchmarking (no checkpoint is
    available): matrices N(0, std) rounded to bf16, norm gains 1, lm_head tied
    to the embedding -- the initialisation BASELINE.json's Qwen3 configs name.
    Returns the packed layout ``Qwen3.load`` takes."""
    rng = np.random.default_rng(seed)
    shapes = layer_shapes(cfg)
    parts = []
    for _ in range(cfg["n_layers"]):
        for name, shp in zip(LAYER_FIELDS, shapes):
            if len(shp) == 1:
                parts.append(np.ones(shp, np.float32))
            else:
                parts.append(bf16_round(rng.standard_normal(shp, dtype=np.float32) * std).ravel())
    layers = np.concatenate([p.ravel() for p in parts])
    embed = bf16_round(rng.standard_normal((cfg["vocab"], cfg["hidden"]), dtype=np.float32) * std)
    return {"embed": embed, "layers": layers, "final_norm": np.ones(cfg["hidden"], np.float32),
            "lm_head": embed}
