"""ctypes bindings for the parity checker.

TEST INFRASTRUCTURE ONLY.  Only tests/, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of bench.py import this module.

* :class:`Oracle` wraps ``oracle/_build/libsa_oracle.so``: the C restatement
  of the reference's arithmetic (``oracle/sa_oracle.c``).
* :class:`Reference` wraps ``oracle/_ref/libsa_ref.so``: the reference's own
  CPU implementation compiled from its sources by ``oracle/Makefile``.

Both take and return numpy arrays.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "_build", "libsa_oracle.so")
REF_SO = os.path.join(HERE, "_ref", "libsa_ref.so")

_fp = C.POINTER(C.c_float)
_i64p = C.POINTER(C.c_int64)


def build(quiet: bool = True) -> None:
    """Run ``make -C oracle`` (the reference part only when its tree exists)."""
    subprocess.run(["make", "-C", HERE], check=True,
                   stdout=subprocess.DEVNULL if quiet else None)


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


def _p(a: np.ndarray):
    return a.ctypes.data_as(_fp)


class Qwen3Cfg(C.Structure):
    """Mirror of ``orc_qwen3_cfg`` / ``RefCfg``."""
    _fields_ = [("vocab", C.c_int), ("hidden", C.c_int), ("n_layers", C.c_int),
                ("hq", C.c_int), ("hkv", C.c_int), ("head_dim", C.c_int),
                ("inter", C.c_int), ("eps", C.c_float), ("theta", C.c_float)]


def layer_floats(cfg: Qwen3Cfg) -> int:
    H, D, I = cfg.hidden, cfg.head_dim, cfg.inter
    return (H + cfg.hq * D * H + 2 * cfg.hkv * D * H + 2 * D + H * cfg.hq * D + H
            + 3 * I * H)


def bf16_round(x: np.ndarray) -> np.ndarray:
    """Round fp32 to the nearest bf16 (ties to even); returns fp32 values.
    32-bit arithmetic: u + 0x7FFF + lsb stays below 2^32 for every non-NaN
    pattern; NaNs are made quiet and truncated."""
    x = _f32(x)
    u = x.view(np.uint32)
    r = (u >> 16) & np.uint32(1)
    r += np.uint32(0x7FFF)
    r += u
    r &= np.uint32(0xFFFF0000)
    nan = (u & np.uint32(0x7FFFFFFF)) > np.uint32(0x7F800000)
    if nan.any():
        r[nan] = (u[nan] | np.uint32(0x00400000)) & np.uint32(0xFFFF0000)
    return r.view(np.float32).reshape(x.shape)


class Oracle:
    """The C restatement (oracle/sa_oracle.c)."""

    def __init__(self, path: str = ORACLE_SO):
        if not os.path.exists(path):
            build()
        L = C.CDLL(path)
        self.L = L
        L.orc_naive_attention.argtypes = [_fp, _fp, _fp, C.c_int, C.c_int, C.c_float, _fp]
        L.orc_streaming_attention.argtypes = [_fp, _fp, _fp, C.c_int, C.c_int, C.c_int, C.c_float, _fp]
        L.orc_streaming_chunked.argtypes = [_fp, _fp, _fp, C.c_int, C.c_int, C.c_int, C.c_int, C.c_float, _fp]
        L.orc_partial.argtypes = [_fp, _fp, _fp, C.c_int, C.c_int, C.c_int, C.c_int, C.c_float, _fp, _fp, _fp]
        L.orc_merge.argtypes = [_fp, _fp, _fp, C.c_float, C.c_float, _fp, C.c_int]
        L.orc_gqa_decode.argtypes = [_fp, _fp, _fp, C.c_longlong, C.c_int, C.c_int, C.c_int,
                                     C.c_int, C.c_int, C.c_float, _fp]
        L.orc_causal_prefill.argtypes = [_fp, _fp, _fp, _fp, C.c_int, C.c_int, C.c_int, C.c_int,
                                         C.c_int, C.c_int] + [C.c_longlong] * 6 + [C.c_int, C.c_float]
        L.orc_rms_norm.argtypes = [_fp, _fp, C.c_int, C.c_int, C.c_float, _fp]
        L.orc_linear.argtypes = [_fp, _fp, C.c_int, C.c_int, C.c_int, _fp]
        L.orc_rope_tables.argtypes = [C.c_int, C.c_int, C.c_float, _fp, _fp]
        L.orc_qwen3_forward.argtypes = [C.POINTER(Qwen3Cfg), _fp, _fp, _fp, _fp, _i64p, C.c_int,
                                        _fp, _fp, C.c_int, C.c_int, C.c_int, _fp]
        L.orc_qwen3_forward.restype = C.c_int

    # -- single-query attention -------------------------------------------
    def naive(self, q, k, v, scale=1.0):
        q, k, v = _f32(q), _f32(k), _f32(v)
        T, d = k.shape
        out = np.empty(d, np.float32)
        self.L.orc_naive_attention(_p(q), _p(k), _p(v), T, d, scale, _p(out))
        return out

    def streaming(self, q, k, v, block=64, scale=1.0):
        q, k, v = _f32(q), _f32(k), _f32(v)
        T, d = k.shape
        out = np.empty(d, np.float32)
        self.L.orc_streaming_attention(_p(q), _p(k), _p(v), T, d, block, scale, _p(out))
        return out

    def chunked(self, q, k, v, block=64, threads=8, scale=1.0):
        q, k, v = _f32(q), _f32(k), _f32(v)
        T, d = k.shape
        out = np.empty(d, np.float32)
        self.L.orc_streaming_chunked(_p(q), _p(k), _p(v), T, d, block, threads, scale, _p(out))
        return out

    def partial(self, q, k, v, t0, t1, block=64, scale=1.0):
        q, k, v = _f32(q), _f32(k), _f32(v)
        d = k.shape[1]
        m, l = np.zeros(1, np.float32), np.zeros(1, np.float32)
        o = np.empty(d, np.float32)
        self.L.orc_partial(_p(q), _p(k), _p(v), t0, t1, d, block, scale, _p(m), _p(l), _p(o))
        return float(m[0]), float(l[0]), o

    def merge(self, parts):
        """Fold (m, l, O) partials left to right into a fresh (-inf, 1, 0) state."""
        d = parts[0][2].shape[0]
        m = np.array([-np.inf], np.float32)
        l = np.array([1.0], np.float32)
        o = np.zeros(d, np.float32)
        for pm, pl, po in parts:
            po = _f32(po)
            self.L.orc_merge(_p(m), _p(l), _p(o), pm, pl, _p(po), d)
        return float(m[0]), float(l[0]), o

    def gqa_decode(self, q, k, v, block=64, scale=1.0):
        """q [hq, d]; k, v [hkv, T, d] -> [hq, d]."""
        q, k, v = _f32(q), _f32(k), _f32(v)
        hq, d = q.shape
        hkv, T, _ = k.shape
        out = np.empty((hq, d), np.float32)
        self.L.orc_gqa_decode(_p(q), _p(k), _p(v), T * d, T, d, hq, hkv, block, scale, _p(out))
        return out

    def causal_prefill(self, q, k, v, scale, q_pos0=0, kv_block=64):
        """q [Sq, hq, d]; k, v [Skv, hkv, d] (token-major) -> [Sq, hq, d]."""
        q, k, v = _f32(q), _f32(k), _f32(v)
        Sq, hq, d = q.shape
        Skv, hkv, _ = k.shape
        out = np.empty_like(q)
        self.L.orc_causal_prefill(_p(q), _p(k), _p(v), _p(out), Sq, Skv, q_pos0, hq, hkv, d,
                                  hq * d, d, hkv * d, d, hq * d, d, kv_block, scale)
        return out

    # -- Qwen3 ---------------------------------------------------------------
    def qwen3_forward(self, cfg: Qwen3Cfg, w: dict, ids, kc=None, vc=None, max_seq=0, pos0=0,
                      all_logits=True):
        ids = np.ascontiguousarray(ids, np.int64)
        S = ids.shape[0]
        logits = np.empty((S if all_logits else 1, cfg.vocab), np.float32)
        kp = _p(kc) if kc is not None else None
        vp = _p(vc) if vc is not None else None
        rc = self.L.orc_qwen3_forward(C.byref(cfg), _p(w["embed"]), _p(w["layers"]),
                                      _p(w["final_norm"]), _p(w["lm_head"]),
                                      ids.ctypes.data_as(_i64p), S, kp, vp, max_seq, pos0,
                                      1 if all_logits else 0, _p(logits))
        if rc != 0:
            raise ValueError(f"orc_qwen3_forward failed: {rc}")
        return logits


class Reference:
    """The reference's CPU implementation (oracle/_ref/libsa_ref.so)."""

    def __init__(self, path: str = REF_SO):
        if not os.path.exists(path):
            raise FileNotFoundError(
                f"{path} missing: build it with `make -C oracle` where the reference tree exists")
        L = C.CDLL(path)
        self.L = L
        L.ref_last_error.restype = C.c_char_p
        L.ref_naive_attention_serial.argtypes = [_fp, _fp, _fp, C.c_int, C.c_int, _fp]
        L.ref_naive_attention_omp.argtypes = [_fp, _fp, _fp, C.c_int, C.c_int, C.c_int, _fp]
        L.ref_streaming_attention_serial.argtypes = [_fp, _fp, _fp, C.c_int, C.c_int, C.c_int, _fp]
        L.ref_streaming_attention_omp.argtypes = [_fp, _fp, _fp, C.c_int, C.c_int, C.c_int, C.c_int, _fp]
        L.ref_gqa_decode_omp.argtypes = [_fp, _fp, _fp, C.c_longlong, C.c_int, C.c_int, C.c_int,
                                         C.c_int, C.c_int, C.c_int, C.c_float, _fp]
        L.ref_causal_prefill.argtypes = [_fp, _fp, _fp, C.c_int, C.c_int, C.c_int, C.c_int,
                                         C.c_float, C.c_int, C.c_int, C.c_int, _fp]
        L.ref_causal_prefill.restype = C.c_int
        L.ref_qwen3_create.argtypes = [C.POINTER(Qwen3Cfg), _fp, _fp, _fp, _fp]
        L.ref_qwen3_create.restype = C.c_void_p
        L.ref_qwen3_destroy.argtypes = [C.c_void_p]
        L.ref_qwen3_forward.argtypes = [C.c_void_p, _i64p, C.c_int, C.c_int, _fp]
        L.ref_qwen3_forward.restype = C.c_int
        L.ref_kv_create.argtypes = [C.c_int, C.c_int, C.c_int, C.c_int]
        L.ref_kv_create.restype = C.c_void_p
        L.ref_kv_destroy.argtypes = [C.c_void_p]
        L.ref_kv_len.argtypes = [C.c_void_p]
        L.ref_kv_len.restype = C.c_longlong
        L.ref_qwen3_forward_cached.argtypes = [C.c_void_p, C.c_void_p, _i64p, C.c_int, C.c_int, _fp]
        L.ref_qwen3_forward_cached.restype = C.c_int

    def _err(self, what):
        raise RuntimeError(f"{what}: {self.L.ref_last_error().decode()}")

    def naive_serial(self, q, k, v):
        q, k, v = _f32(q), _f32(k), _f32(v)
        T, d = k.shape
        out = np.empty(d, np.float32)
        self.L.ref_naive_attention_serial(_p(q), _p(k), _p(v), T, d, _p(out))
        return out

    def streaming_serial(self, q, k, v, block=64):
        q, k, v = _f32(q), _f32(k), _f32(v)
        T, d = k.shape
        out = np.empty(d, np.float32)
        self.L.ref_streaming_attention_serial(_p(q), _p(k), _p(v), T, d, block, _p(out))
        return out

    def streaming_omp(self, q, k, v, block=64, threads=0):
        q, k, v = _f32(q), _f32(k), _f32(v)
        T, d = k.shape
        out = np.empty(d, np.float32)
        self.L.ref_streaming_attention_omp(_p(q), _p(k), _p(v), T, d, block, threads, _p(out))
        return out

    def gqa_decode_omp(self, q, k, v, block=64, threads=0, scale=1.0, out=None):
        """q [hq, d]; k, v [hkv, T, d] (contiguous) -> [hq, d]."""
        q, k, v = _f32(q), _f32(k), _f32(v)
        hq, d = q.shape
        hkv, T, _ = k.shape
        if out is None:
            out = np.empty((hq, d), np.float32)
        self.L.ref_gqa_decode_omp(_p(q), _p(k), _p(v), T * d, T, d, hq, hkv, block, threads,
                                  scale, _p(out))
        return out

    def causal_prefill(self, q, k, v, scale, q_block=32, kv_block=64, standard=False, avx2=False):
        """q [Sq, hq, d]; k, v [S, hkv, d] (token-major, Sq == S) -> [S, hq, d].
        standard: ops::self_attention with the causal mask; avx2: the
        reference's self_attention_streaming_blockwise_avx2; else the scalar
        self_attention_streaming_blockwise."""
        q, k, v = _f32(q), _f32(k), _f32(v)
        S, hq, d = q.shape
        hkv = k.shape[1]
        qh = np.ascontiguousarray(q.transpose(1, 0, 2))
        kh = np.ascontiguousarray(k.transpose(1, 0, 2))
        vh = np.ascontiguousarray(v.transpose(1, 0, 2))
        out = np.empty_like(qh)
        if self.L.ref_causal_prefill(_p(qh), _p(kh), _p(vh), S, hq, hkv, d, scale, q_block,
                                     kv_block, 1 if standard else (2 if avx2 else 0), _p(out)):
            self._err("ref_causal_prefill")
        return np.ascontiguousarray(out.transpose(1, 0, 2))

    # -- Qwen3 ---------------------------------------------------------------
    def qwen3(self, cfg: Qwen3Cfg, w: dict) -> "RefQwen3":
        return RefQwen3(self, cfg, w)


class RefQwen3:
    def __init__(self, ref: Reference, cfg: Qwen3Cfg, w: dict):
        self.ref, self.cfg = ref, cfg
        self.h = ref.L.ref_qwen3_create(C.byref(cfg), _p(w["embed"]), _p(w["layers"]),
                                        _p(w["final_norm"]), _p(w["lm_head"]))

    @classmethod
    def from_safetensors(cls, ref: Reference, path: str) -> "RefQwen3":
        """Weights read by the reference's own load_qwen3_weights
        (qwen3_loader.cpp:140-297)."""
        self = cls.__new__(cls)
        self.ref, self.cfg = ref, Qwen3Cfg()
        ref.L.ref_qwen3_load.restype = C.c_void_p
        ref.L.ref_qwen3_load.argtypes = [C.c_char_p, C.c_void_p]
        self.h = ref.L.ref_qwen3_load(os.fsencode(path), C.byref(self.cfg))
        if not self.h:
            ref._err("ref_qwen3_load")
        return self

    def close(self):
        if self.h:
            self.ref.L.ref_qwen3_destroy(self.h)
            self.h = None

    __del__ = close

    def forward(self, ids, method=0):
        ids = np.ascontiguousarray(ids, np.int64)
        S = ids.shape[0]
        logits = np.empty((S, self.cfg.vocab), np.float32)
        if self.ref.L.ref_qwen3_forward(self.h, ids.ctypes.data_as(_i64p), S, method, _p(logits)):
            self.ref._err("ref_qwen3_forward")
        return logits

    def new_cache(self, max_seq):
        return self.ref.L.ref_kv_create(self.cfg.n_layers, self.cfg.hkv, self.cfg.head_dim, max_seq)

    def forward_cached(self, kv, ids, method=0):
        ids = np.ascontiguousarray(ids, np.int64)
        S = ids.shape[0]
        logits = np.empty((S, self.cfg.vocab), np.float32)
        if self.ref.L.ref_qwen3_forward_cached(self.h, kv, ids.ctypes.data_as(_i64p), S, method,
                                               _p(logits)):
            self.ref._err("ref_qwen3_forward_cached")
        return logits

    def free_cache(self, kv):
        self.ref.L.ref_kv_destroy(kv)


def make_qwen3_weights(cfg: Qwen3Cfg, seed: int, std: float = 0.02) -> dict:
    """Seeded random-init weights, N(0, std) for matrices, gains 1, tied lm_head.

    Every value is bf16-representable (rounded once), so a bf16 device copy and
    the fp32 CPU checkers see identical weights.
    """
    rng = np.random.default_rng(seed)
    H, D, I, V = cfg.hidden, cfg.head_dim, cfg.inter, cfg.vocab
    QD, KD = cfg.hq * D, cfg.hkv * D

    def mat(r, c):
        return bf16_round(rng.standard_normal((r, c), dtype=np.float32) * std)

    ones = lambda n: np.ones(n, np.float32)
    parts = []
    for _ in range(cfg.n_layers):
        parts += [ones(H), mat(QD, H), mat(KD, H), mat(KD, H), ones(D), ones(D), mat(H, QD),
                  ones(H), mat(I, H), mat(I, H), mat(H, I)]
    layers = np.concatenate([p.ravel() for p in parts]).astype(np.float32)
    assert layers.size == layer_floats(cfg) * cfg.n_layers
    embed = mat(V, H)
    return {"embed": embed, "layers": layers, "final_norm": ones(H), "lm_head": embed}
