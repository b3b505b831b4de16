"""Seeded synthetic inputs shared by the golden-fixture generator, the tests and
bench.py.  Every array is derived from numpy's PCG64 generator, so the same
seed gives the same bytes here and on the GPU box (same image)."""
from __future__ import annotations

import hashlib

import numpy as np

# Shapes of the golden single-query cases: the reference's own unit test sweeps
# T in {512..4096} and d in {64, 128, 256} with block 64
# (tensor_cpp/tests/unit/test_streaming_attention.cpp:65-108); ragged T (not a
# multiple of the block), T < block and T = 1 are added edge cases.
SINGLE_CASES = [(512, 64), (1000, 128), (4096, 256), (8192, 128), (1, 128), (63, 128), (2049, 64)]
GQA_CASES = [  # (hq, hkv, T, d)
    (16, 8, 2048, 128), (16, 8, 777, 128), (4, 4, 300, 64), (8, 2, 1500, 64), (4, 2, 513, 256)]
PREFILL_CASES = [  # (S, hq, hkv, d)
    (200, 4, 2, 128), (130, 2, 1, 128), (70, 2, 2, 128)]


def rng(seed: int) -> np.random.Generator:
    return np.random.default_rng(seed)


def normal(seed: int, shape) -> np.ndarray:
    return rng(seed).standard_normal(shape, dtype=np.float32)


def single_query(T: int, d: int, seed: int):
    g = rng(seed)
    q = g.standard_normal(d, dtype=np.float32)
    k = g.standard_normal((T, d), dtype=np.float32)
    v = g.standard_normal((T, d), dtype=np.float32)
    return q, k, v


def gqa(hq: int, hkv: int, T: int, d: int, seed: int):
    g = rng(seed)
    q = g.standard_normal((hq, d), dtype=np.float32)
    k = g.standard_normal((hkv, T, d), dtype=np.float32)
    v = g.standard_normal((hkv, T, d), dtype=np.float32)
    return q, k, v


def prefill(S: int, hq: int, hkv: int, d: int, seed: int):
    g = rng(seed)
    q = g.standard_normal((S, hq, d), dtype=np.float32)
    k = g.standard_normal((S, hkv, d), dtype=np.float32)
    v = g.standard_normal((S, hkv, d), dtype=np.float32)
    return q, k, v


def digest(*arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()[:16]
