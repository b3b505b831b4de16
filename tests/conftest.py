import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
TESTS = os.path.dirname(os.path.abspath(__file__))
for p in (ROOT, TESTS):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (runs through libsa_cuda.so on cuda:0)")


def _has_gpu() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


HAS_GPU = _has_gpu()


def pytest_collection_modifyitems(config, items):
    if HAS_GPU:
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for it in items:
        if "gpu" in it.keywords:
            it.add_marker(skip)


@pytest.fixture(scope="session")
def oracle():
    from oracle.oracle import Oracle
    return Oracle()


@pytest.fixture(scope="session")
def reference():
    from oracle.oracle import REF_SO, Reference
    if not os.path.exists(REF_SO):
        pytest.skip("oracle/_ref/libsa_ref.so not built (needs the reference tree)")
    return Reference()


@pytest.fixture(scope="session")
def ctx():
    from streaming_attention_b200 import Context
    c = Context(0)
    yield c
    c.close()


def golden(name: str):
    import numpy as np
    return np.load(os.path.join(TESTS, "golden", name))
