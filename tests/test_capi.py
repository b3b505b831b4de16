"""The C-ABI library loads and exports every symbol include/*.h declares; host
side argument checking works without a GPU.  CPU only."""
import ctypes as C
import glob
import os
import re

import pytest

from conftest import HAS_GPU, ROOT


def _declared():
    names = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        src = open(h).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        names |= set(re.findall(r"\b(sa_[a-z0-9_]+)\s*\(", src))
    return sorted(names)


def test_header_declares_entry_points():
    names = _declared()
    assert "sa_attn_decode" in names and "sa_ctx_create" in names


def test_library_exports_every_declared_symbol():
    from streaming_attention_b200._capi import LIB_PATH, SIGNATURES
    L = C.CDLL(LIB_PATH)
    missing = [n for n in _declared() if not hasattr(L, n)]
    assert not missing, f"declared in include/ but not exported: {missing}"
    # and the Python binding knows the signature of each one
    assert set(_declared()) <= set(SIGNATURES), set(_declared()) - set(SIGNATURES)


def test_version_and_error_strings():
    from streaming_attention_b200 import lib
    assert b"sm_100a" in lib().sa_version()
    assert isinstance(lib().sa_last_error(), bytes)


@pytest.mark.skipif(HAS_GPU, reason="checks the no-GPU error path")
def test_ctx_create_without_gpu_reports_error():
    from streaming_attention_b200 import Context, SAError
    with pytest.raises(SAError) as e:
        Context(0)
    assert e.value.code in (-1, -2)


def test_null_ctx_is_an_argument_error():
    from streaming_attention_b200 import lib
    assert lib().sa_attn_decode(None, 0, None, None, None, 0, 1, 128, 1, 1, 64, 1.0, None, 0) == -1
    assert b"ctx is NULL" in lib().sa_last_error()
    assert lib().sa_ctx_synchronize(None) == -1
