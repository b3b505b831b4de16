"""ctypes declarations of the C ABI in include/sa_cuda.h."""
from __future__ import annotations

import ctypes as C
import os
import threading

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libsa_cuda.so")

SA_OK = 0
SA_ERR_ARG = -1
SA_ERR_CUDA = -2
SA_ERR_OOM = -3
SA_ERR_TIMEOUT = -4
SA_ERR_NCCL = -5
SA_ERR_RANGE = -6
SA_ERR_FULL = -7

SA_SP_HANDLE_BYTES = 128
SA_SPP_HANDLE_BYTES = 128

SA_F32 = 0
SA_BF16 = 1
SA_HOST_PTRS = 1
SA_KV_STATIC = 2

_vp = C.c_void_p
_fp = C.POINTER(C.c_float)

# (name, restype, argtypes) for every entry point of include/sa_cuda.h
SIGNATURES = {
    "sa_last_error": (C.c_char_p, []),
    "sa_version": (C.c_char_p, []),
    "sa_device_count": (C.c_int, [C.POINTER(C.c_int)]),
    "sa_ctx_create": (C.c_int, [C.c_int, C.POINTER(_vp)]),
    "sa_ctx_destroy": (C.c_int, [_vp]),
    "sa_ctx_set_stream": (C.c_int, [_vp, _vp]),
    "sa_ctx_stream": (_vp, [_vp]),
    "sa_ctx_synchronize": (C.c_int, [_vp]),
    "sa_ctx_num_sms": (C.c_int, [_vp]),
    "sa_attn_decode": (C.c_int, [_vp, C.c_int, _vp, _vp, _vp, C.c_longlong, C.c_int, C.c_int,
                                 C.c_int, C.c_int, C.c_int, C.c_float, _vp, C.c_uint]),
    "sa_attn_decode_partial": (C.c_int, [_vp, C.c_int, _vp, _vp, _vp, C.c_longlong, C.c_int,
                                         C.c_int, C.c_int, C.c_int, C.c_int, C.c_float, _vp, _vp,
                                         _vp, C.c_uint]),
    "sa_attn_merge": (C.c_int, [_vp, C.c_int, C.c_int, C.c_int, _vp, _vp, _vp, _vp, _vp, _vp,
                                C.c_uint]),
    "sa_attn_decode_step": (C.c_int, [_vp, C.c_int, _vp, _vp, _vp, _vp, _vp, C.c_int, C.c_int,
                                      C.c_int, C.c_int, C.c_int, C.c_int, C.c_float, _vp, C.c_uint]),
    "sa_attn_prefill": (C.c_int, [_vp, _vp, _vp, _vp, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int,
                                  C.c_int, C.c_longlong, C.c_longlong, C.c_float, _vp, C.c_int,
                                  C.c_longlong, C.c_uint]),
    "sa_qwen3_create": (C.c_int, [_vp, _vp, C.POINTER(_vp)]),
    "sa_safetensors_inspect": (C.c_int, [C.c_char_p, _vp]),
    "sa_qwen3_load_safetensors": (C.c_int, [_vp, C.c_char_p, C.c_int, C.c_float, C.c_float, C.POINTER(_vp)]),
    "sa_qwen3_create_tp": (C.c_int, [_vp, _vp, C.c_int, C.c_int, C.POINTER(_vp)]),
    "sa_qwen3_load_safetensors_tp": (C.c_int, [_vp, C.c_char_p, C.c_int, C.c_float, C.c_float, C.c_int, C.c_int,
                                               C.POINTER(_vp)]),
    "sa_qwen3_tp_handle": (C.c_int, [_vp, _vp]),
    "sa_qwen3_tp_connect": (C.c_int, [_vp, _vp]),
    "sa_qwen3_create_sp": (C.c_int, [_vp, _vp, C.c_int, C.c_int, C.POINTER(_vp)]),
    "sa_qwen3_load_safetensors_sp": (C.c_int, [_vp, C.c_char_p, C.c_int, C.c_float, C.c_float, C.c_int, C.c_int,
                                               C.POINTER(_vp)]),
    "sa_qwen3_sp_handle": (C.c_int, [_vp, _vp]),
    "sa_qwen3_sp_connect": (C.c_int, [_vp, _vp]),
    "sa_qwen3_destroy": (C.c_int, [_vp]),
    "sa_qwen3_set_embed": (C.c_int, [_vp, _fp, _fp, _fp]),
    "sa_qwen3_set_layer": (C.c_int, [_vp, C.c_int] + [_fp] * 11),
    "sa_qwen3_reset": (C.c_int, [_vp]),
    "sa_qwen3_cache_len": (C.c_int, [_vp]),
    "sa_qwen3_read_kv": (C.c_int, [_vp, C.c_int, _vp, _vp, C.c_int]),
    "sa_qwen3_write_kv": (C.c_int, [_vp, C.c_int, _vp, _vp, C.c_int, C.c_int]),
    "sa_qwen3_set_cache_len": (C.c_int, [_vp, C.c_int]),
    "sa_qwen3_forward": (C.c_int, [_vp, C.POINTER(C.c_int64), C.c_int, C.c_int, _fp, C.c_int,
                                   C.c_uint]),
    "sa_qwen3_generate": (C.c_int, [_vp, C.POINTER(C.c_int64), C.c_int, C.c_int,
                                    C.POINTER(C.c_int64), C.c_uint]),
    "sa_attn_prompt_f32": (C.c_int, [_vp, _vp, _vp, _vp, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int,
                                     C.c_int, C.c_int, C.c_longlong, C.c_longlong, C.c_float, _vp,
                                     C.c_longlong, C.c_uint]),
    "sa_sp_create": (C.c_int, [_vp, C.c_int, C.c_int, C.c_int, C.c_int, C.POINTER(_vp)]),
    "sa_sp_handle": (C.c_int, [_vp, _vp]),
    "sa_sp_connect": (C.c_int, [_vp, _vp]),
    "sa_sp_connect_local": (C.c_int, [C.POINTER(_vp), C.c_int]),
    "sa_sp_destroy": (C.c_int, [_vp]),
    "sa_spp_create": (C.c_int, [_vp, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.POINTER(_vp)]),
    "sa_spp_handle": (C.c_int, [_vp, _vp]),
    "sa_spp_connect": (C.c_int, [_vp, _vp]),
    "sa_spp_connect_local": (C.c_int, [C.POINTER(_vp), C.c_int]),
    "sa_spp_destroy": (C.c_int, [_vp]),
    "sa_spp_prefill": (C.c_int, [_vp, _vp, _vp, _vp, C.c_int, C.c_int, C.c_int, C.c_int, C.c_float, _vp,
                                 C.c_int, C.c_uint]),
    "sa_attn_decode_sp": (C.c_int, [_vp, C.c_int, _vp, _vp, _vp, C.c_longlong, C.c_int, C.c_int,
                                    C.c_int, C.c_int, C.c_int, C.c_float, _vp, _vp, _vp, C.c_uint]),
    "sa_attn_decode_noalloc": (C.c_int, [_vp, C.c_int, _vp, _vp, _vp, C.c_longlong, C.c_int,
                                         C.c_int, C.c_int, C.c_int, C.c_int, C.c_float, _vp]),
}


class SAError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"[{code}] {msg}")
        self.code = code


_lib = None
_lock = threading.Lock()


def lib() -> C.CDLL:
    """Load libsa_cuda.so (raises if it has not been built)."""
    global _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise ImportError(
                    f"{LIB_PATH} is missing: build it with `make -C streaming_attention_b200` "
                    "(or __graft_entry__.build()); there is no CPU fallback")
            L = C.CDLL(LIB_PATH)
            for name, (res, args) in SIGNATURES.items():
                f = getattr(L, name)
                f.restype = res
                f.argtypes = args
            _lib = L
    return _lib


def check(rc: int) -> None:
    if rc != SA_OK:
        raise SAError(rc, lib().sa_last_error().decode())


class Context:
    """One sa_ctx: a GPU, a stream and the library's scratch on that GPU."""

    def __init__(self, device: int = 0):
        self.device = device
        h = _vp()
        check(lib().sa_ctx_create(device, C.byref(h)))
        self.h = h

    def close(self) -> None:
        if getattr(self, "h", None):
            lib().sa_ctx_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    @property
    def stream(self) -> int:
        return lib().sa_ctx_stream(self.h) or 0

    def set_stream(self, stream_ptr: int | None) -> None:
        check(lib().sa_ctx_set_stream(self.h, stream_ptr))

    def synchronize(self) -> None:
        check(lib().sa_ctx_synchronize(self.h))

    @property
    def num_sms(self) -> int:
        return lib().sa_ctx_num_sms(self.h)


_default: dict[int, Context] = {}


def default_context(device: int = 0) -> Context:
    if device not in _default:
        _default[device] = Context(device)
    return _default[device]
