"""streaming_attention_b200 -- B200-native (sm_100a) streaming attention.

Python view of ``libsa_cuda.so`` (declared in ``include/sa_cuda.h``) through
ctypes.  The functions mirror the reference's operator interface for the hot
path, with the same names and argument meaning as ``attention/src/attention.h``
(``streaming_attention_*``, ``naive_attention_*``) and
``tensor_cpp/include/tensor_cpp/ops.h``.  Every call goes to the CUDA library;
there is no CPU path, and importing fails loudly if the library is missing.
"""
from ._capi import (  # noqa: F401
    LIB_PATH,
    SA_BF16,
    SA_F32,
    SA_HOST_PTRS,
    Context,
    SAError,
    lib,
)
from .attention import (  # noqa: F401
    attn_decode,
    attn_decode_partial,
    attn_decode_step,
    attn_merge,
    attn_prefill,
    attn_prompt_f32,
    naive_attention_cuda,
    streaming_attention_cuda,
    streaming_attention_mpi_cuda,
)

from .qwen3 import QWEN3_0_6B, Qwen3, Qwen3Config  # noqa: F401

__all__ = [
    "Context", "SAError", "lib", "LIB_PATH", "SA_F32", "SA_BF16", "SA_HOST_PTRS",
    "attn_decode", "attn_decode_partial", "attn_decode_step", "attn_merge", "attn_prefill", "attn_prompt_f32", "streaming_attention_cuda",
    "naive_attention_cuda", "streaming_attention_mpi_cuda", "Qwen3", "Qwen3Config", "QWEN3_0_6B",
]
