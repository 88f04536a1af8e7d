"""ctypes view of include/ntb200.h: the C ABI exactly as a non-torch caller binds it.

Every function takes device pointers (ints), element counts and element strides, a
dtype code and a CUDA stream handle, and returns an NTB200 status (0 = ok).
``call(name, *args)`` raises ``NtB200Error`` with the library's status string and detail
for a non-zero status."""

from __future__ import annotations

import ctypes
from ctypes import c_char_p, c_float, c_int, c_int64, c_size_t, c_void_p
from pathlib import Path

LIBRARY = Path(__file__).resolve().parents[1] / "_lib" / "libntb200.so"

DTYPE_F32, DTYPE_BF16, DTYPE_F16, DTYPE_I32, DTYPE_I64 = 0, 1, 2, 3, 4
DEVERR_WAIT_TIMEOUT, DEVERR_INDEX_RANGE = 1, 2

# name -> (restype, argtypes); mirrors include/ntb200.h
SIGNATURES: dict[str, tuple[object, list[object]]] = {
    "ntb200_version": (c_int, []),
    "ntb200_status_string": (c_char_p, [c_int]),
    "ntb200_last_error": (c_char_p, []),
    "ntb200_read_device_error": (c_int, [ctypes.POINTER(c_int), c_void_p]),
    "ntb200_rms_norm": (
        c_int,
        [c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64, c_int64, c_float, c_int, c_void_p],
    ),
    "ntb200_fused_add_rms_norm": (
        c_int,
        [c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64, c_int64, c_int64,
         c_float, c_int, c_void_p],
    ),
    "ntb200_gemma_rms_norm": (
        c_int,
        [c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64, c_int64, c_float, c_int, c_void_p],
    ),
    "ntb200_gemma_fused_add_rms_norm": (
        c_int,
        [c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64, c_int64, c_int64,
         c_float, c_int, c_void_p],
    ),
    "ntb200_silu_and_mul": (
        c_int, [c_void_p, c_void_p, c_int64, c_int64, c_int64, c_int64, c_int, c_void_p]
    ),
    "ntb200_rotary_embedding_neox": (
        c_int,
        [c_void_p, c_int, c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64, c_int64,
         c_int64, c_int64, c_int64, c_int64, c_int64, c_int64, c_int64, c_int, c_void_p],
    ),
    "ntb200_reshape_and_cache": (
        c_int,
        [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int64, c_int64, c_int64,
         c_int64, c_int64, c_int64, c_int64, c_int64, c_int64, c_int64, c_int64, c_int64, c_int,
         c_void_p],
    ),
    "ntb200_rope_and_cache": (
        c_int,
        [c_void_p, c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int]
        + [c_int64] * 19 + [c_int, c_void_p],
    ),
    "ntb200_embedding": (
        c_int,
        [c_void_p, c_void_p, c_int, c_void_p, c_int64, c_int64, c_int64, c_int64, c_int64, c_int,
         c_void_p],
    ),
    "ntb200_paged_attention_decode_workspace_size": (
        c_size_t, [c_int64, c_int64, c_int64, c_int64, c_int64, c_int64]
    ),
    "ntb200_paged_attention_decode": (
        c_int,
        [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64,
         c_int64, c_int64, c_int64, c_int64, c_int64, c_int64, c_float, c_int64, c_int64,
         c_int64, c_int64, c_int64, c_int64, c_int64, c_void_p, c_size_t, c_int, c_void_p],
    ),
    "ntb200_paged_attention_prefill": (
        c_int,
        [c_void_p] * 7 + [c_int64] * 10 + [c_float, c_int] + [c_int64] * 7 + [c_int, c_void_p],
    ),
    "ntb200_paged_attention_decode_varlen": (
        c_int,
        [c_void_p] * 7 + [c_int64] * 9 + [c_float] + [c_int64] * 7 + [c_void_p, c_size_t, c_int, c_void_p],
    ),
    "ntb200_paged_attention_varlen": (
        c_int,
        [c_void_p] * 7 + [c_int64] * 11 + [c_float] + [c_int64] * 7 + [c_void_p, c_size_t, c_int, c_void_p],
    ),
    "ntb200_flash_attn_varlen": (
        c_int,
        [c_void_p] * 6 + [c_int64] * 7 + [c_float, c_int] + [c_int64] * 8 + [c_int, c_void_p],
    ),
    "ntb200_paged_attention_decode_noalloc": (
        c_int,
        [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64,
         c_int64, c_int64, c_int64, c_int64, c_int64, c_int64, c_float, c_int64, c_int64,
         c_int64, c_int64, c_int64, c_int64, c_int64, c_int, c_void_p],
    ),
    "ntb200_linear_workspace_size": (c_size_t, [c_int64, c_int64, c_int64]),
    "ntb200_linear": (
        c_int,
        [c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64, c_int64, c_int64,
         c_int64, c_void_p, c_size_t, c_int, c_void_p],
    ),
    "ntb200_linear_silu_and_mul": (
        c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64, c_int64, c_int64, c_int64, c_int, c_void_p]
    ),
    "ntb200_rms_norm_linear": (
        c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_float, c_void_p, c_int64, c_int64, c_int64,
                c_int64, c_int64, c_int64, c_int64, c_int64, c_int, c_void_p]
    ),
    "ntb200_linear_argmax_workspace_size": (c_size_t, [c_int64, c_int64, c_int64]),
    "ntb200_linear_argmax": (
        c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64, c_int64, c_int64, c_void_p, c_size_t,
                c_int, c_void_p]
    ),
    "ntb200_top_k_top_p": (c_int, [c_void_p, c_int64, c_int64, c_int64, c_void_p, c_int, c_void_p, c_void_p]),
    "ntb200_random_sample": (
        c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64, c_int64, c_void_p]
    ),
    "ntb200_allreduce_buffer_size": (c_size_t, [c_int64, c_int, c_int]),
    "ntb200_allreduce_oneshot": (
        c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int, c_int, c_int, c_void_p]
    ),
    "ntb200_allreduce_twoshot": (
        c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int, c_int, c_int, c_void_p]
    ),
}


class NtB200Error(RuntimeError):
    def __init__(self, name: str, status: int, detail: str):
        super().__init__(f"{name} -> {status}: {detail}")
        self.status = status


_lib: ctypes.CDLL | None = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not LIBRARY.exists():
            raise RuntimeError(f"{LIBRARY} is not built; run `python vllm-nt_b200/csrc/build.py`")
        handle = ctypes.CDLL(str(LIBRARY))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _lib = handle
    return _lib


def call(name: str, *args) -> int:
    status = getattr(lib(), name)(*args)
    if status != 0:
        detail = lib().ntb200_last_error().decode(errors="replace")
        status_str = lib().ntb200_status_string(status).decode()
        raise NtB200Error(name, status, f"{status_str}: {detail}")
    return status


def read_device_error(stream: int = 0) -> int:
    word = c_int(0)
    call("ntb200_read_device_error", ctypes.byref(word), c_void_p(stream))
    return word.value
