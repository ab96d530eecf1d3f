"""ctypes binding of ``libnwd.so`` (declared in ``include/nwd.h``).

The library is loaded from this package directory.  There is no fallback: if
the shared object is missing or fails to load, every call raises.
"""
from __future__ import annotations

import ctypes
import os
import re

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG_DIR, "libnwd.so")
HEADER_PATH = os.path.join(os.path.dirname(PKG_DIR), "include", "nwd.h")

NWD_OK = 0
NWD_ERR_INVALID = 1
NWD_ERR_RANGE = 2
NWD_ERR_UNSUPPORTED = 3
NWD_ERR_WORKSPACE = 4
NWD_ERR_CUDA = 5
NWD_ERR_NCCL = 6
NWD_ERR_TIMEOUT = 7
NWD_ERR_DEVICE = 8

NWD_DEVERR_PIPE_TIMEOUT = 1
NWD_DEVERR_ROW_RANGE = 2


class NwdError(RuntimeError):
    """A non-zero status from the library; ``str()`` is nwd_last_error()."""

    def __init__(self, status: int, message: str):
        super().__init__(message)
        self.status = status


_P = ctypes.c_void_p
_u32 = ctypes.c_uint32
_u64 = ctypes.c_uint64
_f32 = ctypes.c_float
_sz = ctypes.c_size_t

# name -> (restype, argtypes)
SIGNATURES = {
    "nwd_last_error": (ctypes.c_char_p, []),
    "nwd_version": (ctypes.c_char_p, []),
    "nwd_status_name": (ctypes.c_char_p, [ctypes.c_int]),
    "nwd_kv_append": (ctypes.c_int, [_P, _P, _u32, _u32, _u32, _u32, _P]),
    "nwd_kv_append_kv": (ctypes.c_int, [_P, _P, _P, _P, _u32, _u32, _u32, _u32, _P]),
    "nwd_kv_append_batched": (ctypes.c_int, [_P, _P, _P, _P, _u64, _P, _P, _u32, _u32, _u32,
                                             _P, _P]),
    "nwd_attn_decode_workspace_size": (ctypes.c_int, [_u32, _u32, _u32, _u32,
                                                      ctypes.POINTER(_sz)]),
    "nwd_workspace_init": (ctypes.c_int, [_P, _sz, _P]),
    "nwd_workspace_check": (ctypes.c_int, [_P, _sz, ctypes.POINTER(_u32), _P]),
    "nwd_attn_decode": (ctypes.c_int, [_P, _P, _P, _P, _u32, _u32, _u32, _u32, _u32, _f32, _P,
                                       _sz, _P]),
    "nwd_attn_decode_noalloc": (ctypes.c_int, [_P, _P, _P, _P, _u32, _u32, _u32, _u32, _u32,
                                               _f32, _P]),
    "nwd_noalloc_check": (ctypes.c_int, [ctypes.POINTER(_u32), _P]),
    "nwd_attn_decode_plan": (ctypes.c_int, [_u32, _u32, _u32, _u32, _u32] +
                             [ctypes.POINTER(ctypes.c_int)] * 5),
    "nwd_kv_append_attn_decode": (ctypes.c_int, [_P, _P, _P, _P, _P, _P, _u32, _u32, _u32, _u32,
                                                 _u32, _f32, _P, _sz, _P]),
    "nwd_attn_decode_batched": (ctypes.c_int, [_P, _P, _P, _u64, _P, _P, _P, _u32, _u32, _u32,
                                               _u32, _f32, _P, _sz, _P]),
    "nwd_kv_append_attn_decode_batched": (ctypes.c_int, [_P, _P, _P, _P, _P, _u64, _P, _P, _P,
                                                         _u32, _u32, _u32, _u32, _f32, _P, _sz,
                                                         _P]),
    "nwd_attn_decode_partial": (ctypes.c_int, [_P, _P, _P, _u64, _P, _P, _P, _P, _u32, _u32, _u32,
                                               _u32, _f32, _P, _sz, _P]),
    "nwd_attn_merge": (ctypes.c_int, [_P, _P, _P, _u32, _u32, _u32, _u32, _P]),
    "nwd_attn_merge_packed": (ctypes.c_int, [_P, _P, _u32, _u32, _u32, _u32, _P]),
    "nwd_q4_gemv": (ctypes.c_int, [_P, _P, _P, _P, _P, _u32, _u32, _u32, _u32, _P]),
    "nwd_prefetch_l2": (ctypes.c_int, [_P, _P, _u32, _P]),
    "nwd_selftest_wait_timeout": (ctypes.c_int, [_P, _sz, _P]),
    "nwd_q4_gemv_f16a": (ctypes.c_int, [_P, _P, _P, _P, _P, _u32, _u32, _u32, _u32, _P]),
    "nwd_q4_qkv_append": (ctypes.c_int, [_P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P,
                                         _u32, _u32, _u32, _u32, _u32, _u32, _P]),
    "nwd_fill_normal_f16": (ctypes.c_int, [_P, _u64, _u64, _u64, _P]),
    "nwd_kv_append_rows": (ctypes.c_int, [_P, _P, _P, _P, _u64, _P, _u32, _u32, _u32, _u32, _u32,
                                          _P, _sz, _P]),
    "nwd_attn_prefill": (ctypes.c_int, [_P, _P, _P, _u64, _P, _P, _u32, _u32, _u32, _u32, _u32,
                                        _u32, _f32, _P, _sz, _P]),
    "nwd_mgpu_unique_id": (ctypes.c_int, [_P]),
    "nwd_mgpu_init": (ctypes.c_int, [_P, ctypes.c_int, ctypes.c_int, ctypes.c_int, _u32, _u32,
                                     ctypes.POINTER(_P)]),
    "nwd_mgpu_workspace_size": (ctypes.c_int, [ctypes.c_int, _u32, _u32, _u32, _u32,
                                               ctypes.POINTER(_sz)]),
    "nwd_mgpu_decode_step": (ctypes.c_int, [_P, _P, _P, _P, _u64, _P, _P, _P, _u32, _u32, _u32,
                                            _u32, _f32, _P, _sz, _P]),
    "nwd_mgpu_sync": (ctypes.c_int, [_P]),
    "nwd_mgpu_set_timing": (ctypes.c_int, [_P, ctypes.c_int]),
    "nwd_mgpu_step_times": (ctypes.c_int, [_P, ctypes.POINTER(_f32), ctypes.POINTER(_f32)]),
    "nwd_mgpu_destroy": (ctypes.c_int, [_P]),
    "nwd_mgpu_abort": (ctypes.c_int, [_P]),
    "nwd_mgpu_nccl_version": (ctypes.c_int, [ctypes.POINTER(ctypes.c_int)]),
    "nwd_mgpu_exchange_mode": (ctypes.c_int, [_P, ctypes.POINTER(ctypes.c_int)]),
    "nwd_set_device": (ctypes.c_int, [ctypes.c_int]),
    "nwd_device_count": (ctypes.c_int, [ctypes.POINTER(ctypes.c_int)]),
    "nwd_alloc": (ctypes.c_int, [_sz, ctypes.POINTER(_P)]),
    "nwd_free": (ctypes.c_int, [_P]),
    "nwd_memcpy_h2d": (ctypes.c_int, [_P, _P, _sz, _P]),
    "nwd_memcpy_d2h": (ctypes.c_int, [_P, _P, _sz, _P]),
    "nwd_stream_create": (ctypes.c_int, [ctypes.POINTER(_P)]),
    "nwd_stream_destroy": (ctypes.c_int, [_P]),
    "nwd_stream_synchronize": (ctypes.c_int, [_P]),
}

_lib = None


def header_symbols(path: str = HEADER_PATH) -> list[str]:
    """Function names declared in include/nwd.h."""
    text = open(path).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return re.findall(r"^\s*(?:const\s+)?\w+\s*\*?\s*(nwd_\w+)\s*\(", text, flags=re.M)


def load():
    """Load libnwd.so (once).  Raises if it is missing: there is no fallback."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"{LIB_PATH} is missing: build it with __graft_entry__.build() "
            "(nvcc, sm_100a); this package has no CPU or PyTorch fallback")
    lib = ctypes.CDLL(LIB_PATH)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def check(status: int) -> None:
    if status != NWD_OK:
        lib = load()
        msg = lib.nwd_last_error().decode(errors="replace")
        name = lib.nwd_status_name(status).decode()
        raise NwdError(status, f"{name}: {msg}")


def call(name: str, *args) -> None:
    check(getattr(load(), name)(*args))


def version() -> str:
    return load().nwd_version().decode()
