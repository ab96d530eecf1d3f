"""The C-ABI library loads and exports every symbol include/nwd.h declares.

These checks make no compute call, so they run without a GPU.  Argument
checks that fail before any CUDA call (range, null pointers) are exercised
too: they must return their status without launching anything.
"""
from __future__ import annotations

import ctypes

import pytest


def test_library_exports_header_symbols(nwd):
    from importlib import import_module
    _lib = import_module(nwd.__name__ + "._lib")
    syms = _lib.header_symbols()
    assert len(syms) >= 15
    lib = _lib.load()
    missing = [s for s in syms if not hasattr(lib, s)]
    assert not missing, missing
    # every declared symbol has a ctypes signature, and vice versa
    assert set(syms) == set(_lib.SIGNATURES), set(syms) ^ set(_lib.SIGNATURES)


def test_version_and_status_names(nwd):
    from importlib import import_module
    _lib = import_module(nwd.__name__ + "._lib")
    lib = _lib.load()
    assert "sm_100a" in nwd.version()
    assert lib.nwd_status_name(0) == b"NWD_OK"
    assert lib.nwd_status_name(2) == b"NWD_ERR_RANGE"
    assert lib.nwd_status_name(99) == b"NWD_ERR_UNKNOWN"


def test_range_error_before_launch(nwd):
    """seq >= maxSeq fails like engine/runtime.js:448, with no CUDA call."""
    from importlib import import_module
    _lib = import_module(nwd.__name__ + "._lib")
    lib = _lib.load()
    dummy = ctypes.c_void_p(16)
    st = lib.nwd_kv_append(dummy, dummy, 256, 8, 128, 256, None)
    assert st == _lib.NWD_ERR_RANGE
    assert lib.nwd_last_error() == b"seq 256 exceeds maxSeq 256"
    st = lib.nwd_kv_append_attn_decode(dummy, dummy, dummy, dummy, dummy, dummy, 40, 8, 128, 300,
                                       256, 0.0, dummy, 1 << 20, None)
    assert st == _lib.NWD_ERR_RANGE
    assert b"exceeds maxSeq" in lib.nwd_last_error()
    with pytest.raises(_lib.NwdError, match="seq 256 exceeds maxSeq 256"):
        _lib.check(lib.nwd_kv_append(dummy, dummy, 256, 8, 128, 256, None))


def test_null_pointer_errors(nwd):
    from importlib import import_module
    _lib = import_module(nwd.__name__ + "._lib")
    lib = _lib.load()
    assert lib.nwd_kv_append(None, None, 0, 8, 128, 256, None) == _lib.NWD_ERR_INVALID
    assert lib.nwd_attn_merge(None, None, None, 1, 1, 1, 128, None) == _lib.NWD_ERR_INVALID
    assert lib.nwd_workspace_init(None, 0, None) == _lib.NWD_ERR_WORKSPACE
    v = ctypes.c_uint32()
    assert lib.nwd_workspace_check(None, 0, ctypes.byref(v), None) == _lib.NWD_ERR_WORKSPACE
    assert lib.nwd_attn_decode_workspace_size(1, 40, 8, 128, None) == _lib.NWD_ERR_INVALID


def test_shape_errors_before_launch(nwd):
    from importlib import import_module
    _lib = import_module(nwd.__name__ + "._lib")
    lib = _lib.load()
    sz = ctypes.c_size_t()
    # group not integral, head_dim unsupported, group too large: all rejected
    # before the device is queried
    assert lib.nwd_attn_decode_workspace_size(1, 40, 7, 128, ctypes.byref(sz)) == _lib.NWD_ERR_INVALID
    assert lib.nwd_attn_decode_workspace_size(1, 40, 8, 64, ctypes.byref(sz)) == _lib.NWD_ERR_UNSUPPORTED
    assert lib.nwd_attn_decode_workspace_size(1, 32, 2, 128, ctypes.byref(sz)) == _lib.NWD_ERR_UNSUPPORTED


def test_ops_reject_cpu_tensors(ops):
    import torch
    src = torch.zeros(1024, dtype=torch.float16)
    cache = torch.zeros(256, 8, 128, dtype=torch.float16)
    with pytest.raises(ValueError, match="CUDA tensor"):
        ops.kv_append(src, cache, ops.KvParams(0, 8, 128))


def test_prefetch_argument_errors_before_launch(nwd):
    """nwd_prefetch_l2 refuses more than 16 ranges and null pointers before any CUDA
    call; zero ranges (or only empty ones) is a no-op."""
    from importlib import import_module
    _lib = import_module(nwd.__name__ + "._lib")
    lib = _lib.load()
    ptrs = (ctypes.c_void_p * 17)(*([16] * 17))
    sizes = (ctypes.c_uint64 * 17)(*([64] * 17))
    assert lib.nwd_prefetch_l2(ptrs, sizes, 17, None) == _lib.NWD_ERR_INVALID
    assert b"at most 16" in lib.nwd_last_error()
    assert lib.nwd_prefetch_l2(None, None, 2, None) == _lib.NWD_ERR_INVALID
    null = (ctypes.c_void_p * 1)(None)
    assert lib.nwd_prefetch_l2(null, sizes, 1, None) == _lib.NWD_ERR_INVALID
    assert lib.nwd_prefetch_l2(None, None, 0, None) == _lib.NWD_OK
    empty = (ctypes.c_uint64 * 1)(0)
    assert lib.nwd_prefetch_l2(null, empty, 1, None) == _lib.NWD_OK


def test_mgpu_entry_points_before_any_device(nwd):
    """The multi-GPU entry points load NCCL at run time: a communicator id is made
    without a GPU, and argument errors come back before any CUDA or NCCL call."""
    from importlib import import_module
    _lib = import_module(nwd.__name__ + "._lib")
    lib = _lib.load()
    uid = (ctypes.c_uint8 * 128)()
    assert lib.nwd_mgpu_unique_id(uid) == _lib.NWD_OK, lib.nwd_last_error()
    assert any(bytes(uid))
    ver = ctypes.c_int(0)
    assert lib.nwd_mgpu_nccl_version(ctypes.byref(ver)) == _lib.NWD_OK
    assert ver.value >= 21400  # ncclCommInitRankConfig and non-blocking communicators
    h = ctypes.c_void_p()
    assert lib.nwd_mgpu_init(uid, 2, 2, 0, 1000, 1000, ctypes.byref(h)) == _lib.NWD_ERR_INVALID
    assert b"rank 2 outside world 2" in lib.nwd_last_error()
    assert lib.nwd_mgpu_init(uid, 2, 0, 0, 0, 1000, ctypes.byref(h)) == _lib.NWD_ERR_INVALID
    assert lib.nwd_mgpu_init(None, 2, 0, 0, 1, 1, ctypes.byref(h)) == _lib.NWD_ERR_INVALID
    assert lib.nwd_mgpu_sync(None) == _lib.NWD_ERR_INVALID
    assert lib.nwd_mgpu_destroy(None) == _lib.NWD_OK
    assert lib.nwd_mgpu_workspace_size(0, 1, 32, 8, 128, ctypes.byref(ctypes.c_size_t())) == \
        _lib.NWD_ERR_INVALID
    p = ctypes.c_void_p(1)
    assert lib.nwd_alloc(0, ctypes.byref(p)) == _lib.NWD_OK and not p.value
    assert lib.nwd_free(None) == _lib.NWD_OK
    assert lib.nwd_memcpy_h2d(None, None, 16, None) == _lib.NWD_ERR_INVALID


def test_cpp_host_links_only_the_library(nwd):
    """nwd_host (the C++ engine host) needs libnwd.so and the C/C++ runtime only: no
    Python, no PyTorch, no separate CUDA runtime."""
    import os
    import subprocess
    pkg = os.path.dirname(nwd.__file__)
    host = os.path.join(pkg, "nwd_host")
    assert os.path.exists(host)
    deps = subprocess.run(["ldd", host], capture_output=True, text=True).stdout
    assert os.path.join(pkg, "libnwd.so") in deps
    assert "torch" not in deps and "python" not in deps and "libcudart" not in deps
    p = subprocess.run([host], capture_output=True, text=True)
    assert p.returncode == 2 and "usage" in p.stderr
