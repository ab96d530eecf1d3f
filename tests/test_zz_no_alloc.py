"""nwd_attn_decode_noalloc: decode attention with no caller workspace.

Some hosts of this library cannot allocate device memory for it: a JavaScript
engine that hands an addon the GPU buffers it already owns, or an embedder
whose memory is budgeted up front, has no allocator to give the library a
workspace.  For them the library offers one entry point whose scratch is a
fixed array inside the library.  These tests call it through the C ABI and
compare it with nwd_attn_decode (caller workspace) and with the CPU oracle on
the same inputs.  Consecutive calls share that scratch, so one test makes two
calls in a row that both use it (more than 2048 rows, different shapes), and
reads its device error word afterwards through nwd_noalloc_check.

This file is collected last on purpose (its name sorts after the others).
"""
from __future__ import annotations

import ctypes
import importlib

import pytest
import torch

from devutil import to_dev, vals
from tolerance import assert_attn_close

pytestmark = pytest.mark.gpu

PKG = "nemotron-webgpu-decode_b200"


def _noalloc(lib, q, k, v, o, nh, nkv, hd, seq, cap):
    stream = torch.cuda.current_stream().cuda_stream
    return lib.nwd_attn_decode_noalloc(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(),
                                       nh, nkv, hd, seq, cap, ctypes.c_float(0.0), stream)


def _check(lib) -> int:
    err = ctypes.c_uint32(0xFFFFFFFF)
    st = lib.nwd_noalloc_check(ctypes.byref(err), torch.cuda.current_stream().cuda_stream)
    assert st == 0, lib.nwd_last_error()
    return err.value


# Each sequence of calls runs in one test: the first two use the scratch
# (split-KV path), the last runs on the short path (no scratch) in between or
# after, so a stale ticket or header left by one call would show in the next.
@pytest.mark.parametrize("calls", [
    [(40, 8, 20000), (32, 8, 70000), (40, 8, 151)],
    [(32, 8, 151), (32, 4, 9000), (40, 8, 33000)],
])
def test_noalloc_matches_workspace_entry_point_and_oracle(oracle, calls):
    _lib = importlib.import_module(PKG + "._lib")
    ops = importlib.import_module(PKG + ".ops")
    lib = _lib.load()
    hd = 128
    for call, (nh, nkv, L) in enumerate(calls):
        qb = oracle.normal_f16(nh * hd, 7 + call)
        kb = oracle.normal_f16(L * nkv * hd, 8 + call)
        vb = oracle.normal_f16(L * nkv * hd, 9 + call)
        q, k, v = to_dev(qb, (nh, hd)), to_dev(kb, (L, nkv, hd)), to_dev(vb, (L, nkv, hd))
        o_ref = torch.empty(nh, hd, dtype=torch.float16, device="cuda")
        ops.attention(q, k, v, o_ref, ops.AttnParams(nh, nkv, hd, L))
        o = torch.full((nh, hd), 5.0, dtype=torch.float16, device="cuda")
        st = _noalloc(lib, q, k, v, o, nh, nkv, hd, L, L)
        assert st == 0, lib.nwd_last_error()
        torch.cuda.synchronize()
        what = f"call {call}: Hq={nh} Hkv={nkv} L={L}"
        ref = oracle.attention(qb, kb, vb, nh, nkv, hd, L)
        assert_attn_close(vals(o), ref, what + " vs oracle")
        assert_attn_close(vals(o), vals(o_ref), what + " vs nwd_attn_decode")
        assert _check(lib) == 0, what


def test_noalloc_rejects_shapes_beyond_its_scratch():
    _lib = importlib.import_module(PKG + "._lib")
    lib = _lib.load()
    t = torch.zeros(16, dtype=torch.float16, device="cuda")
    # 128 kv heads need more merge tickets than the built-in scratch holds
    st = _noalloc(lib, t, t, t, t, 128, 128, 128, 1, 1)
    assert st == _lib.NWD_ERR_UNSUPPORTED
    assert b"built-in scratch" in lib.nwd_last_error()
    assert _check(lib) == 0
