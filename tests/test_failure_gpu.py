"""Failure detection on the GPU without a fault: a bounded device wait is made to run
out (a barrier that nothing completes), the kernel returns, the host reads the status
from the workspace's error word, and the context stays usable."""
from __future__ import annotations

import time

import pytest
import torch

from devutil import to_dev, vals
from tolerance import assert_attn_close

pytestmark = pytest.mark.gpu


def test_device_wait_runs_out_and_reports(ops, oracle):
    from importlib import import_module
    _lib = import_module(ops.__name__.rsplit(".", 1)[0] + "._lib")
    ws = ops.Workspace(1, 8, 2, 128)
    assert ws.check() == 0
    t0 = time.monotonic()
    err = ops.selftest_wait_timeout(ws)
    elapsed = time.monotonic() - t0
    assert err == _lib.NWD_DEVERR_PIPE_TIMEOUT, err
    assert 1.0 < elapsed < 30.0, elapsed  # the 2 s device limit, not a hang
    assert ws.check() == 0  # the check cleared the word
    # the same stream and workspace serve an ordinary call afterwards
    nh, nkv, hd, L = 8, 2, 128, 3000
    q = oracle.normal_f16(nh * hd, 81)
    k = oracle.normal_f16(L * nkv * hd, 82)
    v = oracle.normal_f16(L * nkv * hd, 83)
    o = torch.empty(nh, hd, dtype=torch.float16, device="cuda")
    ops.attention(to_dev(q, (nh, hd)), to_dev(k, (L, nkv, hd)), to_dev(v, (L, nkv, hd)), o,
                  ops.AttnParams(nh, nkv, hd, L), workspace=ws)
    assert_attn_close(vals(o), oracle.attention(q, k, v, nh, nkv, hd, L), "after the timeout")
    assert ws.check() == 0
