"""Causal prefill on tcgen05 (nwd_attn_prefill) and the multi-row kv_append path,
against the oracle: the reference computes a prompt one decode step per token
(engine/runtime.js:640-643), so token i of a chunk attends rows 0..start_pos+i."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from devutil import bits, to_dev, vals
from tolerance import assert_attn_close

pytestmark = pytest.mark.gpu


def _case(ops, oracle, batch, n_q, start_pos, nh, nkv, seed, extra=0):
    hd = 128
    rows_per = start_pos + n_q + extra
    rows = batch * rows_per
    offs = np.arange(batch, dtype=np.int64) * rows_per
    kp = oracle.normal_f16(rows * nkv * hd, seed).reshape(rows, nkv, hd)
    vp = oracle.normal_f16(rows * nkv * hd, seed + 1).reshape(rows, nkv, hd)
    kc = oracle.normal_f16(batch * n_q * nkv * hd, seed + 2).reshape(batch, n_q, nkv, hd)
    vc = oracle.normal_f16(batch * n_q * nkv * hd, seed + 3).reshape(batch, n_q, nkv, hd)
    q = oracle.normal_f16(batch * n_q * nh * hd, seed + 4).reshape(batch, n_q, nh, hd)
    dk, dv = to_dev(kp), to_dev(vp)
    ro = torch.tensor(offs, device="cuda")
    # the chunk's K/V through the kv_append path, then attention
    ops.kv_append_rows(to_dev(kc), to_dev(vc), dk, dv, ro, start_pos)
    o = torch.full((batch, n_q, nh, hd), 9.0, dtype=torch.float16, device="cuda")
    ops.attention_prefill(to_dev(q), dk, dv, ro, o, start_pos, nh, nkv, hd)
    for b in range(batch):
        kp[offs[b] + start_pos: offs[b] + start_pos + n_q] = kc[b]
        vp[offs[b] + start_pos: offs[b] + start_pos + n_q] = vc[b]
    assert np.array_equal(bits(dk), kp) and np.array_equal(bits(dv), vp)
    ref = oracle.attention_prefill(q, kp, vp, offs, n_q, start_pos, nh, nkv, hd)
    return vals(o), ref


@pytest.mark.parametrize("batch,n_q,start_pos,nh,nkv", [
    (1, 128, 0, 4, 1),     # one tile, diagonal block only
    (2, 200, 0, 8, 2),     # a partial second tile
    (1, 256, 300, 8, 2),   # chunk after 300 cached rows: unaligned key blocks
    (2, 129, 0, 40, 8),    # engine shape, group 5
    (1, 1, 777, 32, 8),    # one token: a decode step through the prefill kernel
    (3, 300, 45, 64, 8),   # group 8, three sequences of three tiles each, unaligned start
    (4, 260, 1000, 16, 2), # long cached prefix: many key blocks before the diagonal
])
def test_prefill_vs_oracle(ops, oracle, batch, n_q, start_pos, nh, nkv):
    got, ref = _case(ops, oracle, batch, n_q, start_pos, nh, nkv, seed=batch * 100 + n_q)
    assert_attn_close(got, ref, f"B={batch} n_q={n_q} start={start_pos} Hq={nh}")


def test_prefill_config4_sequence(ops, oracle):
    """One sequence of config 4: 2048 prompt tokens, Hq=32, Hkv=8, causal."""
    got, ref = _case(ops, oracle, 1, 2048, 0, 32, 8, seed=4)
    assert_attn_close(got, ref, "2048-token chunk")


def test_prefill_workspace_clean(ops):
    ws = ops.Scratch()
    q = torch.randn(1, 300, 8, 128, device="cuda").half()
    k = torch.randn(300, 2, 128, device="cuda").half()
    o = torch.empty_like(q)
    ops.attention_prefill(q, k, k, torch.zeros(1, dtype=torch.int64, device="cuda"), o, 0, 8, 2,
                          workspace=ws)
    assert ws.check() == 0
    assert torch.isfinite(o.float()).all()


@pytest.mark.parametrize("n_q,start_pos", [(200, 0), (256, 300), (77, 1000)])
def test_prefill_ignores_rows_past_chunk(ops, oracle, n_q, start_pos):
    """Cache rows past the chunk's end hold NaN (an unwritten pool): the key
    block that straddles the end must not let them into the output."""
    nh, nkv, hd, extra = 8, 2, 128, 200
    rows = start_pos + n_q + extra
    kp = oracle.normal_f16(rows * nkv * hd, 11).reshape(rows, nkv, hd)
    vp = oracle.normal_f16(rows * nkv * hd, 12).reshape(rows, nkv, hd)
    q = oracle.normal_f16(n_q * nh * hd, 13).reshape(1, n_q, nh, hd)
    nan = np.uint16(0x7E00)
    kd, vd = kp.copy(), vp.copy()
    kd[start_pos + n_q:] = nan
    vd[start_pos + n_q:] = nan
    ro = torch.zeros(1, dtype=torch.int64, device="cuda")
    o = torch.empty((1, n_q, nh, hd), dtype=torch.float16, device="cuda")
    ops.attention_prefill(to_dev(q), to_dev(kd), to_dev(vd), ro, o, start_pos, nh, nkv, hd)
    got = vals(o)
    assert np.isfinite(got).all()
    ref = oracle.attention_prefill(q, kp, vp, np.zeros(1, np.int64), n_q, start_pos, nh, nkv, hd)
    assert_attn_close(got, ref, f"n_q={n_q} start={start_pos} NaN past the chunk")
