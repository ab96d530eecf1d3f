"""Parity at the exact shapes ``bench.py`` times, against the CPU oracle
(restatement of kernels/sparse_attn.wgsl:32-113 and kernels/kv_append.wgsl:13-18).

* Config 3 (the headline): the full 256-sequence seed-3 pool of
  ``bench.Config3``, two fused append + attention steps exactly as the bench
  launches them (the stream-K split over 256 x 8 pairs of up to 8 208 rows);
  every one of the 256 x 32 heads against the oracle, and the whole K/V pool
  bit-exact after the appends.
* Config 5: 4 sequences x 1 048 576 rows at Hq=32, Hkv=8 cut into 8 shards as
  8 ranks would hold them, one shard-partial launch per shard (each the launch
  one rank of an 8-GPU run makes), the packed partials merged in shard order;
  sequences 0 and 3 against the float64 oracle.
* Config 4: the full 8 x 2048 prompt batch through nwd_kv_append_rows +
  nwd_attn_prefill, the pool bit-exact and sequences 0 and 7 against the oracle
  (one decode step per prompt token, engine/runtime.js:640-643).
"""
from __future__ import annotations

import importlib
import os
import sys

import numpy as np
import pytest
import torch

from devutil import bits, vals
from tolerance import assert_attn_close

pytestmark = pytest.mark.gpu

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if REPO not in sys.path:
    sys.path.insert(0, REPO)

HQ, HKV, HD = 32, 8, 128


@pytest.fixture(scope="module")
def bench():
    return importlib.import_module("bench")


def test_config3_full_pool_two_steps(ops, oracle, bench):
    W = bench.Config3(ops, torch, 0, 1, "weak", torch.device("cuda", 0))
    sd = W.seeds
    k = oracle.normal_f16(W.rows * HKV * HD, sd["k"]).reshape(W.rows, HKV, HD)
    v = oracle.normal_f16(W.rows * HKV * HD, sd["v"]).reshape(W.rows, HKV, HD)
    q = oracle.normal_f16(W.B * HQ * HD, sd["q"]).reshape(W.B, HQ, HD)
    kn = oracle.normal_f16(W.B * HKV * HD, sd["kn"]).reshape(W.B, HKV, HD)
    vn = oracle.normal_f16(W.B * HKV * HD, sd["vn"]).reshape(W.B, HKV, HD)
    assert np.array_equal(bits(W.k_pool), k) and np.array_equal(bits(W.v_pool), v)
    for s in range(2):
        W.step(s)
        torch.cuda.synchronize()
        pos = W.pos_host[s]
        rows = W.offs + pos
        k[rows] = kn
        v[rows] = vn
        assert np.array_equal(bits(W.k_pool), k), f"step {s}: K pool differs"
        assert np.array_equal(bits(W.v_pool), v), f"step {s}: V pool differs"
        ref = oracle.attention_batched(q, k, v, W.offs, (pos + 1).astype(np.int32), HQ, HKV, HD)
        assert_attn_close(vals(W.o), ref, f"config 3 step {s} (256 sequences x 32 heads)")
    assert W.ws.check() == 0


def test_config5_eight_shards(ops, oracle):
    B, L, S = 4, 1 << 20, 8
    row = HKV * HD
    dev = torch.device("cuda", 0)
    k_pool = torch.empty(B * L, HKV, HD, dtype=torch.float16, device=dev)
    v_pool = torch.empty_like(k_pool)
    # the bench's fill: element offsets follow the global row index
    ops.fill_normal(k_pool, 5000)
    ops.fill_normal(v_pool, 5001)
    q = ops.fill_normal(torch.empty(B, HQ, HD, dtype=torch.float16, device=dev), 5002)
    packed = torch.empty(S, B * HQ * (HD + 2), dtype=torch.float32, device=dev)
    n_o = B * HQ * HD
    ws = ops.Workspace(B, HQ, HKV, HD, dev)
    for r in range(S):
        lo, hi = L * r // S, L * (r + 1) // S
        ro = torch.tensor([b * L + lo for b in range(B)], dtype=torch.int64, device=dev)
        sl = torch.full((B,), hi - lo, dtype=torch.int32, device=dev)
        part_o = packed[r, :n_o].view(B, HQ, HD)
        part_ml = packed[r, n_o:].view(B, HQ, 2)
        ops.attention_partial(q, k_pool, v_pool, ro, sl, part_o, part_ml, HQ, HKV, HD,
                              workspace=ws)
    o = torch.empty(B, HQ, HD, dtype=torch.float16, device=dev)
    ops.merge_packed(packed, o)
    torch.cuda.synchronize()
    assert ws.check() == 0
    got = vals(o)
    qh = oracle.normal_f16(B * HQ * HD, 5002).reshape(B, HQ, HD)
    assert np.array_equal(bits(q), qh)
    del k_pool, v_pool
    torch.cuda.empty_cache()
    for b in (0, 3):
        kb = oracle.normal_f16(L * row, 5000, b * L * row)
        vb = oracle.normal_f16(L * row, 5001, b * L * row)
        ref = oracle.attention_batched(qh[b], kb, vb, [0], [L], HQ, HKV, HD, f64=True)
        assert_attn_close(got[b:b + 1], ref, f"config 5 sequence {b}: 8 shards of 131072 rows")


def test_config4_full_batch(ops, oracle):
    B, S, seed = 8, 2048, 4000
    dev = torch.device("cuda", 0)
    f16 = torch.float16
    k_pool = torch.full((B * S, HKV, HD), float("nan"), dtype=f16, device=dev)
    v_pool = torch.full_like(k_pool, float("nan"))
    k_new = ops.fill_normal(torch.empty(B, S, HKV, HD, dtype=f16, device=dev), seed)
    v_new = ops.fill_normal(torch.empty(B, S, HKV, HD, dtype=f16, device=dev), seed + 1)
    q = ops.fill_normal(torch.empty(B, S, HQ, HD, dtype=f16, device=dev), seed + 2)
    o = torch.empty(B, S, HQ, HD, dtype=f16, device=dev)
    ro = torch.arange(B, dtype=torch.int64, device=dev) * S
    ws = ops.Scratch(dev)
    ops.kv_append_rows(k_new, v_new, k_pool, v_pool, ro, 0, workspace=ws)
    ops.attention_prefill(q, k_pool, v_pool, ro, o, 0, HQ, HKV, HD, workspace=ws)
    torch.cuda.synchronize()
    assert ws.check() == 0
    kh = oracle.normal_f16(B * S * HKV * HD, seed).reshape(B * S, HKV, HD)
    vh = oracle.normal_f16(B * S * HKV * HD, seed + 1).reshape(B * S, HKV, HD)
    qh = oracle.normal_f16(B * S * HQ * HD, seed + 2).reshape(B, S, HQ, HD)
    assert np.array_equal(bits(k_pool), kh) and np.array_equal(bits(v_pool), vh)
    got = vals(o)
    for b in (0, 7):
        ref = oracle.attention_prefill(qh[b:b + 1], kh, vh, np.array([b * S], np.int64), S, 0,
                                       HQ, HKV, HD)
        assert_attn_close(got[b:b + 1], ref, f"config 4 sequence {b} (2048 causal tokens)")
