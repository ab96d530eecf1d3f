"""Decode attention on the GPU against the oracle (kernels/sparse_attn.wgsl:32-113).

Tolerance: max-abs 2e-3 and max-rel 1e-2 on fp16 outputs (tests/tolerance.py).
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from devutil import bits, to_dev, vals
from golden.make_golden import CASES, case_inputs
from tolerance import assert_attn_close, f16

pytestmark = pytest.mark.gpu


def _single(ops, oracle, nh, nkv, L, cap, seed, scale=0.0):
    hd = 128
    q = oracle.normal_f16(nh * hd, seed)
    k = oracle.normal_f16(cap * nkv * hd, seed + 1)
    v = oracle.normal_f16(cap * nkv * hd, seed + 2)
    o = torch.empty(nh, hd, dtype=torch.float16, device="cuda")
    ops.attention(to_dev(q, (nh, hd)), to_dev(k, (cap, nkv, hd)), to_dev(v, (cap, nkv, hd)), o,
                  ops.AttnParams(nh, nkv, hd, L), scale=scale)
    ref = oracle.attention(q, k, v, nh, nkv, hd, L, scale=scale)
    return vals(o), ref


@pytest.mark.parametrize("nh", [40, 32])
@pytest.mark.parametrize("L", [1, 2, 15, 16, 17, 63, 64, 65, 127, 128, 129, 151, 255, 256, 257,
                               1000, 1024, 4096, 16384, 32768])
def test_single_sequence(ops, oracle, nh, L):
    got, ref = _single(ops, oracle, nh, 8, L, L + 3, seed=1000 + L)
    assert_attn_close(got, ref, f"Hq={nh} L={L}")


@pytest.mark.parametrize("L", [1, 64, 256, 300])
def test_last_row_of_buffer(ops, oracle, L):
    """seq equal to the cache capacity: the TMA box must not read past it."""
    got, ref = _single(ops, oracle, 40, 8, L, L, seed=7)
    assert_attn_close(got, ref, f"cap=L={L}")


@pytest.mark.parametrize("nh,nkv", [(8, 8), (16, 8), (24, 8), (56, 8), (64, 8), (16, 2), (5, 1)])
def test_group_sizes(ops, oracle, nh, nkv):
    got, ref = _single(ops, oracle, nh, nkv, 777, 800, seed=31)
    assert_attn_close(got, ref, f"Hq={nh} Hkv={nkv}")


@pytest.mark.parametrize("nh,nkv,L", [(8, 8, 3000), (64, 8, 3000), (16, 2, 9000), (5, 1, 12000),
                                      (3, 1, 2049), (40, 8, 2049)])
def test_group_sizes_split(ops, oracle, nh, nkv, L):
    """Group sizes on the split-KV kernel (past the short kernel's 2 048 rows): with one or
    two kv heads a pair is cut into up to one piece per SM, so the last CTA merges up
    to ~148 partials (many batches of loads) and every CTA's range prefetch differs."""
    got, ref = _single(ops, oracle, nh, nkv, L, L + 7, seed=91 + L)
    assert_attn_close(got, ref, f"Hq={nh} Hkv={nkv} L={L}")


@pytest.mark.parametrize("nh,nkv,L", [(8, 8, 151), (16, 8, 33), (24, 8, 151), (56, 8, 200),
                                      (64, 8, 256), (16, 2, 97), (5, 1, 151), (3, 1, 1)])
def test_group_sizes_short(ops, oracle, nh, nkv, L):
    """Every group size (1..8) on the single-CTA-per-kv-head kernel (<= 256 rows)."""
    got, ref = _single(ops, oracle, nh, nkv, L, L + 5, seed=41 + L)
    assert_attn_close(got, ref, f"Hq={nh} Hkv={nkv} L={L}")


@pytest.mark.parametrize("L", [200, 500])
def test_custom_scale(ops, oracle, L):
    got, ref = _single(ops, oracle, 32, 8, L, 512, seed=5, scale=0.03)
    assert_attn_close(got, ref, f"scale=0.03 L={L}")


def test_zero_length_writes_zeros(ops):
    o = torch.full((32, 128), 7.0, dtype=torch.float16, device="cuda")
    k = torch.randn(4, 8, 128, device="cuda").half()
    q = torch.randn(32, 128, device="cuda").half()
    ops.attention(q, k, k, o, ops.AttnParams(32, 8, 128, 0))
    assert not o.any()


@pytest.mark.parametrize("name", list(CASES))
def test_golden_cases_batched(ops, golden, name):
    nh, nkv, hd, lens, caps, seeds = CASES[name]
    q, k, v, offs, L, rows = case_inputs(nh, nkv, hd, lens, caps, seeds)
    B = len(L)
    o = torch.empty(B, nh, hd, dtype=torch.float16, device="cuda")
    ops.attention_batched(to_dev(q, (B, nh, hd)), to_dev(k, (rows, nkv, hd)),
                          to_dev(v, (rows, nkv, hd)), torch.tensor(offs, device="cuda"),
                          torch.tensor(L, device="cuda"), o, nh, nkv, hd)
    assert_attn_close(vals(o), golden[f"case/{name}/out"], name)


def test_ragged_batch_vs_oracle(ops, oracle):
    rng = np.random.default_rng(3)
    B, nh, nkv, hd = 64, 32, 8, 128
    L = rng.integers(0, 3000, B).astype(np.int32)
    L[:4] = [0, 1, 64, 65]
    caps = L + rng.integers(0, 40, B)
    offs = np.concatenate([[0], np.cumsum(caps)[:-1]]).astype(np.int64)
    rows = int(caps.sum())
    q = oracle.normal_f16(B * nh * hd, 71)
    k = oracle.normal_f16(rows * nkv * hd, 72)
    v = oracle.normal_f16(rows * nkv * hd, 73)
    o = torch.empty(B, nh, hd, dtype=torch.float16, device="cuda")
    ops.attention_batched(to_dev(q, (B, nh, hd)), to_dev(k, (rows, nkv, hd)),
                          to_dev(v, (rows, nkv, hd)), torch.tensor(offs, device="cuda"),
                          torch.tensor(L, device="cuda"), o, nh, nkv, hd)
    ref = oracle.attention_batched(q, k, v, offs, L, nh, nkv, hd)
    assert_attn_close(vals(o), ref, "ragged B=64")


def test_large_batch_tiny_and_empty_sequences(ops, oracle):
    """Many pieces per CTA, empty sequences spread over the CTAs that own them."""
    rng = np.random.default_rng(17)
    B, nh, nkv, hd = 1000, 40, 8, 128
    L = rng.integers(0, 100, B).astype(np.int32)
    L[rng.choice(B, 150, replace=False)] = 0
    caps = np.maximum(L, 1)
    offs = np.concatenate([[0], np.cumsum(caps)[:-1]]).astype(np.int64)
    rows = int(caps.sum())
    q = oracle.normal_f16(B * nh * hd, 171)
    k = oracle.normal_f16(rows * nkv * hd, 172)
    v = oracle.normal_f16(rows * nkv * hd, 173)
    o = torch.full((B, nh, hd), 3.0, dtype=torch.float16, device="cuda")
    ops.attention_batched(to_dev(q, (B, nh, hd)), to_dev(k, (rows, nkv, hd)),
                          to_dev(v, (rows, nkv, hd)), torch.tensor(offs, device="cuda"),
                          torch.tensor(L, device="cuda"), o, nh, nkv, hd)
    ref = oracle.attention_batched(q, k, v, offs, L, nh, nkv, hd)
    assert_attn_close(vals(o), ref, "B=1000 tiny/empty")
    assert not vals(o)[L == 0].any()


def test_repeat_calls_identical_and_clean(ops, oracle):
    """Workspace tickets / queue reset between calls; results are deterministic."""
    nh, nkv, hd, L = 40, 8, 128, 20000
    q = to_dev(oracle.normal_f16(nh * hd, 1), (nh, hd))
    k = to_dev(oracle.normal_f16(L * nkv * hd, 2), (L, nkv, hd))
    v = to_dev(oracle.normal_f16(L * nkv * hd, 3), (L, nkv, hd))
    ws = ops.Workspace(1, nh, nkv, hd)
    outs = []
    for _ in range(4):
        o = torch.empty(nh, hd, dtype=torch.float16, device="cuda")
        ops.attention(q, k, v, o, ops.AttnParams(nh, nkv, hd, L), workspace=ws)
        outs.append(bits(o))
    assert all(np.array_equal(outs[0], x) for x in outs[1:])
    assert ws.check() == 0
    # the same workspace then serves a shorter sequence correctly
    o = torch.empty(nh, hd, dtype=torch.float16, device="cuda")
    ops.attention(q, k, v, o, ops.AttnParams(nh, nkv, hd, 5000), workspace=ws)
    ref = oracle.attention(bits(q), bits(k), bits(v), nh, nkv, hd, 5000)
    assert_attn_close(vals(o), ref, "after reuse")
    assert ws.check() == 0


def test_engine_trace_config1(engine_mod, oracle):
    """Config 1: 24 prompt steps + 127 decode steps through the fused step,
    checked against the oracle at every step (runtime.js:447-467 ordering)."""
    nh, nkv, hd, cap = 40, 8, 128, 256
    layer = engine_mod.DecodeAttention(nh, nkv, hd, cap)
    kc = np.zeros((cap, nkv, hd), np.uint16)
    vc = np.zeros((cap, nkv, hd), np.uint16)
    worst = 0.0
    for step in range(24 + 127):
        q = oracle.normal_f16(nh * hd, 1, step * nh * hd)
        kn = oracle.normal_f16(nkv * hd, 2, step * nkv * hd)
        vn = oracle.normal_f16(nkv * hd, 3, step * nkv * hd)
        out = layer.step(to_dev(q, (nh, hd)), to_dev(kn, (nkv, hd)), to_dev(vn, (nkv, hd)))
        oracle.kv_append(kn, kc, step, nkv, hd)
        oracle.kv_append(vn, vc, step, nkv, hd)
        ref = oracle.attention(q, kc, vc, nh, nkv, hd, step + 1)
        mab, _ = assert_attn_close(vals(out), ref, f"step {step}")
        worst = max(worst, mab)
    assert layer.seq == 151
    assert np.array_equal(bits(layer.k_cache), kc) and np.array_equal(bits(layer.v_cache), vc)
    assert layer.workspace.check() == 0


@pytest.mark.parametrize("seq", [0, 255, 256, 700, 2047, 2100])
def test_fused_append_single(ops, oracle, seq):
    """kv_append + attention in one call at the one-CTA, cluster and general
    kernels' row counts (seq + 1 rows): the new row lands in the caches and in
    the output; every other cache row is untouched."""
    nh, nkv, hd, cap = 40, 8, 128, seq + 9
    q = oracle.normal_f16(nh * hd, 51)
    kn = oracle.normal_f16(nkv * hd, 52)
    vn = oracle.normal_f16(nkv * hd, 53)
    kc = oracle.normal_f16(cap * nkv * hd, 54).reshape(cap, nkv, hd)
    vc = oracle.normal_f16(cap * nkv * hd, 55).reshape(cap, nkv, hd)
    dk, dv = to_dev(kc), to_dev(vc)
    o = torch.empty(nh, hd, dtype=torch.float16, device="cuda")
    ops.kv_append_attention(to_dev(q, (nh, hd)), to_dev(kn, (nkv, hd)), to_dev(vn, (nkv, hd)),
                            dk, dv, o, ops.AttnParams(nh, nkv, hd, seq))
    oracle.kv_append(kn, kc, seq, nkv, hd)
    oracle.kv_append(vn, vc, seq, nkv, hd)
    ref = oracle.attention(q, kc, vc, nh, nkv, hd, seq + 1)
    assert_attn_close(vals(o), ref, f"fused append at row {seq}")
    assert np.array_equal(bits(dk), kc) and np.array_equal(bits(dv), vc)


def test_engine_prompt_chunk_then_steps(engine_mod, oracle):
    """Config 1 with the 24-token prompt as one chunk (DecodeAttention.prefill,
    the tcgen05 kernel) instead of 24 steps, then 127 decode steps: every output matches
    the reference's token-by-token order (runtime.js:640-646)."""
    nh, nkv, hd, cap, n_prompt = 40, 8, 128, 256, 24
    layer = engine_mod.DecodeAttention(nh, nkv, hd, cap)
    kc = np.zeros((cap, nkv, hd), np.uint16)
    vc = np.zeros((cap, nkv, hd), np.uint16)
    qs = [oracle.normal_f16(nh * hd, 1, t * nh * hd) for t in range(24 + 127)]
    ks = [oracle.normal_f16(nkv * hd, 2, t * nkv * hd) for t in range(24 + 127)]
    vs = [oracle.normal_f16(nkv * hd, 3, t * nkv * hd) for t in range(24 + 127)]
    out = layer.prefill(to_dev(np.stack(qs[:n_prompt]), (n_prompt, nh, hd)),
                        to_dev(np.stack(ks[:n_prompt]), (n_prompt, nkv, hd)),
                        to_dev(np.stack(vs[:n_prompt]), (n_prompt, nkv, hd)))
    assert layer.seq == n_prompt
    got = vals(out)
    for t in range(n_prompt):
        oracle.kv_append(ks[t], kc, t, nkv, hd)
        oracle.kv_append(vs[t], vc, t, nkv, hd)
        ref = oracle.attention(qs[t], kc, vc, nh, nkv, hd, t + 1)
        assert_attn_close(got[t], ref, f"prompt token {t}")
    for t in range(n_prompt, 24 + 127):
        out = layer.step(to_dev(qs[t], (nh, hd)), to_dev(ks[t], (nkv, hd)),
                         to_dev(vs[t], (nkv, hd)))
        oracle.kv_append(ks[t], kc, t, nkv, hd)
        oracle.kv_append(vs[t], vc, t, nkv, hd)
        assert_attn_close(vals(out), oracle.attention(qs[t], kc, vc, nh, nkv, hd, t + 1),
                          f"step {t}")
    assert np.array_equal(bits(layer.k_cache), kc) and np.array_equal(bits(layer.v_cache), vc)
    assert layer.workspace.check() == 0


def test_engine_prompt_chunk_past_max_seq(engine_mod, ops):
    layer = engine_mod.DecodeAttention(32, 8, 128, max_seq=16)
    q = torch.randn(10, 32, 128, device="cuda").half()
    kv = torch.randn(10, 8, 128, device="cuda").half()
    layer.prefill(q, kv, kv)
    with pytest.raises(ops.NwdError, match="seq 16 exceeds maxSeq 16"):
        layer.prefill(q, kv, kv)
    assert layer.seq == 10


def test_engine_max_seq_error(engine_mod, ops):
    layer = engine_mod.DecodeAttention(32, 8, 128, max_seq=2)
    q = torch.randn(32, 128, device="cuda").half()
    kv = torch.randn(8, 128, device="cuda").half()
    layer.step(q, kv, kv)
    layer.step(q, kv, kv)
    with pytest.raises(ops.NwdError, match="seq 2 exceeds maxSeq 2"):
        layer.step(q, kv, kv)
    layer.reset()
    assert layer.seq == 0 and not layer.k_cache.any()


def test_batched_fused_append(engine_mod, oracle):
    rng = np.random.default_rng(9)
    B, nh, nkv, hd = 24, 32, 8, 128
    L0 = rng.integers(0, 1500, B).astype(np.int32)
    L0[:3] = [0, 63, 64]
    steps = 3
    caps = L0 + steps
    att = engine_mod.BatchedDecodeAttention(caps, nh, nkv, hd)
    rows = att.pool_rows
    k0 = oracle.normal_f16(rows * nkv * hd, 81).reshape(rows, nkv, hd)
    v0 = oracle.normal_f16(rows * nkv * hd, 82).reshape(rows, nkv, hd)
    att.k_pool.copy_(to_dev(k0, (rows, nkv, hd)))
    att.v_pool.copy_(to_dev(v0, (rows, nkv, hd)))
    att.lengths.copy_(torch.tensor(L0, device="cuda"))
    offs = att.row_offset.cpu().numpy()
    L = L0.copy()
    for s in range(steps):
        q = oracle.normal_f16(B * nh * hd, 90 + s)
        kn = oracle.normal_f16(B * nkv * hd, 95 + s).reshape(B, nkv, hd)
        vn = oracle.normal_f16(B * nkv * hd, 99 + s).reshape(B, nkv, hd)
        out = att.step(to_dev(q, (B, nh, hd)), to_dev(kn), to_dev(vn))
        for b in range(B):
            k0[offs[b] + L[b]] = kn[b]
            v0[offs[b] + L[b]] = vn[b]
        L += 1
        ref = oracle.attention_batched(q, k0, v0, offs, L, nh, nkv, hd)
        assert_attn_close(vals(out), ref, f"step {s}")
    assert np.array_equal(bits(att.k_pool), k0) and np.array_equal(bits(att.v_pool), v0)
    assert np.array_equal(att.lengths.cpu().numpy(), L)
    assert att.workspace.check() == 0


def test_partial_and_merge(ops, oracle):
    """Shard one sequence's rows three ways; GPU partials + GPU merge == whole."""
    nh, nkv, hd, L = 32, 8, 128, 30000
    B = 2
    q = oracle.normal_f16(B * nh * hd, 41)
    k = oracle.normal_f16(2 * L * nkv * hd, 42)
    v = oracle.normal_f16(2 * L * nkv * hd, 43)
    dq, dk, dv = to_dev(q, (B, nh, hd)), to_dev(k, (2 * L, nkv, hd)), to_dev(v, (2 * L, nkv, hd))
    cuts = [0, 7000, 7001, 30000]
    parts_o, parts_ml = [], []
    for a, b in zip(cuts[:-1], cuts[1:]):
        offs = np.array([a, L + a], np.int64)
        lens = np.array([b - a, b - a], np.int32)
        po = torch.empty(B, nh, hd, dtype=torch.float32, device="cuda")
        pml = torch.empty(B, nh, 2, dtype=torch.float32, device="cuda")
        ops.attention_partial(dq, dk, dv, torch.tensor(offs, device="cuda"),
                              torch.tensor(lens, device="cuda"), po, pml, nh, nkv, hd)
        ro, rml = oracle.attention_partial(q, k, v, offs, lens, nh, nkv, hd)
        m = pml.cpu().numpy()[..., 0]
        # m is a reference maximum: within 8 (log2 units) below the true one
        assert (m <= rml[..., 0] + 1e-3).all() and (m >= rml[..., 0] - 8 - 1e-3).all()
        # compare on a common max: l * 2^(m - m_ref), o * 2^(m - m_ref)
        f = np.exp2(m - rml[..., 0])
        np.testing.assert_allclose(pml.cpu().numpy()[..., 1] * f, rml[..., 1], rtol=2e-3)
        np.testing.assert_allclose(po.cpu().numpy() * f[..., None], ro, rtol=5e-3,
                                   atol=5e-3 * np.abs(ro).max())
        parts_o.append(po)
        parts_ml.append(pml)
    o = torch.empty(B, nh, hd, dtype=torch.float16, device="cuda")
    ops.merge(torch.stack(parts_o), torch.stack(parts_ml), o)
    ref = oracle.attention_batched(q, k, v, np.array([0, L], np.int64),
                                   np.array([L, L], np.int32), nh, nkv, hd)
    assert_attn_close(vals(o), ref, "3-shard merge")


@pytest.mark.parametrize("shards", [1, 3, 6])
def test_merge_packed(ops, oracle, shards):
    """Partials written straight into packed buffers (o, then (m, l)), one buffer per
    shard as an all-gather would deliver them; merge_packed == merge, and == whole."""
    nh, nkv, hd, L, B = 16, 4, 128, 9000, 2
    q = oracle.normal_f16(B * nh * hd, 61)
    k = oracle.normal_f16(B * L * nkv * hd, 62)
    v = oracle.normal_f16(B * L * nkv * hd, 63)
    dq, dk, dv = to_dev(q, (B, nh, hd)), to_dev(k, (B * L, nkv, hd)), to_dev(v, (B * L, nkv, hd))
    cuts = [L * i // shards for i in range(shards + 1)]
    bufs = []
    for a, b in zip(cuts[:-1], cuts[1:]):
        buf, po, pml = ops.packed_partials(B, nh, hd, device="cuda")
        offs = torch.tensor([a, L + a], dtype=torch.int64, device="cuda")
        lens = torch.tensor([b - a, b - a], dtype=torch.int32, device="cuda")
        ops.attention_partial(dq, dk, dv, offs, lens, po, pml, nh, nkv, hd)
        bufs.append(buf)
    g = torch.stack(bufs)
    o_packed = torch.empty(B, nh, hd, dtype=torch.float16, device="cuda")
    ops.merge_packed(g, o_packed)
    n = B * nh * hd
    o_plain = torch.empty_like(o_packed)
    ops.merge(g[:, :n].reshape(shards, B, nh, hd).contiguous(),
              g[:, n:].reshape(shards, B, nh, 2).contiguous(), o_plain)
    assert torch.equal(o_packed, o_plain)
    ref = oracle.attention_batched(q, k, v, np.array([0, L], np.int64),
                                   np.array([L, L], np.int32), nh, nkv, hd)
    assert_attn_close(vals(o_packed), ref, f"{shards}-shard packed merge")


def test_long_sequence_262k(ops, oracle):
    """A 262144-row sequence (1 GiB of K+V) against the oracle."""
    nh, nkv, hd, L = 32, 8, 128, 262144
    q = oracle.normal_f16(nh * hd, 51)
    k = oracle.normal_f16(L * nkv * hd, 52)
    v = oracle.normal_f16(L * nkv * hd, 53)
    o = torch.empty(nh, hd, dtype=torch.float16, device="cuda")
    ops.attention(to_dev(q, (nh, hd)), to_dev(k, (L, nkv, hd)), to_dev(v, (L, nkv, hd)), o,
                  ops.AttnParams(nh, nkv, hd, L))
    ref = oracle.attention_batched(q, k, v, [0], [L], nh, nkv, hd, f64=True)[0]
    assert_attn_close(vals(o), ref, "L=262144")


def test_long_context_1m_rows_via_sharded_path(oracle):
    """A 1 048 576-row sequence (Hq=8, Hkv=2: 1 GiB of K+V) through the shard
    partial + merge path of mgpu.ShardedDecode (one process holds the shard)."""
    import importlib
    mgpu = importlib.import_module("nemotron-webgpu-decode_b200.mgpu")
    nh, nkv, hd, L = 8, 2, 128, 1 << 20
    sd = mgpu.ShardedDecode([L], nh, nkv, hd, device="cuda")
    k = oracle.normal_f16(L * nkv * hd, 61)
    v = oracle.normal_f16(L * nkv * hd, 62)
    q = oracle.normal_f16(nh * hd, 63)
    sd.k_pool.copy_(to_dev(k, (L, nkv, hd)))
    sd.v_pool.copy_(to_dev(v, (L, nkv, hd)))
    out = sd.step(to_dev(q, (1, nh, hd)))
    ref = oracle.attention_batched(q, k, v, [0], [L], nh, nkv, hd, f64=True)
    assert_attn_close(vals(out), ref, "L=1M sharded path")
    assert sd.workspace.check() == 0
