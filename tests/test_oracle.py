"""The CPU oracle against the golden fixtures and known answers (no GPU).

The oracle restates kernels/sparse_attn.wgsl:32-113 and kernels/kv_append.wgsl:13-18.
Parity with the reference itself is unpinned (no reference tests, no runnable
WGSL here); these tests pin the oracle against an independent float64 numpy
restatement (tests/golden) and against hand-derivable answers.
"""
from __future__ import annotations

import numpy as np
import pytest

from golden.make_golden import CASES, case_inputs
from tolerance import assert_attn_close, f16


def test_f16_conversions_exhaustive(oracle):
    bits = np.arange(65536, dtype=np.uint16)
    f = oracle.f16_bits_to_f32(bits)
    ref = bits.view(np.float16).astype(np.float32)
    nan = np.isnan(ref)
    assert np.array_equal(f[~nan].view(np.uint32), ref[~nan].view(np.uint32))
    assert np.isnan(f[nan]).all()
    # round trip of every finite half
    assert np.array_equal(oracle.f32_to_f16_bits(f[~nan]), bits[~nan])


def test_f32_to_f16_round_to_nearest_even(oracle):
    rng = np.random.default_rng(0)
    x = (rng.standard_normal(200_000) * 10.0 ** rng.uniform(-9, 5, 200_000)).astype(np.float32)
    edge = np.array([65504, 65519.996, 65520, -65520, 6e-8, 2.98e-8, 2.9802322e-08, 1e-45, 0.0,
                     -0.0, np.inf, -np.inf, 6.103515625e-05, 6.1e-05], np.float32)
    x = np.concatenate([x, edge])
    with np.errstate(over="ignore"):
        ref = x.astype(np.float16).view(np.uint16)
    assert np.array_equal(oracle.f32_to_f16_bits(x), ref)


def test_generator_matches_golden(oracle, golden):
    n = 0
    for k in golden.files:
        if k.startswith("gen/"):
            seed, off = map(int, k[4:].split("_"))
            assert np.array_equal(oracle.normal_f16(64, seed, off), golden[k]), k
            n += 1
    assert n >= 8


def test_generator_statistics(oracle):
    x = f16(oracle.normal_f16(1_000_000, 7))
    assert abs(x.mean()) < 5e-3
    assert abs(x.std() - 1.0) < 5e-3
    assert x.min() > -6.1 and x.max() < 6.1
    # streams with different seeds / offsets differ; same (seed, offset) repeats
    assert not np.array_equal(oracle.normal_f16(64, 1), oracle.normal_f16(64, 2))
    assert np.array_equal(oracle.normal_f16(10, 3, 5), oracle.normal_f16(15, 3)[5:])


@pytest.mark.parametrize("name", list(CASES))
def test_oracle_matches_golden(oracle, golden, name):
    nh, nkv, hd, lens, caps, seeds = CASES[name]
    q, k, v, offs, L, rows = case_inputs(nh, nkv, hd, lens, caps, seeds)
    assert np.array_equal(golden[f"case/{name}/lengths"], L)
    out = oracle.attention_batched(q, k, v, offs, L, nh, nkv, hd)
    # fp16 output as the kernels produce it
    out16 = f16(oracle.f32_to_f16_bits(out))
    assert_attn_close(out16, golden[f"case/{name}/out"], name)
    # the f32 restatement itself is much closer than the tolerance
    assert np.abs(out - golden[f"case/{name}/out"]).max() < 1e-5


def test_single_call_equals_batched(oracle):
    nh, nkv, hd, L = 40, 8, 128, 151
    q = oracle.normal_f16(nh * hd, 1)
    k = oracle.normal_f16(256 * nkv * hd, 2)
    v = oracle.normal_f16(256 * nkv * hd, 3)
    a = oracle.attention(q, k, v, nh, nkv, hd, L)
    b = oracle.attention_batched(q, k, v, [0], [L], nh, nkv, hd)[0]
    assert np.array_equal(a, b)


def test_kat_single_key_is_v_row(oracle):
    nh, nkv, hd = 32, 8, 128
    q = oracle.normal_f16(nh * hd, 5)
    k = oracle.normal_f16(4 * nkv * hd, 6)
    v = oracle.normal_f16(4 * nkv * hd, 7)
    out = oracle.attention(q, k, v, nh, nkv, hd, 1)
    vrow = f16(v).reshape(4, nkv, hd)[0]
    for h in range(nh):
        assert np.array_equal(out[h], vrow[h // 4].astype(np.float32))


def test_kat_equal_keys_average_v(oracle):
    nh, nkv, hd, L = 8, 2, 128, 64
    q = oracle.normal_f16(nh * hd, 8)
    krow = oracle.normal_f16(nkv * hd, 9)
    k = np.tile(krow, L)
    # V rows: small integers so the mean is exact in f32
    vals = (np.arange(L * nkv * hd) % 7 - 3).astype(np.float16).view(np.uint16)
    out = oracle.attention(q, k, vals, nh, nkv, hd, L)
    mean = f16(vals).reshape(L, nkv, hd).mean(axis=0)
    for h in range(nh):
        np.testing.assert_allclose(out[h], mean[h // 4], atol=1e-6)


def test_kat_one_hot_score(oracle):
    """A key aligned with q and scaled large dominates: O ~ that V row."""
    nh, nkv, hd, L = 4, 1, 128, 32
    qv = np.zeros((nh, hd), np.float16)
    qv[:, 0] = 8.0
    k = np.zeros((L, nkv, hd), np.float16)
    k[17, 0, 0] = 8.0  # score 64 / sqrt(128) ~ 5.7 -> use a larger scale
    v = f16(oracle.normal_f16(L * nkv * hd, 10)).astype(np.float16).reshape(L, nkv, hd)
    out = oracle.attention(qv.view(np.uint16), k.view(np.uint16), v.view(np.uint16), nh, nkv, hd,
                           L, scale=1.0)
    for h in range(nh):
        np.testing.assert_allclose(out[h], v[17, 0].astype(np.float32), atol=1e-6)


def test_empty_sequence_is_zero(oracle):
    q = oracle.normal_f16(32 * 128, 1)
    k = oracle.normal_f16(8 * 8 * 128, 2)
    out = oracle.attention(q, k, k, 32, 8, 128, 0)
    assert not out.any()


def test_kv_append_writes_one_row(oracle):
    n_kv, hd, cap = 8, 128, 16
    cache = oracle.normal_f16(cap * n_kv * hd, 3).reshape(cap, n_kv, hd)
    before = cache.copy()
    src = oracle.normal_f16(n_kv * hd, 4)
    oracle.kv_append(src, cache, 5, n_kv, hd)
    assert np.array_equal(cache[5].reshape(-1), src)
    mask = np.ones(cap, bool)
    mask[5] = False
    assert np.array_equal(cache[mask], before[mask])


def test_partial_merge_equals_whole(oracle):
    nh, nkv, hd, L = 40, 8, 128, 1000
    q = oracle.normal_f16(nh * hd, 1)
    k = oracle.normal_f16(L * nkv * hd, 2)
    v = oracle.normal_f16(L * nkv * hd, 3)
    whole = oracle.attention_batched(q, k, v, [0], [L], nh, nkv, hd, f64=True)[0]
    for cuts in ([0, 1000], [0, 500, 1000], [0, 1, 2, 999, 1000], [0, 0, 300, 1000, 1000]):
        parts = [oracle.attention_partial(q, k, v, [a], [b - a], nh, nkv, hd)
                 for a, b in zip(cuts[:-1], cuts[1:])]
        merged = oracle.merge(np.stack([p[0] for p in parts]), np.stack([p[1] for p in parts]))
        np.testing.assert_allclose(merged.reshape(nh, hd), whole, atol=2e-6, rtol=0)


def test_f64_and_f32_restatements_agree_long(oracle):
    """Drift check of the f32 (WGSL-order) restatement at a longer length."""
    nh, nkv, hd, L = 8, 2, 128, 20000
    q = oracle.normal_f16(nh * hd, 11)
    k = oracle.normal_f16(L * nkv * hd, 12)
    v = oracle.normal_f16(L * nkv * hd, 13)
    a = oracle.attention_batched(q, k, v, [0], [L], nh, nkv, hd)
    b = oracle.attention_batched(q, k, v, [0], [L], nh, nkv, hd, f64=True)
    assert np.abs(a - b).max() < 2e-5


def _q4_numpy_f64(a, B, scales, zp):
    """kernels/matmul_nbits_sg.wgsl:25-72 restated in numpy float64, independently of the
    C oracle: element j of word w of block blk is bits [4j, 4j+4) of B[n, blk, w] (the
    shader's lo/hi byte-nibble interleave, :37-40) and multiplies A[32*blk + 8*w + j];
    the zero point of (n, blk) is nibble n*n_blocks + blk of zp (:25-28)."""
    n, nb = scales.shape
    shifts = (4 * np.arange(8, dtype=np.uint32))[None, None, None, :]
    q = ((B.astype(np.uint32)[..., None] >> shifts) & 15).reshape(n, nb, 32).astype(np.float64)
    idx = np.arange(n * nb).reshape(n, nb)
    z = ((zp[idx // 8] >> ((idx % 8) * 4).astype(np.uint32)) & 15).astype(np.float64)
    a64 = np.asarray(a, np.float64).reshape(nb, 32)
    return (((q - z[..., None]) * a64[None]).sum(-1) * scales.astype(np.float64)).sum(-1)


@pytest.mark.parametrize("n,n_blocks", [(7, 1), (40, 98), (33, 160)])
def test_q4_gemv_oracle_vs_numpy(oracle, n, n_blocks):
    """The oracle's q4 GEMV (the parity reference for the projections around the path)
    against an independent float64 numpy restatement of the shader, and its epilogues."""
    B, scales, zp = oracle.q4_weights(n, n_blocks, seed=n + n_blocks)
    a = oracle.f16_bits_to_f32(oracle.normal_f16(32 * n_blocks, 5))
    ref = _q4_numpy_f64(a, B, scales, zp)
    np.testing.assert_allclose(oracle.q4_gemv_f64(a, B, scales, zp), ref, rtol=1e-12, atol=1e-9)
    tol = 1e-5 * max(float(np.abs(ref).max()), 1.0)
    got = oracle.q4_gemv(a, B, scales, zp)
    assert float(np.abs(got - ref).max()) <= tol
    relu2 = np.maximum(ref, 0.0) ** 2
    got1 = oracle.q4_gemv(a, B, scales, zp, epilogue=1)
    assert float(np.abs(got1 - relu2).max()) <= 1e-5 * max(float(np.abs(relu2).max()), 1.0)
    y0 = np.linspace(-1, 1, n).astype(np.float32)
    got2 = oracle.q4_gemv(a, B, scales, zp, epilogue=2, y=y0)
    assert float(np.abs(got2 - (y0 + ref)).max()) <= tol


def test_prefill_oracle_is_one_decode_step_per_token(oracle):
    """The prefill oracle is the reference's prompt loop (engine/runtime.js:640-643):
    token i of a chunk starting at row start_pos is a decode step over rows
    0..start_pos+i, bit-identical to the decode oracle on the same rows."""
    nh, nkv, hd, n_q, start, batch = 4, 2, 128, 5, 3, 2
    rows = start + n_q
    kp = oracle.normal_f16(batch * rows * nkv * hd, 71).reshape(batch * rows, nkv, hd)
    vp = oracle.normal_f16(batch * rows * nkv * hd, 72).reshape(batch * rows, nkv, hd)
    q = oracle.normal_f16(batch * n_q * nh * hd, 73).reshape(batch, n_q, nh, hd)
    offs = np.arange(batch, dtype=np.int64) * rows
    pre = oracle.attention_prefill(q, kp, vp, offs, n_q, start, nh, nkv, hd)
    for b in range(batch):
        for i in range(n_q):
            k = kp[offs[b]: offs[b] + rows]
            v = vp[offs[b]: offs[b] + rows]
            step = oracle.attention(q[b, i], k, v, nh, nkv, hd, start + i + 1)
            assert np.array_equal(pre[b, i], step), (b, i)
