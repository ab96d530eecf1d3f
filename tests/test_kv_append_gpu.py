"""kv_append on the GPU is bit-exact against kernels/kv_append.wgsl:13-18 (oracle)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from devutil import bits, to_dev

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("n_kv,hd,cap,seq", [(8, 128, 256, 0), (8, 128, 256, 151), (8, 128, 256, 255),
                                             (2, 128, 7, 6), (3, 5, 9, 4)])
def test_kv_append_bit_exact(ops, oracle, n_kv, hd, cap, seq):
    cache_h = oracle.normal_f16(cap * n_kv * hd, 100 + seq).reshape(cap, n_kv, hd)
    src_h = oracle.normal_f16(n_kv * hd, 200 + seq)
    cache = to_dev(cache_h)
    ops.kv_append(to_dev(src_h), cache, ops.KvParams(seq, n_kv, hd))
    torch.cuda.synchronize()
    ref = cache_h.copy()
    oracle.kv_append(src_h, ref, seq, n_kv, hd)
    assert np.array_equal(bits(cache), ref)  # whole cache: row seq written, others untouched


def test_kv_append_kv_pair(ops, oracle):
    n_kv, hd, cap, seq = 8, 128, 256, 77
    kc_h = oracle.normal_f16(cap * n_kv * hd, 1).reshape(cap, n_kv, hd)
    vc_h = oracle.normal_f16(cap * n_kv * hd, 2).reshape(cap, n_kv, hd)
    ks, vs = oracle.normal_f16(n_kv * hd, 3), oracle.normal_f16(n_kv * hd, 4)
    kc, vc = to_dev(kc_h), to_dev(vc_h)
    ops.kv_append_kv(to_dev(ks), to_dev(vs), kc, vc, ops.KvParams(seq, n_kv, hd))
    oracle.kv_append(ks, kc_h, seq, n_kv, hd)
    oracle.kv_append(vs, vc_h, seq, n_kv, hd)
    assert np.array_equal(bits(kc), kc_h) and np.array_equal(bits(vc), vc_h)


def test_kv_append_range_error_launches_nothing(ops, oracle):
    cache = torch.zeros(4, 8, 128, dtype=torch.float16, device="cuda")
    src = torch.ones(1024, dtype=torch.float16, device="cuda")
    with pytest.raises(ops.NwdError, match="seq 4 exceeds maxSeq 4"):
        ops.kv_append(src, cache, ops.KvParams(4, 8, 128))
    torch.cuda.synchronize()
    assert not cache.any()


def test_kv_append_batched(ops, oracle):
    B, n_kv, hd = 6, 8, 128
    caps = np.array([5, 1, 9, 3, 4, 2])
    offs = np.concatenate([[0], np.cumsum(caps)[:-1]]).astype(np.int64)
    rows = int(caps.sum())
    pos = np.array([0, 0, 8, 2, 4, 1], np.int32)  # sequence 4: pos 4 in a region of 4 rows is
    # still inside the pool (row offs[4]+4 = offs[5]); the last one, row 24, is the pool's last
    pool_k = oracle.normal_f16(rows * n_kv * hd, 9).reshape(rows, n_kv, hd)
    pool_v = oracle.normal_f16(rows * n_kv * hd, 10).reshape(rows, n_kv, hd)
    ks = oracle.normal_f16(B * n_kv * hd, 11).reshape(B, n_kv, hd)
    vs = oracle.normal_f16(B * n_kv * hd, 12).reshape(B, n_kv, hd)
    dk, dv = to_dev(pool_k), to_dev(pool_v)
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    ops.kv_append_batched(to_dev(ks), to_dev(vs), dk, dv, torch.tensor(offs, device="cuda"),
                          torch.tensor(pos, device="cuda"), err_count=err)
    for b in range(B):
        pool_k[offs[b] + pos[b]] = ks[b]
        pool_v[offs[b] + pos[b]] = vs[b]
    assert np.array_equal(bits(dk), pool_k) and np.array_equal(bits(dv), pool_v)
    assert int(err.item()) == 0
    # out-of-pool rows are skipped and counted
    bad = np.array([0, 0, 0, 0, 0, 99], np.int32)
    before = bits(dk).copy()
    ops.kv_append_batched(to_dev(ks), to_dev(vs), dk, dv, torch.tensor(offs, device="cuda"),
                          torch.tensor(bad, device="cuda"), err_count=err)
    assert int(err.item()) == 1
    after = bits(dk)
    for b in range(5):
        before[offs[b]] = ks[b]
    assert np.array_equal(after, before)


def test_generator_bit_exact(ops, oracle, golden):
    for k in golden.files:
        if not k.startswith("gen/"):
            continue
        seed, off = map(int, k[4:].split("_"))
        t = torch.empty(64, dtype=torch.float16, device="cuda")
        ops.fill_normal(t, seed, off)
        assert np.array_equal(bits(t), golden[k]), k
    n = 3_000_001
    t = torch.empty(n, dtype=torch.float16, device="cuda")
    ops.fill_normal(t, 5, 123)
    assert np.array_equal(bits(t), oracle.normal_f16(n, 5, 123))
