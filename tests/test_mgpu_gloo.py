"""Multi-rank host logic on CPU (gloo, world size 2): the sharded long-context
step (shard bounds, all-gather layout, merge in rank order) and the bench's
cross-rank timing reduction and sequence sharding.  The GPU kernels are
replaced by the oracle here; the same code paths run over NCCL on GPUs."""
from __future__ import annotations

import json
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

import mp_workers

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run(fn, world, tmp_path):
    mp.spawn(fn, args=(world, _port(), REPO, str(tmp_path)), nprocs=world, join=True)
    return [json.load(open(tmp_path / f"rank{r}.json")) for r in range(world)]


@pytest.mark.parametrize("world", [2, 3])
def test_sharded_decode_matches_unsharded(tmp_path, world):
    res = _run(mp_workers.sharded_decode_worker, world, tmp_path)
    for r in res:
        assert r["err"] < 1e-5, r
    # every rank holds the same merged output
    assert len({r["out0"] for r in res}) == 1
    # shards are contiguous, in rank order, and cover every sequence
    for b, L in enumerate([1000, 37, 513]):
        rows = [r["rows"][b] for r in res]
        assert rows[0][0] == 0 and rows[-1][1] == L
        assert all(a[1] == c[0] for a, c in zip(rows, rows[1:]))


def test_bench_rank_helpers(tmp_path):
    res = _run(mp_workers.max_over_ranks_worker, 2, tmp_path)
    for r in res:
        assert r["vals"] == [2.0, 10.0]  # max over ranks, element-wise
        assert r["weak_n"] == 256         # weak scaling: each GPU runs a full batch
    assert res[0]["seeds"] != res[1]["seeds"]
    # strong scaling: the 256 sequences split between the ranks, balanced by rows
    L = np.random.default_rng(3).integers(512, 8193, 256)
    assert sorted(res[0]["strong"] + res[1]["strong"]) == sorted(int(x) for x in L)
    s0, s1 = sum(res[0]["strong"]), sum(res[1]["strong"])
    assert abs(s0 - s1) <= 8192, (s0, s1)


def test_missing_rank_ends_the_step_with_an_error(tmp_path):
    """A rank that stops posting its shard partials (host-side injection) makes the
    other ranks' sharded step fail once the process group's deadline passes, instead of
    waiting for ever; no GPU is involved."""
    res = _run(mp_workers.missing_rank_worker, 2, tmp_path)
    assert res[1] == {"left": True}
    r0 = res[0]
    assert r0["status"] != "completed", r0
    assert r0["elapsed"] < 10 * r0["deadline"], r0
