"""CPU models of the decode kernel's work split and stage-ring protocol.

csrc/decode.cu plans its work per CTA (stream-K ranges cut into pieces at
(sequence, kv head) pair boundaries, or one CTA per pair for small problems)
and runs a producer warp and NG consumer groups over a ring of NST mbarrier-
guarded stages.  Neither can be inspected on the GPU, so both are restated
here and checked:

* the planner: pieces partition every pair exactly, the ticket count of a
  pair (l - f + 1) equals the pieces that exist, and no CTA reuses a partial
  slot;
* the protocol, with PTX mbarrier semantics (a parity wait only compares the
  current phase's parity): every consumer group consumes exactly its own
  stages in order under random timing.  Without the "wait for the slot's
  previous release" gate the two-group ring consumes a stale stage; the model
  shows both.
"""
from __future__ import annotations

import random

import numpy as np
import pytest

TOK, NST, WPG = 64, 5, 4


# ---------------------------------------------------------------- planner

def pair_items(L, pad=1, cost=0):
    """Range items of a (sequence, kv head) pair of L rows: none when empty,
    else L + cost rounded up to pad (a batch's split; a single sequence runs
    with pad 1, cost 0)."""
    return 0 if L == 0 else -(-(L + cost) // pad) * pad


def plan(lens, nkv, grid, min_chunk=256, pair_max=512, split_k=0, pad=1, cost=0):
    """Pieces (cta, b, hkv, t0, t1, complete, f, l) as decode_kernel walks them.

    split_k > 0: CTA i takes piece i % k of pair i / k (the host's choice for a
    single sequence); otherwise one CTA per pair for small problems, else the
    flattened equal-range split over pair_items(L) items per pair, ranges a
    multiple of pad."""
    B = len(lens)
    S = [0]
    for L in lens:
        S.append(S[-1] + pair_items(L, pad, cost))
    T = nkv * S[B]
    if split_k == 0 and B * nkv <= grid and max(lens) <= pair_max:
        split_k = 1
    W = max((T + grid - 1) // grid, min_chunk)
    W = -(-W // pad) * pad
    out = []
    for i in range(grid):
        if split_k:
            pair, j = divmod(i, split_k)
            if pair < B * nkv:
                b, h = divmod(pair, nkv)
                L = lens[b]
                t0, t1 = j * L // split_k, (j + 1) * L // split_k
                if t1 > t0:
                    out.append((i, b, h, t0, t1, split_k == 1, pair * split_k,
                                pair * split_k + split_k - 1))
            continue
        x0, x1 = min(T, i * W), min(T, i * W + W)
        if x0 >= x1:
            continue
        b = max(j for j in range(B) if S[j] <= x0 // nkv)
        V, L = S[b + 1] - S[b], lens[b]
        h, t0 = divmod(x0 - nkv * S[b], V)
        pstart, x = x0 - t0, x0

        def next_pair(b, h):
            h += 1
            if h == nkv:
                h = 0
                b += 1
                while b + 1 < B and S[b + 1] == S[b]:
                    b += 1
            return b, h, S[b + 1] - S[b], lens[b]

        if t0 >= L:  # starts past the pair's rows
            x = pstart + V
            if x < x1:
                b, h, V, L = next_pair(b, h)
            pstart, t0 = x, 0
        f = pstart // W
        while x < x1:
            ln = min(L - t0, x1 - x)
            t1 = t0 + ln
            l = i if t1 == L else (pstart + L - 1) // W
            out.append((i, b, h, t0, t1, t0 == 0 and t1 == L, f, l))
            x = pstart + V
            if t1 < L or x >= x1:
                break
            b, h, V, L = next_pair(b, h)
            pstart, t0, f = x, 0, i
    return out, S


def check_plan(lens, nkv, grid, **kw):
    pieces, S = plan(lens, nkv, grid, **kw)
    cover, slots = {}, set()
    for (i, b, h, t0, t1, comp, f, l) in pieces:
        assert 0 <= t0 < t1 <= lens[b]
        cover.setdefault((b, h), []).append((t0, t1, i, f, l))
        if not comp:
            s = 2 * i + (0 if t0 > 0 else 1)
            assert s not in slots, "partial slot reused"
            slots.add(s)
    for b, L in enumerate(lens):
        for h in range(nkv):
            if L == 0:
                assert (b, h) not in cover
                continue
            ps = sorted(cover[(b, h)])
            assert ps[0][0] == 0 and ps[-1][1] == L
            assert all(a[1] == c[0] for a, c in zip(ps, ps[1:]))
            f, l = ps[0][3], ps[0][4]
            assert all(p[3] == f and p[4] == l for p in ps)
            if len(ps) > 1:
                assert l - f + 1 == len(ps)
                assert [p[2] for p in ps] == list(range(f, l + 1))
    return pieces


def host_split(L, nkv, sms=148, min_chunk=256, pair_max=512):
    """The host's choice for a single sequence: (grid, k)."""
    k = 1 if L <= pair_max else max(1, min(sms // nkv, -(-L // min_chunk)))
    return nkv * k, k


def test_planner_single_sequence_aligned_split():
    for L in (1, 151, 512, 513, 1024, 4097, 32768, 262144, 1 << 20):
        for nkv in (1, 8, 16):
            grid, k = host_split(L, nkv)
            pieces = check_plan([L], nkv, grid, split_k=k)
            # every CTA holds at most one piece: no CTA straddles two kv heads
            ctas = [p[0] for p in pieces]
            assert len(ctas) == len(set(ctas))


def test_planner_bench_shapes():
    check_plan([262144], 8, 148)
    check_plan([32768], 8, 148)
    check_plan([151], 8, 8)  # engine trace: one CTA per kv head
    lens = np.random.default_rng(3).integers(512, 8193, 256) + 1
    pieces = check_plan([int(x) for x in lens], 8, 148)
    per_cta = {}
    for p in pieces:
        per_cta.setdefault(p[0], 0)
        per_cta[p[0]] += p[4] - p[3]
    # unpadded: every CTA streams the same rows (the last one the remainder)
    sizes = sorted(per_cta.values())
    assert sizes[-1] - sizes[1] <= 0


def _stages(pieces, ng=2):
    """Stages each CTA issues: a piece's tiles rounded up to a multiple of ng."""
    per = {}
    for (i, b, h, t0, t1, *_r) in pieces:
        n = -(-(t1 - t0) // TOK)
        per[i] = per.get(i, 0) + -(-n // ng) * ng
    return per


def test_planner_padded_split_balances_stages_on_config3():
    """The batch split as the kernel runs it (pairs padded to 2 stages): cut
    points fall on whole stage pairs, so every CTA but the last issues the same
    number of stages; unpadded, a CTA whose range holds many pair ends issues
    up to 4 % more than the mean."""
    lens = [int(x) for x in np.random.default_rng(3).integers(512, 8193, 256) + 1]
    flat = _stages(check_plan(lens, 8, 148))
    padded_pieces = check_plan(lens, 8, 148, pad=2 * TOK)
    padded = _stages(padded_pieces)
    assert max(flat.values()) > 1.03 * np.mean(list(flat.values()))
    W = -(-(8 * sum(pair_items(L, 2 * TOK) for L in lens) // 148) // (2 * TOK)) * 2 * TOK
    assert all(padded[i] == W // TOK for i in range(147))
    assert padded[147] <= W // TOK
    for (i, b, h, t0, t1, *_r) in padded_pieces:
        assert t0 % (2 * TOK) == 0 and (t1 % (2 * TOK) == 0 or t1 == lens[b])


def test_planner_padded_random_shapes():
    rng = np.random.default_rng(1)
    for _ in range(300):
        B = int(rng.integers(1, 120))
        hi = int(rng.choice([3, 100, 5000, 70000]))
        lens = [int(x) for x in rng.integers(0, hi, B)]
        if sum(lens) == 0:
            continue
        pad = int(rng.choice([64, 128]))
        cost = int(rng.choice([0, 64, 200, 1000]))
        pieces = check_plan(lens, int(rng.choice([1, 2, 8])), int(rng.choice([8, 37, 148])),
                            min_chunk=int(rng.choice([64, 256])), pad=pad, cost=cost)
        for (i, b, h, t0, t1, *_r) in pieces:
            assert t0 % pad == 0 and (t1 % pad == 0 or t1 == lens[b])


def prefetch_rows(L, nkv, grid, cta, split_k=0, min_chunk=256, cap=8, div=4):
    """The (kv head, first row) of the K/V tiles CTA `cta` prefetches into L2 before its
    dependency wait, for a single sequence of L rows: csrc/decode.cu's restatement."""
    T = nkv * L
    W = max((T + grid - 1) // grid, min_chunk)
    x0, x1 = min(T, cta * W), min(T, cta * W + W)
    x, xe = x0, x1
    if split_k:
        j, h = cta % split_k, cta // split_k
        x = h * L + j * L // split_k
        xe = h * L + (j + 1) * L // split_k if h < nkv else x
    budget = min(cap, ((xe - x) // TOK) // div) if xe > x else 0
    out = []
    while x < xe and budget > 0:
        h, t = divmod(x, L)
        n = min(L - t, xe - x)
        r = 0
        while r < n and budget > 0:
            out.append((h, t + r))
            r += TOK
            budget -= 1
        x += n
    return out


@pytest.mark.parametrize("L,nkv", [(2049, 8), (4096, 8), (16384, 8), (32768, 8), (262144, 8),
                                   (12000, 1), (9000, 2), (5000, 3)])
def test_prefetch_stays_inside_the_ctas_pieces(L, nkv):
    """Every tile a CTA prefetches starts on a row its own pieces stream (so the
    prefetch only moves bytes that CTA reads right after the wait), there are
    1 / div of its range's whole tiles (at most cap: half and 16 unclustered, a
    quarter and 8 clustered), and they are its first ones."""
    for (split, cap, div) in [(s, c, d) for s in (True, False) for c, d in ((16, 2), (8, 4))]:
        grid, k = host_split(L, nkv)
        if not split:
            grid, k = 148, 0
        pieces, _ = plan([L], nkv, grid, split_k=k)
        for cta in range(grid):
            mine = [(h, t0, t1) for (i, b, h, t0, t1, *_rest) in pieces if i == cta]
            tiles = prefetch_rows(L, nkv, grid, cta, split_k=k, cap=cap, div=div)
            rows = sum(t1 - t0 for _, t0, t1 in mine)
            assert len(tiles) == min(cap, (rows // TOK) // div)
            for h, r in tiles:
                assert any(h == ph and t0 <= r < t1 for ph, t0, t1 in mine)
            # the first tiles of the range, in stream order
            expect = []
            for h, t0, t1 in mine:
                expect += [(h, r) for r in range(t0, t1, TOK)]
            assert tiles == expect[:len(tiles)]


def test_planner_random_shapes():
    rng = np.random.default_rng(0)
    for _ in range(200):
        B = int(rng.integers(1, 200))
        hi = int(rng.choice([3, 100, 5000, 70000]))
        lens = [int(x) for x in rng.integers(0, hi, B)]
        if sum(lens) == 0:
            continue
        check_plan(lens, int(rng.choice([1, 2, 8])), int(rng.choice([8, 37, 148])),
                   min_chunk=int(rng.choice([64, 256])))


# ---------------------------------------------------------------- protocol

class Bar:
    """mbarrier: arrival count, transaction bytes, phase; parity waits."""

    def __init__(self, count):
        self.count, self.pending, self.tx, self.phase = count, count, 0, 0

    def arrive(self, tx=0):
        self.tx += tx
        self.pending -= 1
        self._step()

    def complete_tx(self, n):
        self.tx -= n
        self._step()

    def _step(self):
        if self.pending == 0 and self.tx == 0:
            self.phase += 1
            self.pending = self.count

    def passed(self, parity):  # mbarrier.try_wait.parity
        return (self.phase & 1) != parity


def simulate(piece_stages, ngroups, gate, seed):
    rng = random.Random(seed)
    full = [Bar(1) for _ in range(NST)]
    empty = [Bar(WPG) for _ in range(NST)]
    csync = Bar(WPG * ngroups * 32)
    prog = []
    for k, n in enumerate(piece_stages):
        n2 = -(-n // ngroups) * ngroups
        syncs = 2 + 3 * (k % 2)  # complete pieces: 2 syncs; partial pieces: 5
        for s in range(n2):
            prog.append((s < n, s + ngroups >= n2, syncs))
    prog += [None] * ngroups
    hdr = [None] * NST
    flight = []

    def producer():
        slot = phase = 0
        for c, op in enumerate(prog):
            while not empty[slot].passed(phase ^ 1):
                yield
            hdr[slot] = (c, op)
            if op is not None and op[0]:
                full[slot].arrive(tx=32768)
                flight.append([slot, rng.choice([1, 3, 10, 80, 400])])
            else:
                full[slot].arrive()
            slot += 1
            if slot == NST:
                slot, phase = 0, phase ^ 1
            yield

    def consumer(g):
        slot, phase, cph, expect = g, 0, 0, g
        while True:
            if gate and ngroups > 1:
                while not empty[slot].passed(phase ^ 1):
                    yield
            while not full[slot].passed(phase):
                yield
            c, op = hdr[slot]
            if c != expect:
                raise AssertionError(f"group {g} consumed stage {c}, expected {expect}")
            expect += ngroups
            if op is None:
                return
            for _ in range(rng.randint(0, 3)):
                yield
            empty[slot].arrive()
            slot += ngroups
            if slot >= NST:
                slot, phase = slot - NST, phase ^ 1
            if op[1]:
                for _ in range(op[2]):
                    for _ in range(32):
                        csync.arrive()
                    while not csync.passed(cph):
                        yield
                    cph ^= 1

    actors = [producer()] + [consumer(g) for g in range(ngroups) for _ in range(WPG)]
    alive, steps = list(actors), 0
    while alive:
        steps += 1
        assert steps < 2_000_000, "deadlock"
        for f in list(flight):
            f[1] -= 1
            if f[1] <= 0:
                full[f[0]].complete_tx(32768)
                flight.remove(f)
        a = rng.choice(alive)
        try:
            next(a)
        except StopIteration:
            alive.remove(a)


@pytest.mark.parametrize("ngroups", [1, 2])
def test_ring_protocol(ngroups):
    for seed in range(40):
        rng = random.Random(seed)
        pieces = [rng.choice([1, 2, 3, 4, 5, 7, 12, 40]) for _ in range(rng.randint(1, 10))]
        simulate(pieces, ngroups, gate=True, seed=seed)


def test_two_groups_without_gate_consume_stale_stage():
    failures = 0
    for seed in range(40):
        rng = random.Random(seed)
        pieces = [rng.choice([1, 2, 3, 4, 5, 7, 12, 40]) for _ in range(rng.randint(1, 10))]
        try:
            simulate(pieces, 2, gate=False, seed=seed)
        except AssertionError:
            failures += 1
    assert failures > 0
