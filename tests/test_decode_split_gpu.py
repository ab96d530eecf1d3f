"""The batched decode's work split under each of its settings, against the
oracle (kernels/sparse_attn.wgsl:32-113, kernels/kv_append.wgsl:13-18).

A batch's flattened split charges each (sequence, kv head) pair its rows plus
a fixed cost, rounded up to whole pairs of stages, so a CTA's range can start
or end in a pair's padding and hold no rows there.  These cases run ragged
batches (empty sequences, one-row sequences, 63/64/65 rows, long ones), the
fused append, and the shard partial with its merge under the default split,
pieces cut at any row (NWD_DECODE_PAIR_PAD=0), rows only (NWD_DECODE_PAIR_COST=0)
and costs large enough that most range ends fall in padding.  The tuning is
read once per process, so each setting runs in a child process.
"""
from __future__ import annotations

import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))

CHILD = r"""
import importlib, sys
import numpy as np, torch
sys.path[:0] = [{repo!r}, {oracle!r}, {tests!r}]
import oracle as O
from tolerance import assert_attn_close
from devutil import to_dev, vals, bits
ops = importlib.import_module("nemotron-webgpu-decode_b200.ops")
engine = importlib.import_module("nemotron-webgpu-decode_b200.engine")
hd, nkv = 128, 8
rng = np.random.default_rng(11)
for nh, B, hi in ((32, 64, 3000), (40, 40, 6000), (32, 300, 200)):
    L = rng.integers(0, hi, B).astype(np.int32)
    L[:6] = [0, 1, 63, 64, 65, 0]
    caps = np.maximum(L, 1)
    offs = np.concatenate([[0], np.cumsum(caps)[:-1]]).astype(np.int64)
    rows = int(caps.sum())
    q = O.normal_f16(B * nh * hd, 200 + B)
    k = O.normal_f16(rows * nkv * hd, 201 + B)
    v = O.normal_f16(rows * nkv * hd, 202 + B)
    o = torch.full((B, nh, hd), 3.0, dtype=torch.float16, device="cuda")
    ops.attention_batched(to_dev(q, (B, nh, hd)), to_dev(k, (rows, nkv, hd)),
                          to_dev(v, (rows, nkv, hd)), torch.tensor(offs, device="cuda"),
                          torch.tensor(L, device="cuda"), o, nh, nkv, hd)
    ref = O.attention_batched(q, k, v, offs, L, nh, nkv, hd)
    assert_attn_close(vals(o), ref, f"ragged Hq={{nh}} B={{B}}")
    assert not vals(o)[L == 0].any()
# the fused append over a ragged batch, two steps
B, nh = 24, 32
L0 = rng.integers(0, 2500, B).astype(np.int32)
L0[:3] = [0, 63, 64]
att = engine.BatchedDecodeAttention(L0 + 2, nh, nkv, hd)
rows = att.pool_rows
k0 = O.normal_f16(rows * nkv * hd, 81).reshape(rows, nkv, hd)
v0 = O.normal_f16(rows * nkv * hd, 82).reshape(rows, nkv, hd)
att.k_pool.copy_(to_dev(k0, (rows, nkv, hd)))
att.v_pool.copy_(to_dev(v0, (rows, nkv, hd)))
att.lengths.copy_(torch.tensor(L0, device="cuda"))
offs = att.row_offset.cpu().numpy()
L = L0.copy()
for s in range(2):
    q = O.normal_f16(B * nh * hd, 90 + s)
    kn = O.normal_f16(B * nkv * hd, 95 + s).reshape(B, nkv, hd)
    vn = O.normal_f16(B * nkv * hd, 99 + s).reshape(B, nkv, hd)
    out = att.step(to_dev(q, (B, nh, hd)), to_dev(kn), to_dev(vn))
    for b in range(B):
        k0[offs[b] + L[b]] = kn[b]
        v0[offs[b] + L[b]] = vn[b]
    L += 1
    assert_attn_close(vals(out), O.attention_batched(q, k0, v0, offs, L, nh, nkv, hd),
                      f"fused append step {{s}}")
assert np.array_equal(bits(att.k_pool), k0) and np.array_equal(bits(att.v_pool), v0)
assert att.workspace.check() == 0
# a sequence's rows in three shards: partials, then the merge
nh, Lr = 32, 20000
q = O.normal_f16(nh * hd, 41)
k = O.normal_f16(Lr * nkv * hd, 42)
v = O.normal_f16(Lr * nkv * hd, 43)
dq, dk, dv = to_dev(q, (1, nh, hd)), to_dev(k, (Lr, nkv, hd)), to_dev(v, (Lr, nkv, hd))
cuts = [0, 5000, 5001, Lr]
po = torch.empty(3, 1, nh, hd, dtype=torch.float32, device="cuda")
pml = torch.empty(3, 1, nh, 2, dtype=torch.float32, device="cuda")
for i in range(3):
    ops.attention_partial(dq, dk, dv, torch.tensor([cuts[i]], dtype=torch.int64, device="cuda"),
                          torch.tensor([cuts[i + 1] - cuts[i]], dtype=torch.int32, device="cuda"),
                          po[i], pml[i], nh, nkv, hd)
o = torch.empty(1, nh, hd, dtype=torch.float16, device="cuda")
ops.merge(po, pml, o)
assert_attn_close(vals(o)[0], O.attention(q, k, v, nh, nkv, hd, Lr), "three shards merged")
print("ok")
"""


@pytest.mark.parametrize("env", [
    {},
    {"NWD_DECODE_PAIR_PAD": "0"},
    {"NWD_DECODE_PAIR_COST": "0"},
    {"NWD_DECODE_PAIR_COST": "3000"},
    {"NWD_DECODE_PAIR_COST": "700", "NWD_DECODE_MIN_CHUNK": "64"},
], ids=["default", "pad0", "cost0", "cost3000", "cost700-chunk64"])
def test_batched_split_settings(env):
    repo = os.path.dirname(HERE)
    code = CHILD.format(repo=repo, oracle=os.path.join(repo, "oracle"), tests=HERE)
    r = subprocess.run([sys.executable, "-c", code], env=dict(os.environ, **env),
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0 and r.stdout.strip().endswith("ok"), r.stdout[-2000:] + r.stderr[-4000:]
