"""Both consumer-group configurations of the decode kernel (one group of four
warps, two groups taking alternate stages) against the oracle.

The library picks the group count by problem size; NWD_DECODE_GROUPS forces
it.  The setting is read once per process, so each case runs in a child
process.
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
ops = importlib.import_module("nemotron-webgpu-decode_b200.ops")
def dev(b, shape):
    return torch.from_numpy(b.view(np.float16).copy()).reshape(shape).cuda()
hd = 128
# single sequences: pair mode, split pairs, long
for nh, nkv, L in [(40, 8, 151), (32, 8, 1000), (40, 8, 4096), (32, 8, 20000), (8, 1, 3000)]:
    q = O.normal_f16(nh * hd, L); k = O.normal_f16(L * nkv * hd, L + 1); v = O.normal_f16(L * nkv * hd, L + 2)
    o = torch.empty(nh, hd, dtype=torch.float16, device="cuda")
    ops.attention(dev(q, (nh, hd)), dev(k, (L, nkv, hd)), dev(v, (L, nkv, hd)), o, ops.AttnParams(nh, nkv, hd, L))
    assert_attn_close(o.float().cpu().numpy(), O.attention(q, k, v, nh, nkv, hd, L), f"single L={{L}}")
# ragged batch with empty sequences, fused append
rng = np.random.default_rng(5)
B, nh, nkv = 40, 40, 8
L = rng.integers(0, 2500, B).astype(np.int32); L[:3] = [0, 1, 64]
caps = L + 1
offs = np.concatenate([[0], np.cumsum(caps)[:-1]]).astype(np.int64)
rows = int(caps.sum())
q = O.normal_f16(B * nh * hd, 1); k = O.normal_f16(rows * nkv * hd, 2); v = O.normal_f16(rows * nkv * hd, 3)
kn = O.normal_f16(B * nkv * hd, 4).reshape(B, nkv, hd); vn = O.normal_f16(B * nkv * hd, 5).reshape(B, nkv, hd)
dk, dv = dev(k, (rows, nkv, hd)), dev(v, (rows, nkv, hd))
o = torch.empty(B, nh, hd, dtype=torch.float16, device="cuda")
ops.kv_append_attention_batched(dev(q, (B, nh, hd)), dev(kn, (B, nkv, hd)), dev(vn, (B, nkv, hd)), dk, dv,
    torch.tensor(offs, device="cuda"), torch.tensor(L, device="cuda"), o, nh, nkv, hd)
kh = k.reshape(rows, nkv, hd).copy(); vh = v.reshape(rows, nkv, hd).copy()
for b in range(B):
    kh[offs[b] + L[b]] = kn[b]; vh[offs[b] + L[b]] = vn[b]
assert_attn_close(o.float().cpu().numpy(), O.attention_batched(q, kh, vh, offs, L + 1, nh, nkv, hd), "batched append")
assert np.array_equal(dk.cpu().numpy().view(np.uint16), kh)
print("ok")
"""


@pytest.mark.parametrize("groups", ["1", "2"])
def test_decode_groups(groups):
    repo = os.path.dirname(HERE)
    code = CHILD.format(repo=repo, oracle=os.path.join(repo, "oracle"), tests=HERE)
    env = dict(os.environ, NWD_DECODE_GROUPS=groups)
    r = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True,
                       timeout=600)
    assert r.returncode == 0 and r.stdout.strip().endswith("ok"), r.stdout[-2000:] + r.stderr[-4000:]
