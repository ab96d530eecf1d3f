"""The single-sequence split-KV decode with its pieces merged inside a
thread-block cluster over distributed shared memory, against the oracle
(kernels/sparse_attn.wgsl:32-113), and the same calls with the cluster merge
turned off (workspace partials + merge ticket).

A single sequence cut into k pieces per kv head runs each kv head's pieces as
one cluster (up to 16 CTAs, as many as fit for every kv head at once).  With
the short-sequence kernel turned off (NWD_DECODE_SHORT_ROWS=0) the lengths
below give cluster sizes 3 to 10 at 8 kv heads and 11 to 16 at 2 kv heads, plus
40 kv heads (group 1), group 8, and lengths past the clustered range.  The
tuning is read once per process, so each setting runs in a child process.
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
cases = [(40, 8, L) for L in (600, 700, 900, 1100, 1300, 1500, 1700, 2000, 2100, 2400, 2600,
                              2900, 3100, 3300, 3400, 3600, 4096, 5000, 33000)]
cases += [(40, 40, 3000), (64, 8, 3000), (32, 8, 4097), (32, 8, 9000)]
# two kv heads: clusters of 11 to 16 fit twice over
cases += [(8, 2, L) for L in (2700, 3000, 3300, 3500, 3800, 4096)]
for nh, nkv, L in cases:
    q = O.normal_f16(nh * hd, L); k = O.normal_f16(L * nkv * hd, L + 1); v = O.normal_f16(L * nkv * hd, L + 2)
    dq, dk, dv = dev(q, (nh, hd)), dev(k, (L, nkv, hd)), dev(v, (L, nkv, hd))
    ref = O.attention(q, k, v, nh, nkv, hd, L)
    outs = []
    for rep in range(2):
        o = torch.full((nh, hd), 7.0, dtype=torch.float16, device="cuda")
        ops.attention(dq, dk, dv, o, ops.AttnParams(nh, nkv, hd, L))
        outs.append(o.cpu())
        assert_attn_close(o.float().cpu().numpy(), ref, f"Hq={{nh}} Hkv={{nkv}} L={{L}} call {{rep}}")
    assert torch.equal(outs[0], outs[1]), f"L={{L}}: repeated calls differ"
# the engine step with the append fused, at a split length
nh, nkv, cap, seq = 40, 8, 4200, 4100
kc = O.normal_f16(cap * nkv * hd, 71).reshape(cap, nkv, hd); vc = O.normal_f16(cap * nkv * hd, 72).reshape(cap, nkv, hd)
q = O.normal_f16(nh * hd, 73); kn = O.normal_f16(nkv * hd, 74); vn = O.normal_f16(nkv * hd, 75)
dk, dv = dev(kc, (cap, nkv, hd)), dev(vc, (cap, nkv, hd))
o = torch.empty(nh, hd, dtype=torch.float16, device="cuda")
# writes row seq, attends seq + 1 rows (runtime.js:451-452)
ops.kv_append_attention(dev(q, (nh, hd)), dev(kn, (nkv, hd)), dev(vn, (nkv, hd)), dk, dv, o,
                        ops.AttnParams(nh, nkv, hd, seq))
kc[seq] = kn.reshape(nkv, hd); vc[seq] = vn.reshape(nkv, hd)
assert np.array_equal(dk.cpu().numpy().view(np.uint16), kc)
assert_attn_close(o.float().cpu().numpy(), O.attention(q, kc, vc, nh, nkv, hd, seq + 1), "fused append")
ws = ops._workspace(1, nh, nkv, hd, torch.device("cuda", 0), None)
assert ws.check() == 0
print("ok")
"""


@pytest.mark.parametrize("cluster", ["16", "0"])
def test_single_sequence_cluster_merge(cluster):
    repo = os.path.dirname(HERE)
    code = CHILD.format(repo=repo, oracle=os.path.join(repo, "oracle"), tests=HERE)
    env = dict(os.environ, NWD_DECODE_SHORT_ROWS="0", NWD_DECODE_CLUSTER=cluster)
    r = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True,
                       timeout=600)
    assert r.returncode == 0 and r.stdout.strip().endswith("ok"), r.stdout[-2000:] + r.stderr[-4000:]
