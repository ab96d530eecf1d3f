"""The C ABI driven by a C++ host with no Python or PyTorch in the process
(``nwd_host``, built from ``nemotron-webgpu-decode_b200/host/nwd_host.cc``).

* The engine trace (config 1: Hq 40, Hkv 8, maxSeq 256, 24 prompt + 127 new
  tokens) in DecodeEngine.submitStep's order (engine/runtime.js:447-467), both
  as the fused step and as the reference's three dispatches
  (runtime.js:389-391), checked against oracle fixtures this test writes; the
  maxSeq guard (runtime.js:448) as a status and message; reset (:630-631).
* The long-context decode sharded over GPUs through nwd_mgpu_* (NCCL loaded by
  the library): one rank, and two ranks on two GPUs, against the float64 oracle.
* A rank that leaves between steps (two GPUs, NVLS off, nothing of the leaving
  rank in flight): the other rank's next step ends with an error status
  within its deadline and its context keeps working.
"""
from __future__ import annotations

import importlib
import json
import os
import subprocess

import numpy as np
import pytest
import torch

from tolerance import assert_attn_close, f16

pytestmark = pytest.mark.gpu

HOST = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                    "nemotron-webgpu-decode_b200", "nwd_host")


def _gpus() -> int:
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


def _child_env(exchange: str = "peer"):
    env = dict(os.environ)
    env["NCCL_NVLS_ENABLE"] = "0"  # no NVLink multicast objects bound to a rank that leaves
    env["NWD_MGPU_P2P"] = "1" if exchange == "peer" else "0"
    return env


def _run(args, timeout=300):
    assert os.path.exists(HOST), "nwd_host is not built (__graft_entry__.build())"
    p = subprocess.run([HOST] + args, capture_output=True, text=True, timeout=timeout,
                       env=_child_env())
    lines = [ln for ln in p.stdout.splitlines() if ln.startswith("{")]
    assert lines, f"no result line (rc {p.returncode}): {p.stdout[-800:]} {p.stderr[-800:]}"
    return p.returncode, json.loads(lines[-1])


def _trace_expected(oracle):
    hq, hkv, hd, cap, steps = 40, 8, 128, 256, 151
    qn, row = hq * hd, hkv * hd
    kc = np.zeros((cap, hkv, hd), np.uint16)
    vc = np.zeros((cap, hkv, hd), np.uint16)
    out = np.empty((steps, hq, hd), np.float32)
    for s in range(steps):
        q = oracle.normal_f16(qn, 101, s * qn)
        oracle.kv_append(oracle.normal_f16(row, 102, s * row), kc, s, hkv, hd)
        oracle.kv_append(oracle.normal_f16(row, 103, s * row), vc, s, hkv, hd)
        out[s] = oracle.attention(q, kc, vc, hq, hkv, hd, s + 1)
    return out


@pytest.mark.parametrize("fused", [1, 0])
def test_engine_trace_from_cpp_host(oracle, tmp_path, fused):
    ref = _trace_expected(oracle)
    exp, out = tmp_path / "expect.bin", tmp_path / "out.bin"
    ref.tofile(exp)
    rc, res = _run(["trace", "--out", str(out), "--expect", str(exp), "--fused", str(fused)])
    assert rc == 0 and res["ok"], res
    assert res["guard_status"] == "NWD_ERR_RANGE" and res["guard_seq"] == 256
    assert res["guard_message"] == "seq 256 exceeds maxSeq 256"  # runtime.js:448
    assert res["reset_step0_bit_exact"] and res["reset_rows_zero"]
    got = f16(np.fromfile(out, np.uint16)).reshape(ref.shape)
    assert_attn_close(got, ref, f"C++ host trace (fused={fused})")


def _mgpu_ref(oracle, B, L, hq, hkv):
    row = hkv * 128
    q = oracle.normal_f16(B * hq * 128, 5002).reshape(B, hq, 128)
    refs = []
    for b in range(B):
        k = oracle.normal_f16(L * row, 5000, b * L * row)
        v = oracle.normal_f16(L * row, 5001, b * L * row)
        refs.append(oracle.attention_batched(q[b], k, v, [0], [L], hq, hkv, 128, f64=True)[0])
    return np.stack(refs)


def _mgpu_ranks(world, tmp_path, extra, exchange="peer"):
    idf = tmp_path / "nccl.id"
    procs = []
    for r in range(world):
        args = [HOST, "mgpu", "--world", str(world), "--rank", str(r), "--device", str(r),
                "--id-file", str(idf)] + extra
        procs.append(subprocess.Popen(args, stdout=subprocess.PIPE, stderr=subprocess.PIPE,
                                      text=True, env=_child_env(exchange)))
    res = []
    for p in procs:
        try:
            so, se = p.communicate(timeout=300)
        except subprocess.TimeoutExpired:
            for q in procs:
                q.kill()
            raise
        lines = [ln for ln in so.splitlines() if ln.startswith("{")]
        assert lines, f"rank gave no result (rc {p.returncode}): {so[-600:]} {se[-600:]}"
        res.append((p.returncode, json.loads(lines[-1])))
    return res


@pytest.mark.parametrize("exchange", ["peer", "nccl"])
@pytest.mark.parametrize("world", [1, 2])
def test_sharded_decode_from_cpp_host(oracle, tmp_path, world, exchange):
    """Both exchanges: partials written into every rank's exchange buffer with a
    waiting merge (peer), and NCCL all-gather + merge (NWD_MGPU_P2P=0)."""
    if _gpus() < world:
        pytest.skip(f"needs {world} GPUs")
    B, L, hq, hkv = 2, 65536, 32, 8
    out = tmp_path / "o.bin"
    res = _mgpu_ranks(world, tmp_path, ["--batch", str(B), "--rows", str(L), "--heads", str(hq),
                                        "--kv-heads", str(hkv), "--steps", "3",
                                        "--out", str(out)], exchange)
    for rc, r in res:
        assert rc == 0 and r["ok"], r
        assert r["exchange"] == exchange, r
    got = f16(np.fromfile(out, np.uint16)).reshape(B, hq, 128)
    assert_attn_close(got, _mgpu_ref(oracle, B, L, hq, hkv),
                      f"sharded over {world} rank(s), {exchange} exchange")


@pytest.mark.parametrize("exchange", ["peer", "nccl"])
def test_rank_leaving_ends_the_next_step_with_an_error(tmp_path, exchange):
    if _gpus() < 2:
        pytest.skip("needs 2 GPUs")
    deadline = 2000
    res = _mgpu_ranks(2, tmp_path, ["--batch", "2", "--rows", "32768", "--steps", "3",
                                    "--leave-after", "1", "--step-deadline-ms", str(deadline),
                                    "--init-deadline-ms", "120000"], exchange)
    (rc0, r0), (rc1, r1) = res
    assert rc1 == 0 and r1.get("left_after") == 1, r1
    assert rc0 == 0 and r0["ok"], r0
    assert r0["failed_step_status"] in ("NWD_ERR_TIMEOUT", "NWD_ERR_NCCL"), r0
    assert r0["elapsed_ms"] < deadline + 10000, r0
    assert r0["after"] == "NWD_OK", r0  # the survivor's context still runs kernels


@pytest.mark.parametrize("exchange", ["peer", "nccl"])
def test_sharded_decode_python_over_the_c_abi(ops, oracle, monkeypatch, exchange):
    """mgpu.Communicator (the library's communicator) at world 1 in this process."""
    monkeypatch.setenv("NWD_MGPU_P2P", "1" if exchange == "peer" else "0")
    mgpu = importlib.import_module(ops.__name__.rsplit(".", 1)[0] + ".mgpu")
    uid = mgpu.share_unique_id(0)
    comm = mgpu.Communicator(uid, 1, 0, torch.cuda.current_device())
    B, L, hq, hkv = 2, 40000, 32, 8
    row = hkv * 128
    dev = torch.device("cuda", torch.cuda.current_device())
    kp = torch.empty(B * L, hkv, 128, dtype=torch.float16, device=dev)
    vp = torch.empty_like(kp)
    ops.fill_normal(kp, 5000)
    ops.fill_normal(vp, 5001)
    q = ops.fill_normal(torch.empty(B, hq, 128, dtype=torch.float16, device=dev), 5002)
    ro = torch.arange(B, dtype=torch.int64, device=dev) * L
    sl = torch.full((B,), L, dtype=torch.int32, device=dev)
    o = torch.empty(B, hq, 128, dtype=torch.float16, device=dev)
    nbytes = comm.workspace_bytes(B, hq, hkv, 128)
    ws = torch.zeros(nbytes + 256, dtype=torch.uint8, device=dev)
    wp = (ws.data_ptr() + 255) // 256 * 256
    comm.set_timing(True)
    comm.decode_step(q.data_ptr(), kp.data_ptr(), vp.data_ptr(), B * L, ro.data_ptr(),
                     sl.data_ptr(), o.data_ptr(), B, hq, hkv, 128, wp, nbytes,
                     torch.cuda.current_stream().cuda_stream)
    comm.sync()
    assert comm.exchange_mode() == exchange
    t_part, t_x = comm.step_times()
    assert t_part > 0 and t_x > 0
    # later steps reuse the exchange slots by parity: same result, bit for bit
    first = o.clone()
    for _ in range(3):
        comm.decode_step(q.data_ptr(), kp.data_ptr(), vp.data_ptr(), B * L, ro.data_ptr(),
                         sl.data_ptr(), o.data_ptr(), B, hq, hkv, 128, wp, nbytes,
                         torch.cuda.current_stream().cuda_stream)
    comm.sync()
    assert torch.equal(o, first)
    comm.close()
    qh = oracle.normal_f16(B * hq * 128, 5002).reshape(B, hq, 128)
    for b in range(B):
        k = oracle.normal_f16(L * row, 5000, b * L * row)
        v = oracle.normal_f16(L * row, 5001, b * L * row)
        ref = oracle.attention_batched(qh[b], k, v, [0], [L], hq, hkv, 128, f64=True)
        assert_attn_close(o[b:b + 1].float().cpu().numpy(), ref, f"world-1 communicator, seq {b}")
