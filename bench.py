#!/usr/bin/env python
"""Decode-attention bench: tokens/s and achieved HBM bandwidth on B200.

Default workload (config 3, the configuration the metric's 1/2/4/8-GPU
scaling is quoted on): 256 independent sequences, Hq=32, Hkv=8, d=128,
per-sequence KV lengths drawn uniformly from [512, 8192] (seed 3), stored
contiguously per sequence in one pool, fp16 q/K/V from the deterministic
N(0,1) generator.  One step = the engine's attention-layer step for every
sequence: append one K/V row at its position and attend over all of its rows
(one fused launch of the library's decode kernel).  Positions cycle over 16
rows so every step attends L_b+1 .. L_b+16 rows (the workload stays at config
3's lengths however many steps run).  On N GPUs the 256 sequences are split
across the GPUs, balanced by rows, with no communication (strong scaling;
``--scaling weak`` runs 256 sequences on every GPU instead).

The same line carries two sub-objects (skipped with ``--no-extras``):
``config5``, the long-context step (4 sequences x 1 048 576 rows, each
sequence's rows sharded over the N GPUs, the partials exchanged over peer
memory, or NCCL, and merged inside the library), with the exchange's measured
share of the step;
and ``config2``, the single-sequence length sweep on rank 0.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl nwd|reference]
                  [--config 3|1|2|4|5|6] [--scaling strong|weak] [--no-extras]

Other configs as lines of their own: 1 engine trace and 2 length sweep (single
sequence, CUDA-graph replay), 4 chunked causal prefill (tcgen05), 5 the
long-context step, 6 the model's 4 attention layers with their q4 projections
(q/k/v + append, attention, o_proj + residual).

``--impl reference`` times the reference's algorithm on the host CPU: the
reference is WGSL for a browser WebGPU device, which this machine cannot run,
so its CPU restatement (oracle/, all host threads) stands in for it, on a
bounded sample of the same workload.
"""
from __future__ import annotations

import argparse
import datetime
import importlib
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

REPO = os.path.dirname(os.path.abspath(__file__))
PKG = "nemotron-webgpu-decode_b200"
METRIC = "decode-attn tokens/s + achieved HBM TB/s vs B200 peak, at 1/2/4/8 GPUs"
HQ, HKV, HD = 32, 8, 128
POS_CYCLE = 16
FALLBACK_HBM_GBS = 6650.0


def peaks():
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def tensor_peak():
    """Dense bf16/fp16 TFLOP/s: the burst figure (a kernel timed alone)."""
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["bf16_tflops"]), "measured"
    except Exception:
        return 1590.0, "fallback"


def profiled_traffic(name: str):
    """dram bytes per launch from a committed ncu summary (profiles/<name>.txt), if any."""
    path = os.path.join(REPO, "profiles", name + ".txt")
    try:
        for line in open(path):
            if line.startswith("dram_bytes_per_launch"):
                return float(line.split()[-1])
    except OSError:
        pass
    return None


# ------------------------------------------------------------------ clocks

class ClockSampler:
    """nvidia-smi samples (every 200 ms) for one GPU, tagged with host time."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    NAMES = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]

    def __init__(self, gpu_id: str):
        self.rows = []
        self.proc = None
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", gpu_id, f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 8:
                self.rows.append((time.monotonic(), parts))

    def stop(self):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self, t0: float, t1: float):
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0,
                    "note": "nvidia-smi unavailable"}
        inside = [r for t, r in self.rows if t0 <= t <= t1]
        window = "timed"
        if len(inside) < 3:
            inside = [r for _, r in self.rows]
            window = "ramp+warmup+timed"
        def num(x):
            try:
                return float(x)
            except ValueError:
                return None
        sm = [num(r[0]) for r in inside if num(r[0]) is not None]
        mx = [num(r[1]) for r in inside if num(r[1]) is not None]
        pw = [num(r[2]) for r in inside if num(r[2]) is not None]
        reasons = set()
        for r in inside:
            for name, v in zip(self.NAMES, r[4:8]):
                if v.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None,
                "power_w_max": max(pw) if pw else None,
                "reasons": sorted(reasons), "samples": len(inside), "window": window}


# ------------------------------------------------------------------ setup


def start_clocks(torch, dev, rank):
    """nvidia-smi sampling of rank 0's GPU (None on the other ranks)."""
    if rank != 0:
        return None
    uuid = str(torch.cuda.get_device_properties(dev).uuid)
    sampler = ClockSampler(uuid if uuid.startswith("GPU-") else "GPU-" + uuid)
    # short timed regions: have at least the first sample before the warm-up starts
    t = time.monotonic()
    while sampler.proc and not sampler.rows and time.monotonic() - t < 5.0:
        time.sleep(0.05)
    return sampler

def import_pkg():
    if REPO not in sys.path:
        sys.path.insert(0, REPO)
    return importlib.import_module(PKG + ".ops")


def import_oracle():
    p = os.path.join(REPO, "oracle")
    if p not in sys.path:
        sys.path.insert(0, p)
    import oracle
    oracle.build()
    # all host cores this process may run on (torchrun sets OMP_NUM_THREADS=1)
    try:
        cores = len(os.sched_getaffinity(0))
    except AttributeError:
        cores = os.cpu_count() or 1
    oracle.set_num_threads(cores)
    return oracle


def config3_lengths():
    return np.random.default_rng(3).integers(512, 8193, 256).astype(np.int64)


def strong_assignment(L, world):
    """Sequence indices of each rank for a strong split, balanced by rows: the
    longest sequence first, each to the rank holding the fewest rows so far
    (ties to the lower rank).  The step time is the slowest rank's, so rows,
    not sequence counts, are what must be even."""
    sums = [0] * world
    sets = [[] for _ in range(world)]
    for i in np.argsort(-np.asarray(L), kind="stable"):
        r = min(range(world), key=lambda x: (sums[x], x))
        sets[r].append(int(i))
        sums[r] += int(L[i])
    return [sorted(s) for s in sets]


def rank_lengths(rank, world, scaling, batch=None):
    L = config3_lengths()
    if batch:
        L = L[:batch]  # profiling captures: the first `batch` sequences
    if scaling == "strong" and world > 1:
        return L[strong_assignment(L, world)[rank]]
    return L


def seeds_for(rank):
    return {"k": 3000 + 100 * rank, "v": 3001 + 100 * rank, "q": 3002 + 100 * rank,
            "kn": 3003 + 100 * rank, "vn": 3004 + 100 * rank}


def max_over_ranks(values, dist=None, device=None):
    """Element-wise max of per-rank floats (timings) across ranks (no-op at N=1)."""
    import torch
    t = torch.tensor([float(v) for v in values], dtype=torch.float64, device=device)
    if dist is not None and dist.is_initialized() and dist.get_world_size() > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return [float(x) for x in t.tolist()]


def sum_over_ranks(values, dist=None, device=None):
    """Element-wise sum of per-rank numbers (work counts) across ranks (no-op at N=1)."""
    import torch
    t = torch.tensor([float(v) for v in values], dtype=torch.float64, device=device)
    if dist is not None and dist.is_initialized() and dist.get_world_size() > 1:
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return [float(x) for x in t.tolist()]


def step_bytes(L_attended):
    """Algorithmic HBM bytes of one step: K+V rows read, q read + o write, new K/V row read+write."""
    B = len(L_attended)
    return float(4096 * np.sum(L_attended) + B * (2 * HQ * HD * 2 + 4 * HKV * HD * 2))


def hold_stream(torch, steps, host_us_per_step=40.0):
    """Keep the current stream busy with a bounded spin (torch.cuda._sleep, a
    fixed number of clock cycles) while the host enqueues `steps` timed
    launches.  The timed window starts after it, so it measures the GPU running
    the steps back to back, not Python's launch rate: a 0.1 ms step (config 3
    on 8 GPUs) otherwise idles whenever the process is descheduled before the
    host has run ahead of the GPU.  Skipped if this PyTorch lacks the helper."""
    sleep = getattr(torch.cuda, "_sleep", None)
    if sleep is not None:
        sleep(int(min(steps * host_us_per_step * 1e-6 * 2.0e9, 4.0e9)))


class Config3:
    def __init__(self, ops, torch, rank, world, scaling, dev, batch=None):
        self.ops, self.torch = ops, torch
        self.L = rank_lengths(rank, world, scaling, batch)
        self.B = len(self.L)
        self.caps = self.L + POS_CYCLE
        self.offs = np.concatenate([[0], np.cumsum(self.caps)[:-1]]).astype(np.int64)
        self.rows = int(self.caps.sum())
        sd = seeds_for(rank)
        self.seeds = sd
        f16 = torch.float16
        self.k_pool = torch.empty(self.rows, HKV, HD, dtype=f16, device=dev)
        self.v_pool = torch.empty_like(self.k_pool)
        ops.fill_normal(self.k_pool, sd["k"])
        ops.fill_normal(self.v_pool, sd["v"])
        self.q = ops.fill_normal(torch.empty(self.B, HQ, HD, dtype=f16, device=dev), sd["q"])
        self.kn = ops.fill_normal(torch.empty(self.B, HKV, HD, dtype=f16, device=dev), sd["kn"])
        self.vn = ops.fill_normal(torch.empty(self.B, HKV, HD, dtype=f16, device=dev), sd["vn"])
        self.o = torch.empty(self.B, HQ, HD, dtype=f16, device=dev)
        self.row_offset = torch.tensor(self.offs, device=dev)
        pos = np.stack([self.L + j for j in range(POS_CYCLE)]).astype(np.int32)  # [cycle, B]
        self.pos_host = pos
        self.pos = torch.tensor(pos, device=dev)
        self.ws = ops.Workspace(self.B, HQ, HKV, HD, dev)

    def step(self, s, q=None, kn=None, vn=None, pos=None, o=None):
        self.ops.kv_append_attention_batched(
            self.q if q is None else q, self.kn if kn is None else kn,
            self.vn if vn is None else vn, self.k_pool, self.v_pool, self.row_offset,
            self.pos[s % POS_CYCLE] if pos is None else pos, self.o if o is None else o,
            HQ, HKV, HD, workspace=self.ws)

    def bytes_for(self, s):
        return step_bytes(self.pos_host[s % POS_CYCLE] + 1)


# ------------------------------------------------------------------ CPU legs

def cpu_sample(oracle, L, offs_unused, seeds, nseq):
    """Host copies of the first `nseq` sequences' K/V (same generator streams as the GPU pool)."""
    caps = L + POS_CYCLE
    offs = np.concatenate([[0], np.cumsum(caps)[:-1]]).astype(np.int64)
    sel = list(range(nseq))
    rows = int(sum(caps[b] for b in sel))
    k = np.empty((rows, HKV, HD), np.uint16)
    v = np.empty((rows, HKV, HD), np.uint16)
    loc = np.zeros(nseq, np.int64)
    r = 0
    for i, b in enumerate(sel):
        n = int(caps[b]) * HKV * HD
        k[r:r + caps[b]] = oracle.normal_f16(n, seeds["k"], int(offs[b]) * HKV * HD).reshape(-1, HKV, HD)
        v[r:r + caps[b]] = oracle.normal_f16(n, seeds["v"], int(offs[b]) * HKV * HD).reshape(-1, HKV, HD)
        loc[i] = r
        r += int(caps[b])
    q = oracle.normal_f16(nseq * HQ * HD, seeds["q"])
    kn = oracle.normal_f16(nseq * HKV * HD, seeds["kn"]).reshape(nseq, HKV * HD)
    vn = oracle.normal_f16(nseq * HKV * HD, seeds["vn"]).reshape(nseq, HKV * HD)
    return k, v, loc, q, kn, vn


def cpu_step(oracle, L, sample, s):
    """The reference's step on the CPU for the sample: kv_append K and V at the
    sequence's position (kv_append.wgsl), then attention over pos+1 rows (sparse_attn.wgsl)."""
    k, v, loc, q, kn, vn = sample
    n = len(loc)
    pos = (L[:n] + (s % POS_CYCLE)).astype(np.int64)
    for i in range(n):
        row = loc[i] + pos[i]
        k[row] = kn[i].reshape(HKV, HD)
        v[row] = vn[i].reshape(HKV, HD)
    return oracle.attention_batched(q, k, v, loc, (pos + 1).astype(np.int32), HQ, HKV, HD)


def cpu_baseline(oracle, L, seeds, seconds=10.0, nseq=8):
    sample = cpu_sample(oracle, L, None, seeds, nseq)
    cpu_step(oracle, L, sample, 0)  # warm
    t0 = time.perf_counter()
    steps = 0
    while True:
        cpu_step(oracle, L, sample, steps)
        steps += 1
        el = time.perf_counter() - t0
        if el >= seconds or steps >= 10000:
            break
    return {"value": nseq * steps / el, "unit": "tokens/s", "cores": oracle.num_threads(),
            "kind": "port",
            "sample": f"first {nseq} of the 256 config-3 sequences (L={list(map(int, L[:nseq]))}), "
                      f"{steps} steps of kv_append + attention in {el:.1f} s"}


def run_reference(args):
    """--impl reference: the reference algorithm (oracle port) on the host cores."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    oracle = import_oracle()
    L = config3_lengths()
    seeds = seeds_for(0)
    nseq = 16
    sample = cpu_sample(oracle, L, None, seeds, nseq)
    for s in range(args.warmup):
        cpu_step(oracle, L, sample, s)
    t0 = time.perf_counter()
    for s in range(args.steps):
        cpu_step(oracle, L, sample, args.warmup + s)
    el = time.perf_counter() - t0
    value = nseq * args.steps / el
    line = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * el / args.steps,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic", "impl": "reference",
        "config": {"workload": "config3-batched-ragged-decode (sample)", "heads": HQ,
                   "kv_heads": HKV, "head_dim": HD, "sample_sequences": nseq,
                   "lengths": list(map(int, L[:nseq]))},
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": oracle.num_threads(),
                         "kind": "port",
                         "sample": f"{nseq} of 256 sequences per step; the reference's WGSL needs a "
                                   "browser WebGPU device (unavailable on this box), so its CPU "
                                   "restatement in oracle/ is timed"},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ------------------------------------------------------------------ GPU arm

def e2e_config3(W, torch, dev, args, s, barrier):
    """Config 3 end to end through ops.kv_append_attention_batched (ctypes -> C ABI)
    with host buffers: per step, q / k_new / v_new / pos from pinned host memory
    (H2D) and o back to pinned host memory (D2H), read by the host.  Two buffer
    sets: step x's inputs cross on one copy stream while step x-1 computes, step
    x's o crosses on another while step x+1 computes; the host waits for step
    x-1's output event before issuing step x+1.  Device-timed from the first
    copy to the last output landing (events on the compute stream, which waits
    for both copy streams at the end)."""
    comp = torch.cuda.current_stream()
    cin, cout = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)
    pin = dict(pin_memory=True)
    q_h = W.q.cpu().pin_memory()
    kn_h = W.kn.cpu().pin_memory()
    vn_h = W.vn.cpu().pin_memory()
    pos_h = torch.tensor(W.pos_host).pin_memory()  # [cycle, B]
    o_h = [torch.empty(W.B, HQ, HD, dtype=torch.float16, **pin) for _ in range(2)]
    q_d = [torch.empty_like(W.q) for _ in range(2)]
    kn_d = [torch.empty_like(W.kn) for _ in range(2)]
    vn_d = [torch.empty_like(W.vn) for _ in range(2)]
    pos_d = [torch.empty(W.B, dtype=torch.int32, device=dev) for _ in range(2)]
    o_d = [torch.empty_like(W.o) for _ in range(2)]
    ev = lambda: torch.cuda.Event()  # noqa: E731
    in_ready = [ev(), ev()]
    done = [ev(), ev()]
    out_done = [ev(), ev()]
    used = [False, False]
    reads = []

    def step(x):
        i = x & 1
        with torch.cuda.stream(cin):
            if used[i]:
                cin.wait_event(done[i])  # buffer set i's previous step has read its inputs
            q_d[i].copy_(q_h, non_blocking=True)
            kn_d[i].copy_(kn_h, non_blocking=True)
            vn_d[i].copy_(vn_h, non_blocking=True)
            pos_d[i].copy_(pos_h[x % POS_CYCLE], non_blocking=True)
            in_ready[i].record(cin)
        comp.wait_event(in_ready[i])
        if used[i]:
            comp.wait_event(out_done[i])  # o_d[i] has been copied out
        W.step(x, q=q_d[i], kn=kn_d[i], vn=vn_d[i], pos=pos_d[i], o=o_d[i])
        done[i].record(comp)
        with torch.cuda.stream(cout):
            cout.wait_event(done[i])
            o_h[i].copy_(o_d[i], non_blocking=True)
            out_done[i].record(cout)
        used[i] = True
        # the host reads step x-1's result before it issues step x+1
        j = i ^ 1
        if prev[0] is not None:
            out_done[j].synchronize()
            reads.append(float(o_h[j][0, 0, 0]))
        prev[0] = x

    prev = [None]
    for _ in range(args.warmup):
        step(s)
        s += 1
    comp.wait_stream(cout)
    barrier()
    prev[0] = None
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(comp)
    cin.wait_stream(comp)
    for _ in range(args.steps):
        step(s)
        s += 1
    comp.wait_stream(cout)
    end.record(comp)
    end.synchronize()
    reads.append(float(o_h[(s - 1) & 1][0, 0, 0]))  # the last step's result
    barrier()
    h2d = W.B * (HQ * HD * 2 + 2 * HKV * HD * 2 + 4)
    d2h = W.B * HQ * HD * 2
    return {"ms": start.elapsed_time(end), "h2d": h2d, "d2h": d2h, "s": s,
            "finite": all(np.isfinite(reads))}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=300)
    ap.add_argument("--warmup", type=int, default=30)
    ap.add_argument("--impl", choices=["nwd", "reference"], default="nwd")
    ap.add_argument("--config", choices=["3", "1", "2", "4", "5", "6"], default="3",
                    help="workload configuration (6 = the attention layers with their q4 projections)")
    ap.add_argument("--scaling", choices=["weak", "strong"], default="strong",
                    help="config 3 at N>1: strong (the 256 sequences split across the GPUs, "
                         "balanced by rows) or weak (256 sequences on every GPU)")
    ap.add_argument("--no-extras", action="store_true",
                    help="config 3: skip the config-5 and config-2 sub-objects of the line")
    ap.add_argument("--ramp-seconds", type=float, default=1.0)
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--prefetch", action="store_true",
                    help="config 6: prefetch the next projections' weights into L2 on a side stream")
    ap.add_argument("--batch", type=int, default=None,
                    help="config 3: only the first N sequences (small profiling captures)")
    ap.add_argument("--kv-len", type=int, default=None,
                    help="config 2: only this length (small profiling captures)")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    if args.impl == "reference":
        return run_reference(args)

    import torch
    import torch.distributed as dist

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        if world == 1 and args.gpus > 1:
            print("run N>1 under torchrun (one process per GPU)", file=sys.stderr)
            return 2
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    ops = import_pkg()
    if args.config == "5":
        return run_config5(args, ops, torch, dist, dev, rank, world)
    if args.config == "4":
        return run_config4(args, ops, torch, dist, dev, rank, world)
    if args.config == "6":
        return run_config6(args, ops, torch, dist, dev, rank, world)
    if args.config != "3":
        return run_small_configs(args, ops, torch, dev, rank, world)

    W = Config3(ops, torch, rank, world, args.scaling, dev, args.batch)
    torch.cuda.synchronize()
    props = torch.cuda.get_device_properties(dev)
    sampler = ClockSampler("GPU-" + str(props.uuid) if not str(props.uuid).startswith("GPU-")
                           else str(props.uuid)) if rank == 0 else None

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    # clock ramp (untimed), then W warm-up steps, then K timed steps
    s = 0
    t_ramp = time.perf_counter()
    while time.perf_counter() - t_ramp < args.ramp_seconds:
        for _ in range(20):
            W.step(s)
            s += 1
        torch.cuda.synchronize()
    for _ in range(args.warmup):
        W.step(s)
        s += 1
    barrier()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0 = time.monotonic()
    hold_stream(torch, args.steps)
    start.record()
    s_first = s
    for _ in range(args.steps):
        W.step(s)
        s += 1
    end.record()
    end.synchronize()
    t1 = time.monotonic()
    barrier()
    ms = start.elapsed_time(end)
    step_bytes_timed = [W.bytes_for(x) for x in range(s_first, s)]

    # roofline pass: per-launch events around the decode kernel (same stream)
    R = min(args.steps, 50)
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(R)]
    rb = []
    for i in range(R):
        evs[i][0].record()
        W.step(s)
        evs[i][1].record()
        rb.append(W.bytes_for(s))
        s += 1
    torch.cuda.synchronize()
    launch_ms = [a.elapsed_time(b) for a, b in evs]
    kern_ms = statistics.mean(launch_ms)
    kern_gbs = statistics.mean(rb) / (kern_ms * 1e-3) / 1e9

    # e2e: host buffers through the public API, every step's inputs copied in from
    # pinned host memory and its output copied back and read by the host, all
    # inside the timed region.  Double-buffered: step x's inputs cross on a copy
    # stream while step x-1 computes, its output crosses on a second copy stream,
    # and the host waits for step x-1's output (not for the whole stream).
    e2e = None
    if not args.no_e2e:
        e2e = e2e_config3(W, torch, dev, args, s, barrier)
        s = e2e.pop("s")

    err = W.ws.check()
    if err:
        print(f"device error word {err} after the bench", file=sys.stderr)
        return 3
    if e2e and not e2e["finite"]:
        print("non-finite output read back in the e2e pass", file=sys.stderr)
        return 3

    # max over ranks (times), sums over ranks (work)
    ms_max, e2e_ms_max = max_over_ranks([ms, e2e["ms"] if e2e else 0.0], dist, dev)
    n_seq, bytes_timed, h2d, d2h = sum_over_ranks(
        [W.B, sum(step_bytes_timed), e2e["h2d"] if e2e else 0, e2e["d2h"] if e2e else 0],
        dist, dev)
    clocks = None
    if sampler:
        sampler.stop()
        clocks = sampler.summary(t0, t1)
    cpu_L, cpu_seeds = W.L, W.seeds
    del W
    torch.cuda.empty_cache()

    # the long-context sharded step and the single-sequence sweep, recorded in
    # the same line (every rank takes part in the sharded step)
    extra5 = extra2 = None
    if not args.no_extras:
        # an error here is recorded in the sub-object and costs the headline
        # nothing (every wait inside is bounded: the communicator's deadlines,
        # the process group's timeout)
        try:
            extra5 = measure_config5(args, ops, torch, dist, dev, rank, world, sub=True)
        except Exception as e:  # noqa: BLE001
            extra5 = {"workload": "config5-long-context-split-kv", "error": str(e)[:300]}
        if rank == 0:
            try:
                extra2 = [summarise_small(x) for x in small_config_lines(args, ops, torch, dev, "2")]
            except Exception as e:  # noqa: BLE001
                extra2 = [{"workload": "config2", "error": str(e)[:300]}]
    if rank == 0:
        tokens = n_seq * args.steps
        value = tokens / (ms_max * 1e-3)
        peak, peak_kind = peaks()
        traffic = profiled_traffic("decode_kernel_config3_traffic")
        strong = args.scaling == "strong" or world == 1
        line = {
            "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_max / args.steps,
            "higher_is_better": True, "scaling": "strong" if strong else "weak",
            "vs_baseline": None, "dtype": "f16", "data": "synthetic",
            "hbm_tbs": bytes_timed / (ms_max * 1e-3) / 1e12,
            "config": {
                "workload": "config3-batched-ragged-decode", "global_batch": int(n_seq),
                "sequences_per_gpu": (f"{int(n_seq)} split across {world} GPUs, balanced by rows"
                                      if strong and world > 1 else int(n_seq) // world),
                "heads": HQ, "kv_heads": HKV, "head_dim": HD,
                "kv_len": "U[512,8192] seed 3 (+1..16 cycling append rows)",
                "accumulate": "f32", "step": "fused kv_append + decode attention, 1 launch",
                "l2": "inputs larger than L2 (~4.6 GB of K/V per step in total)",
                "parallelism": f"sequence-sharded x{world}, no communication"},
            "roofline": {"bound": "hbm", "achieved": kern_gbs, "peak": peak, "unit": "GB/s",
                         "frac": kern_gbs / peak, "traffic": traffic,
                         "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)",
                         "kernel": "decode_kernel", "launch_ms": kern_ms,
                         "algorithmic_bytes_per_launch": statistics.mean(rb)},
            "gpu_launches": args.steps,
            "clocks": clocks,
        }
        if e2e:
            line["e2e"] = {"value": tokens / (e2e_ms_max * 1e-3),
                           "unit": "tokens/s", "h2d_bytes_per_step": int(h2d),
                           "d2h_bytes_per_step": int(d2h),
                           "ms_per_step": e2e_ms_max / args.steps,
                           "path": "ops.kv_append_attention_batched (ctypes -> libnwd.so C ABI), "
                                   "pinned host buffers; inputs cross on a copy stream while the "
                                   "previous step computes, o crosses on a second copy stream, "
                                   "the host reads step x-1's o before issuing step x+1"}
        if extra5:
            line["config5"] = extra5
        if extra2:
            line["config2"] = extra2
        if world == 1 and not args.no_cpu_baseline:
            oracle = import_oracle()
            line["cpu_baseline"] = cpu_baseline(oracle, cpu_L, cpu_seeds, seconds=args.cpu_seconds)
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def summarise_small(ln):
    """The figures of a config-2 line kept in the headline line's sub-object."""
    return {"workload": ln["config"]["workload"], "kv_len": ln["config"]["kv_len"],
            "heads": ln["config"]["heads"], "ms_per_step": ln["ms_per_step"],
            "tokens_per_s": ln["value"], "achieved_gbs": ln["roofline"]["achieved"],
            "frac": ln["roofline"]["frac"], "steps": ln["steps"], "l2": ln["config"]["l2"]}


def run_small_configs(args, ops, torch, dev, rank, world):
    """Secondary lines: config 1 (engine trace) and config 2 (L sweep), Hq=40
    (engine/config.js), on rank 0 (a single sequence does not shard: replicas only)."""
    if rank != 0:
        return 0
    sampler = start_clocks(torch, dev, rank)
    t0 = time.monotonic()
    out = small_config_lines(args, ops, torch, dev, args.config)
    t1 = time.monotonic()
    if sampler:
        sampler.stop()
        clocks = sampler.summary(t0, t1)
        for ln in out:
            ln["clocks"] = clocks
    for ln in out:
        print(json.dumps(ln), flush=True)
    return 0


def small_config_lines(args, ops, torch, dev, which):
    """Lines of config 1 (which="1") or the config-2 sweep (which="2").

    These single-sequence steps take microseconds, so the steps are captured
    once in a CUDA graph (one fused launch per step, in order) and the graph is
    replayed: the timing is the GPU's, not Python's launch overhead.
    """
    engine = importlib.import_module(PKG + ".engine")
    peak, _ = peaks()
    nh = 40
    out = []

    flush = torch.empty(FLUSH_BYTES, dtype=torch.uint8, device=dev)

    def replay_ms(g, reps, stream):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(reps):
            g.replay()
        b.record(stream)
        b.synchronize()
        return a.elapsed_time(b)

    def timed_graph(layer, seqs, q, kn, o):
        """Capture one fused step per entry of `seqs`, each after an L2 flush (a write
        larger than L2), and the same flushes alone; return (ms per step, bytes per
        step, steps): the step's time is replay(flush + step) - replay(flush)."""
        stream = torch.cuda.Stream()
        nbytes = sum(4096 * (x + 1) + 2 * nh * HD * 2 + 4 * HKV * HD * 2 for x in seqs) / len(seqs)
        with torch.cuda.stream(stream):
            for x in seqs:  # warm (and first-call set-up) outside the capture
                layer.seq = x
                layer.step(q, kn, kn, out=o)
            stream.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                for i, x in enumerate(seqs):
                    flush.fill_(i & 0xFF)
                    layer.seq = x
                    layer.step(q, kn, kn, out=o)
            gf = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gf, stream=stream):
                for i in range(len(seqs)):
                    flush.fill_(i & 0xFF)
            reps = max(5, args.steps // len(seqs))
            for _ in range(max(1, args.warmup // len(seqs)) + 2):
                g.replay()
                gf.replay()
            stream.synchronize()
            # interleaved, so clock drift hits both alike
            t_both = t_flush = 0.0
            for _ in range(reps):
                t_both += replay_ms(g, 1, stream)
                t_flush += replay_ms(gf, 1, stream)
        ms = (t_both - t_flush) / (reps * len(seqs))
        del g, gf
        return ms, nbytes, reps * len(seqs)

    def timed_graph_rotating(layers, seqs, q, kn, o):
        """One fused step per (position, sequence), the sequences visited in turn;
        return (ms per step, bytes per step, steps)."""
        stream = torch.cuda.Stream()
        nbytes = sum(4096 * (x + 1) + 2 * nh * HD * 2 + 4 * HKV * HD * 2 for x in seqs) / len(seqs)
        n = len(seqs) * len(layers)
        with torch.cuda.stream(stream):
            for x in seqs:  # warm (and first-call set-up) outside the capture
                for layer in layers:
                    layer.seq = x
                    layer.step(q, kn, kn, out=o)
            stream.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                for x in seqs:
                    for layer in layers:
                        layer.seq = x
                        layer.step(q, kn, kn, out=o)
            reps = max(3, args.steps // n)
            for _ in range(max(1, args.warmup // n) + 2):
                g.replay()
            stream.synchronize()
            t = replay_ms(g, reps, stream)
        del g
        return t / (reps * n), nbytes, reps * n

    def line(workload, ms, nbytes, steps, extra):
        gbs = nbytes / (ms * 1e-3) / 1e9
        cfg = {"workload": workload, "heads": nh, "kv_heads": HKV, "head_dim": HD,
               "launches_per_step": 1, "timing": "CUDA graph replay of the step sequence",
               "l2": f"flushed before every step ({FLUSH_BYTES >> 20} MB write); step time = "
                     "replay(flush + step) - replay(flush)"}
        cfg.update(extra)
        return {"metric": METRIC, "value": 1e3 / ms, "unit": "tokens/s", "n_gpus": 1,
                "steps": steps, "warmup": args.warmup, "ms_per_step": ms,
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f16",
                "data": "synthetic", "hbm_tbs": gbs / 1e3, "config": cfg,
                "roofline": {"bound": "hbm", "achieved": gbs, "peak": peak, "unit": "GB/s",
                             "frac": gbs / peak}}

    if which == "1":
        layer = engine.DecodeAttention(nh, HKV, HD, 256)
        ops.fill_normal(layer.k_cache, 11)
        ops.fill_normal(layer.v_cache, 12)
        q = ops.fill_normal(torch.empty(nh, HD, dtype=torch.float16, device=dev), 13)
        kn = ops.fill_normal(torch.empty(HKV, HD, dtype=torch.float16, device=dev), 14)
        o = torch.empty(nh, HD, dtype=torch.float16, device=dev)
        ms, nbytes, steps = timed_graph(layer, list(range(151)), q, kn, o)  # 24 prompt + 127 decode
        out.append(line("config1-engine-trace", ms, nbytes, steps,
                        {"kv_len": "1..151 (24 prompt + 127 decode steps)"}))
    else:
        for L in ([args.kv_len] if args.kv_len else (1024, 4096, 16384, 32768)):
            # independent sequences whose caches together exceed L2 by far, visited in
            # turn: every step reads its K/V cold (and L2 holds no dirty lines to write back)
            copies = max(2, -(-ROTATE_BYTES // (L * 4096)))
            layers = []
            for c in range(copies):
                layer = engine.DecodeAttention(nh, HKV, HD, L + POS_CYCLE)
                ops.fill_normal(layer.k_cache, 21 + 2 * c)
                ops.fill_normal(layer.v_cache, 22 + 2 * c)
                layers.append(layer)
            q = ops.fill_normal(torch.empty(nh, HD, dtype=torch.float16, device=dev), 23)
            kn = ops.fill_normal(torch.empty(HKV, HD, dtype=torch.float16, device=dev), 24)
            o = torch.empty(nh, HD, dtype=torch.float16, device=dev)
            ms, nbytes, steps = timed_graph_rotating(layers, [L - 1 + j for j in range(POS_CYCLE)],
                                                     q, kn, o)
            out.append(line(f"config2-L{L}", ms, nbytes, steps,
                            {"kv_len": L, "l2": f"{copies} sequences visited in turn "
                             f"({copies * L * 4096 >> 20} MB of K/V > L2); no flush"}))
            del layers
    return out


def run_config4(args, ops, torch, dist, dev, rank, world):
    """Config 4: chunked causal prefill, 8 sequences x 2048 prompt tokens per GPU
    (Hq=32, Hkv=8, d=128, scale 1/sqrt(128)).  A step writes the chunk's K/V rows through
    the kv_append path (nwd_kv_append_rows) and runs the tcgen05 prefill attention.
    Sequences shard across GPUs with no communication (weak scaling)."""
    B, S = 8, 2048
    rows = B * S
    seed = 4000 + 100 * rank
    f16 = torch.float16
    k_pool = torch.empty(rows, HKV, HD, dtype=f16, device=dev)
    v_pool = torch.empty_like(k_pool)
    k_new = ops.fill_normal(torch.empty(B, S, HKV, HD, dtype=f16, device=dev), seed)
    v_new = ops.fill_normal(torch.empty(B, S, HKV, HD, dtype=f16, device=dev), seed + 1)
    q = ops.fill_normal(torch.empty(B, S, HQ, HD, dtype=f16, device=dev), seed + 2)
    o = torch.empty(B, S, HQ, HD, dtype=f16, device=dev)
    ro = torch.arange(B, dtype=torch.int64, device=dev) * S
    ws = ops.Scratch(dev)
    flops = 4.0 * B * HQ * HD * S * (S + 1) / 2  # causal: visible (query, key) pairs only

    def step(qq=None, kk=None, vv=None, oo=None):
        ops.kv_append_rows(k_new if kk is None else kk, v_new if vv is None else vv, k_pool,
                           v_pool, ro, 0, workspace=ws)
        ops.attention_prefill(q if qq is None else qq, k_pool, v_pool, ro,
                              o if oo is None else oo, 0, HQ, HKV, HD, workspace=ws)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    sampler = start_clocks(torch, dev, rank)
    for _ in range(args.warmup):
        step()
    barrier()
    t0 = time.monotonic()
    a, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(args.steps):
        step()
    e.record()
    e.synchronize()
    barrier()
    t1 = time.monotonic()
    if sampler:
        sampler.stop()
    ms = a.elapsed_time(e)
    # the prefill kernel alone, per-launch events
    R = min(args.steps, 20)
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(R)]
    for i in range(R):
        ops.kv_append_rows(k_new, v_new, k_pool, v_pool, ro, 0, workspace=ws)
        evs[i][0].record()
        ops.attention_prefill(q, k_pool, v_pool, ro, o, 0, HQ, HKV, HD, workspace=ws)
        evs[i][1].record()
    torch.cuda.synchronize()
    kern_ms = statistics.mean(x.elapsed_time(y) for x, y in evs)
    # e2e: the chunk's q, k, v from pinned host memory, o back, every step
    q_h, k_h, v_h = q.cpu().pin_memory(), k_new.cpu().pin_memory(), v_new.cpu().pin_memory()
    o_h = torch.empty_like(o, device="cpu").pin_memory()
    qd, kd, vd, od = torch.empty_like(q), torch.empty_like(k_new), torch.empty_like(v_new), \
        torch.empty_like(o)
    stream = torch.cuda.current_stream()

    def e2e_step():
        qd.copy_(q_h, non_blocking=True)
        kd.copy_(k_h, non_blocking=True)
        vd.copy_(v_h, non_blocking=True)
        step(qd, kd, vd, od)
        o_h.copy_(od, non_blocking=True)
        stream.synchronize()

    for _ in range(args.warmup):
        e2e_step()
    barrier()
    a2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a2.record()
    for _ in range(args.steps):
        e2e_step()
    e2.record()
    e2.synchronize()
    barrier()
    ms_max, e2e_max = max_over_ranks([ms, a2.elapsed_time(e2)], dist, dev)
    err = ws.check()
    if rank == 0:
        peak, kind = tensor_peak()
        tflops = flops / (kern_ms * 1e-3) / 1e12
        tokens = B * S * world * args.steps
        line = {
            "metric": METRIC, "value": tokens / (ms_max * 1e-3), "unit": "tokens/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": ms_max / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f16", "data": "synthetic",
            "tflops": flops * world / (ms_max * 1e-3 / args.steps) / 1e12,
            "config": {"workload": "config4-chunked-causal-prefill", "sequences_per_gpu": B,
                       "chunk": S, "heads": HQ, "kv_heads": HKV, "head_dim": HD,
                       "accumulate": "f32 (TMEM)",
                       "step": "kv_append of the chunk's K/V rows + tcgen05 causal prefill",
                       "flops_per_step_per_gpu": flops},
            "roofline": {"bound": "tensor", "achieved": tflops, "peak": peak, "unit": "TFLOP/s",
                         "frac": tflops / peak, "kernel": "prefill_kernel",
                         "launch_ms": kern_ms, "peak_source": f"{kind} (bf16_tflops, burst)"},
            "e2e": {"value": tokens / (e2e_max * 1e-3), "unit": "tokens/s",
                    "h2d_bytes_per_step": (q.numel() + 2 * k_new.numel()) * 2 * world,
                    "d2h_bytes_per_step": o.numel() * 2 * world},
            "gpu_launches": 2 * args.steps,
            "device_error": err,
            "clocks": sampler.summary(t0, t1) if sampler else None,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0 if err == 0 else 3


HIDDEN6, HQ6 = 3136, 40          # engine/config.js: hidden, heads
N_ATTN_LAYERS = 4                 # engine/config.js ATTN_LAYERS
L6 = 150                          # rows already cached (config 1's trace end)
WEIGHT_SETS = 3                   # rotating copies: 3 x 99 MB of q4 weights > L2
FLUSH_BYTES = 192 << 20           # config 1: a write this large evicts L2 (126 MB) before each step
ROTATE_BYTES = 320 << 20          # config 2: K/V of the sequences visited in turn


def _q4_random(ops, torch, n, n_blocks, gen, dev):
    """Synthetic q4 weights in the MatMulNBits layout (uniform nibbles, scales in
    [2^-9, 2^-9 + 2^-7)), generated on the device."""
    b = torch.randint(-2**31, 2**31 - 1, (n, n_blocks, 4), dtype=torch.int32, device=dev,
                      generator=gen)
    s = torch.rand(n, n_blocks, device=dev, generator=gen) * 0.0078125 + 0.001953125
    z = torch.randint(-2**31, 2**31 - 1, ((n * n_blocks + 7) // 8,), dtype=torch.int32,
                      device=dev, generator=gen)
    return ops.Q4Weights(b, s, z)


def run_config6(args, ops, torch, dist, dev, rank, world):
    """Scope row (f): one decode token through the model's 4 attention layers with the
    projections either side of the path, at the engine shape (hidden 3136, Hq 40,
    Hkv 8, d 128, 150 cached rows): per layer the q/k/v q4 GEMVs with k/v appended
    to the cache (one launch), attention, and the o_proj q4 GEMV with the residual
    add (runtime.js:385-394).  Three rotating copies of the 4 layers' weights (296 MB)
    keep every step's weights out of L2.  Each copy's 4 layers are captured once in
    a CUDA graph (12 launches) and replayed.  Replicas only: a single sequence does
    not shard."""
    eng = importlib.import_module(PKG + ".engine")
    gen = torch.Generator(device=dev)
    gen.manual_seed(6000 + rank)
    nb_h, nb_o = HIDDEN6 // 32, HQ6 * HD // 32
    sets = []
    for _ in range(WEIGHT_SETS):
        layers = []
        for _ in range(N_ATTN_LAYERS):
            layer = eng.AttentionLayer(_q4_random(ops, torch, HQ6 * HD, nb_h, gen, dev),
                                       _q4_random(ops, torch, HKV * HD, nb_h, gen, dev),
                                       _q4_random(ops, torch, HKV * HD, nb_h, gen, dev),
                                       _q4_random(ops, torch, HIDDEN6, nb_o, gen, dev),
                                       HQ6, HKV, HD, 256, dev)
            ops.fill_normal(layer.attn.k_cache, 61 + rank)
            ops.fill_normal(layer.attn.v_cache, 62 + rank)
            layers.append(layer)
        sets.append(layers)
    h_norm = torch.randn(N_ATTN_LAYERS, HIDDEN6, device=dev, generator=gen)
    h = torch.randn(HIDDEN6, device=dev, generator=gen)
    weight_bytes = sum(w.b.numel() * 4 + w.scales.numel() * 4 + w.zp.numel() * 4
                       for L in sets[0] for w in (L.wq, L.wk, L.wv, L.wo))
    # algorithmic bytes per token: weights once, K/V rows attended, the new rows,
    # q / o, the residual read + write and the activations
    kv_bytes = N_ATTN_LAYERS * ((L6 + 1) * HKV * HD * 2 * 2 + 2 * HKV * HD * 2)
    act_bytes = N_ATTN_LAYERS * (HIDDEN6 * 4 + 2 * HQ6 * HD * 2 * 2 + 2 * HIDDEN6 * 4)
    step_bytes6 = weight_bytes + kv_bytes + act_bytes

    stream = torch.cuda.Stream(device=dev)
    # optional weight prefetch: during each attention launch a side stream starts the
    # layer's o_proj weights and the next layer's q/k/v weights into L2.  Off by
    # default: measured slower (71.2 against 66.4 us per token), its HBM traffic
    # lands on the latency-bound attention launch
    side = torch.cuda.Stream(device=dev) if args.prefetch else None
    graphs = []
    with torch.cuda.stream(stream):
        for layers in sets:  # eager once (sets the kernels' attributes), then capture
            for L in layers:
                L.attn.seq = L6
            eng.step_layers(layers, h_norm, h, side=side)
        torch.cuda.synchronize()
        for layers in sets:
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                for L in layers:
                    L.attn.seq = L6
                eng.step_layers(layers, h_norm, h, side=side)
            graphs.append(g)
    torch.cuda.synchronize()

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    sampler = start_clocks(torch, dev, rank)
    s = 0
    for _ in range(args.warmup):
        graphs[s % WEIGHT_SETS].replay()
        s += 1
    barrier()
    t0 = time.monotonic()
    a, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(args.steps):
        graphs[s % WEIGHT_SETS].replay()
        s += 1
    e.record()
    e.synchronize()
    barrier()
    t1 = time.monotonic()
    if sampler:
        sampler.stop()
    ms = a.elapsed_time(e)
    # the q/k/v launch alone (the largest kernel): one launch per layer of every weight
    # copy (12, cold weights) captured in a graph, so the time is the GPU's alone
    qkv_graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        with torch.cuda.graph(qkv_graph, stream=stream):
            for layers in sets:
                for L in layers:
                    ops.q4_qkv_append(h_norm[0], L.wq, L.wk, L.wv, L.q, L.attn.k_cache,
                                      L.attn.v_cache, L6, stream=stream)
    torch.cuda.synchronize()
    n_qkv = WEIGHT_SETS * N_ATTN_LAYERS
    qkv_runs = []
    for _ in range(5):
        x, y = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        x.record()
        qkv_graph.replay()
        y.record()
        y.synchronize()
        qkv_runs.append(x.elapsed_time(y) / n_qkv)
    qkv_ms = statistics.median(qkv_runs)
    del qkv_graph
    L0 = sets[0][0]
    qkv_bytes = sum(w.b.numel() * 4 + w.scales.numel() * 4 + w.zp.numel() * 4
                    for w in (L0.wq, L0.wk, L0.wv)) + HIDDEN6 * 4 + (HQ6 + 2 * HKV) * HD * 2
    # e2e: the layers' inputs from pinned host memory and the residual stream back
    e2e = None
    if not args.no_e2e:
        hn_h = h_norm.cpu().pin_memory()
        h_h = torch.empty(HIDDEN6, dtype=torch.float32).pin_memory()
        cur = torch.cuda.current_stream()
        for _ in range(args.warmup):
            h_norm.copy_(hn_h, non_blocking=True)
            graphs[s % WEIGHT_SETS].replay()
            h_h.copy_(h, non_blocking=True)
            cur.synchronize()
            s += 1
        barrier()
        a2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a2.record()
        for _ in range(args.steps):
            h_norm.copy_(hn_h, non_blocking=True)
            graphs[s % WEIGHT_SETS].replay()
            h_h.copy_(h, non_blocking=True)
            cur.synchronize()
            s += 1
        e2.record()
        e2.synchronize()
        barrier()
        e2e = a2.elapsed_time(e2)
    ms_max, qkv_max, e2e_max = max_over_ranks([ms, qkv_ms, e2e or 0.0], dist, dev)
    err = max(L.attn.workspace.check() for layers in sets for L in layers)
    cpu = None
    if rank == 0 and not args.no_cpu_baseline:
        cpu = cpu_baseline_config6(args)
    for g in graphs:
        del g
    graphs.clear()
    if rank == 0:
        peak, kind = peaks()
        gbs = qkv_bytes / (qkv_ms * 1e-3) / 1e9
        line = {
            "metric": "attention-layer decode tokens/s (q/k/v q4 projections + append + "
                      "attention + o_proj + residual, 4 layers)",
            "value": world * args.steps / (ms_max * 1e-3), "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_max / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (random q4 weights, N(0,1) activations and caches)",
            "hbm_tbs": step_bytes6 / (ms_max / args.steps * 1e-3) / 1e12,
            "config": {"workload": "row-f-attention-layers", "layers": N_ATTN_LAYERS,
                       "hidden": HIDDEN6, "heads": HQ6, "kv_heads": HKV, "head_dim": HD,
                       "cached_rows": L6, "weight_sets": WEIGHT_SETS,
                       "weights_mb_per_step": weight_bytes / 1e6,
                       "bytes_per_step": step_bytes6,
                       "l2": "three rotating weight copies (296 MB) > L2",
                       "weight_prefetch": ("off" if side is None else
                                           "each layer's o_proj and the next layer's q/k/v "
                                           "weights into L2 on a side stream during attention"),
                       "launch": "CUDA graph per weight copy (12 launches, + 4 "
                                 "prefetch launches on the side stream)"},
            "roofline": {"bound": "hbm", "achieved": gbs, "peak": peak, "unit": "GB/s",
                         "frac": gbs / peak, "kernel": "q4_gemv_kernel (q/k/v + append)",
                         "launch_ms": qkv_max, "bytes_per_launch": qkv_bytes,
                         "traffic": profiled_traffic("q4_gemv_kernel_config6_traffic"),
                         "peak_source": f"{kind} (hbm_gbs)"},
            "e2e": ({"value": world * args.steps / (e2e_max * 1e-3), "unit": "tokens/s",
                     "h2d_bytes_per_step": N_ATTN_LAYERS * HIDDEN6 * 4,
                     "d2h_bytes_per_step": HIDDEN6 * 4} if e2e is not None else None),
            "cpu_baseline": cpu,
            "gpu_launches": (12 if side is None else 16) * args.steps,
            "device_error": err,
            "clocks": sampler.summary(t0, t1) if sampler else None,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0 if err == 0 else 3


def cpu_baseline_config6(args):
    """The oracle (the reference's algorithm) for one attention layer with its
    projections on the host cores, scaled to the 4 layers of a token."""
    oracle = import_oracle()
    nb_h, nb_o = HIDDEN6 // 32, HQ6 * HD // 32
    wq = oracle.q4_weights(HQ6 * HD, nb_h, 1)
    wk = oracle.q4_weights(HKV * HD, nb_h, 2)
    wv = oracle.q4_weights(HKV * HD, nb_h, 3)
    wo = oracle.q4_weights(HIDDEN6, nb_o, 4)
    kc = oracle.normal_f16(256 * HKV * HD, 5).reshape(256, HKV, HD)
    vc = oracle.normal_f16(256 * HKV * HD, 6).reshape(256, HKV, HD)
    hn = oracle.f16_bits_to_f32(oracle.normal_f16(HIDDEN6, 7))
    h = oracle.f16_bits_to_f32(oracle.normal_f16(HIDDEN6, 8))
    reps, t0 = 0, time.perf_counter()
    while reps < 3 or (time.perf_counter() - t0 < min(args.cpu_seconds, 5.0) and reps < 200):
        q = oracle.f32_to_f16_bits(oracle.q4_gemv(hn, *wq))
        oracle.kv_append(oracle.f32_to_f16_bits(oracle.q4_gemv(hn, *wk)), kc, L6, HKV, HD)
        oracle.kv_append(oracle.f32_to_f16_bits(oracle.q4_gemv(hn, *wv)), vc, L6, HKV, HD)
        o = oracle.attention(q, kc, vc, HQ6, HKV, HD, L6 + 1)
        h = oracle.q4_gemv(o, *wo, epilogue=2, y=h)
        reps += 1
    dt = (time.perf_counter() - t0) / reps
    return {"value": 1.0 / (N_ATTN_LAYERS * dt), "unit": "tokens/s",
            "cores": oracle.num_threads(), "kind": "port",
            "sample": f"{reps} single-layer steps (q/k/v, append, attention over {L6 + 1} rows, "
                      f"o_proj + residual) on the oracle, scaled to {N_ATTN_LAYERS} layers"}


def run_config5(args, ops, torch, dist, dev, rank, world):
    """--config 5: the long-context sharded step as its own line."""
    line = measure_config5(args, ops, torch, dist, dev, rank, world, sub=False)
    err = line.get("device_error", 0) if line else 0
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0 if err == 0 else 3


def measure_config5(args, ops, torch, dist, dev, rank, world, sub=False):
    """Config 5: 4 sequences x 1 048 576 rows (Hq=32, Hkv=8), each sequence's
    rows sharded contiguously over the ranks (strong scaling); a step is the shard
    partial on every GPU, the exchange of the partials (written into every rank's
    buffer over peer memory, or one NCCL all-gather) and the LSE merge, run by
    the library (nwd_mgpu_decode_step) at N > 1, and the partial +
    merge at N = 1.  The K/V data is the same stream whatever the rank count (fill
    offsets follow the global row index), so every N computes the same O.  Returns
    the line (rank 0) or None; with sub=True the figures the config-3 line keeps."""
    mgpu = importlib.import_module(PKG + ".mgpu")
    B, L = 4, 1 << 20
    if args.kv_len and not sub:
        L = args.kv_len
    sd = mgpu.ShardedDecode([L] * B, HQ, HKV, HD, device=dev)
    row_elems = HKV * HD
    for b in range(B):
        lo, hi = sd.global_rows(b)
        off = int(sd.row_offset[b])
        n = hi - lo
        ops.fill_normal(sd.k_pool[off:off + n], 5000, (b * L + lo) * row_elems)
        ops.fill_normal(sd.v_pool[off:off + n], 5001, (b * L + lo) * row_elems)
    q = ops.fill_normal(torch.empty(B, HQ, HD, dtype=torch.float16, device=dev), 5002)
    o = torch.empty(B, HQ, HD, dtype=torch.float16, device=dev)
    torch.cuda.synchronize()
    steps = args.steps
    warmup = args.warmup

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    sampler = None if sub else start_clocks(torch, dev, rank)
    for _ in range(warmup):
        sd.step(q, o)
    sd.sync()
    barrier()
    t0 = time.monotonic()
    a, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    hold_stream(torch, steps)
    a.record()
    for _ in range(steps):
        sd.step(q, o)
    e.record()
    sd.sync()  # bounded by the communicator's deadline at N > 1
    e.synchronize()
    barrier()
    t1 = time.monotonic()
    if sampler:
        sampler.stop()
    ms = a.elapsed_time(e)
    # where a step's time goes: the shard partial, and the exchange + merge.
    # One process: events around each.  Several ranks: the exchange's exposed
    # time is the back-to-back step minus the partial launch alone (timing
    # single synchronised steps would count the ranks' launch skew as exchange)
    R = min(steps, 20)
    part_ms, xchg_ms = [0.0], [0.0]
    if sd.comm is None:
        part_ms, xchg_ms = [], []
        for _ in range(R):
            e0, e1, e2 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
            e0.record()
            sd.partial_fn(q)
            e1.record()
            ops.merge_packed(sd.packed.unsqueeze(0), o)
            e2.record()
            e2.synchronize()
            part_ms.append(e0.elapsed_time(e1))
            xchg_ms.append(e1.elapsed_time(e2))
    # roofline of the shard kernel alone (per-launch events, same stream)
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(R)]
    for i in range(R):
        evs[i][0].record()
        sd.partial_fn(q)
        evs[i][1].record()
    torch.cuda.synchronize()
    kern_ms = statistics.mean(x.elapsed_time(y) for x, y in evs)
    local_rows = sum(hi - lo for lo, hi in (sd.global_rows(b) for b in range(B)))
    kern_bytes = 4096.0 * local_rows + B * HQ * HD * 2 + B * HQ * (HD + 2) * 4
    traffic5 = profiled_traffic("decode_kernel_config5_traffic")
    # e2e: q from pinned host memory, O back to host, every step
    q_h = q.cpu().pin_memory()
    o_h = torch.empty(B, HQ, HD, dtype=torch.float16, pin_memory=True)
    stream = torch.cuda.current_stream()
    for _ in range(warmup):
        q.copy_(q_h, non_blocking=True)
        sd.step(q, o)
        o_h.copy_(o, non_blocking=True)
        sd.sync()
        stream.synchronize()
    barrier()
    a2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a2.record()
    for _ in range(steps):
        q.copy_(q_h, non_blocking=True)
        sd.step(q, o)
        o_h.copy_(o, non_blocking=True)
        sd.sync()
        stream.synchronize()
    e2.record()
    e2.synchronize()
    barrier()
    e2e_ms = a2.elapsed_time(e2)
    ms_max, e2e_max, kern_max, part_max, xchg_max = max_over_ranks(
        [ms, e2e_ms, kern_ms, statistics.mean(part_ms), statistics.mean(xchg_ms)], dist, dev)
    if sd.comm is not None:
        part_max = kern_max
        xchg_max = max(0.0, ms_max / steps - kern_max)
    err = sd.workspace.check()
    exchange = sd.comm.exchange_mode() if sd.comm is not None else "none"
    sd.close()
    del sd
    torch.cuda.empty_cache()
    if rank != 0:
        return None
    peak, kind = peaks()
    total_bytes = 4096.0 * B * L + B * HQ * HD * 4
    achieved = kern_bytes / (kern_ms * 1e-3) / 1e9
    roof = {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
            "frac": achieved / peak, "kernel": "decode_kernel (partial mode), per rank",
            "launch_ms": kern_ms, "peak_source": kind,
            # committed ncu figure for the whole 1-GPU launch (4 x 2^20 rows),
            # scaled to this rank's rows (traffic is proportional to rows)
            "traffic": (None if traffic5 is None else
                        traffic5 * local_rows / (4.0 * (1 << 20)))}
    split = {"partial_ms": part_max, "exchange_ms": xchg_max,
             "exchange_share": xchg_max / (part_max + xchg_max), "exchange": exchange,
             "how": ("the partial: CUDA events around each of "
                     f"{R} back-to-back shard-partial launches, mean, max over ranks; the "
                     "exchange + merge: the timed step (max over ranks) minus that, i.e. "
                     "the part of the step the exchange does not overlap"
                     if world > 1 else
                     f"CUDA events around the partial and the merge, mean of {R}")}
    value = B * steps / (ms_max * 1e-3)
    if sub:
        return {"workload": "config5-long-context-split-kv", "sequences": B, "kv_len": L,
                "scaling": "strong", "n_gpus": world, "value": value, "unit": "tokens/s",
                "ms_per_step": ms_max / steps, "hbm_tbs": total_bytes / (ms_max * 1e-3 / steps)
                / 1e12, "roofline": roof, "step_split": split, "device_error": err,
                "e2e": {"value": B * steps / (e2e_max * 1e-3), "unit": "tokens/s",
                        "h2d_bytes_per_step": B * HQ * HD * 2,
                        "d2h_bytes_per_step": B * HQ * HD * 2}}
    return {
        "metric": METRIC, "value": value, "unit": "tokens/s",
        "n_gpus": world, "steps": steps, "warmup": warmup,
        "ms_per_step": ms_max / steps, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f16", "data": "synthetic",
        "hbm_tbs": total_bytes / (ms_max * 1e-3 / steps) / 1e12,
        "config": {"workload": "config5-long-context-split-kv", "sequences": B,
                   "kv_len": L, "heads": HQ, "kv_heads": HKV, "head_dim": HD,
                   "parallelism": f"rows sharded x{world}, partials exchanged "
                                  f"({exchange}) by nwd_mgpu_decode_step",
                   "step": "shard partial + exchange + LSE merge"},
        "roofline": roof, "step_split": split,
        "e2e": {"value": B * steps / (e2e_max * 1e-3), "unit": "tokens/s",
                "h2d_bytes_per_step": B * HQ * HD * 2, "d2h_bytes_per_step": B * HQ * HD * 2},
        "gpu_launches": (3 if world > 1 else 2) * steps,
        "device_error": err,
        "clocks": sampler.summary(t0, t1) if sampler else None,
    }


if __name__ == "__main__":
    sys.exit(main())
