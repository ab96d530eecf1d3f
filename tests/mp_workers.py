"""Worker functions for the multi-process (gloo, CPU) tests.

Module-level so torch.multiprocessing can spawn them; each returns through a
file because spawned processes cannot return values.
"""
from __future__ import annotations

import importlib
import json
import os
import sys

import numpy as np


def _init(rank, world, port):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    return dist


def sharded_decode_worker(rank, world, port, repo, outdir):
    sys.path[:0] = [repo, os.path.join(repo, "oracle"), os.path.join(repo, "tests")]
    import torch
    import oracle as O
    dist = _init(rank, world, port)
    mgpu = importlib.import_module("nemotron-webgpu-decode_b200.mgpu")
    B, nh, nkv, hd = 3, 8, 2, 128
    lengths = [1000, 37, 513]
    total = sum(lengths)
    offs = np.concatenate([[0], np.cumsum(lengths)[:-1]]).astype(np.int64)
    q = O.normal_f16(B * nh * hd, 1)
    k = O.normal_f16(total * nkv * hd, 2).reshape(total, nkv, hd)
    v = O.normal_f16(total * nkv * hd, 3).reshape(total, nkv, hd)

    def partial_fn(qt):
        # the oracle computes this rank's shard partial (the GPU kernel's job)
        lo_hi = [mgpu.shard_bounds(L, world, rank) for L in lengths]
        so = np.array([offs[b] + lo for b, (lo, hi) in enumerate(lo_hi)], np.int64)
        sl = np.array([hi - lo for lo, hi in lo_hi], np.int32)
        po, pml = O.attention_partial(q, k, v, so, sl, nh, nkv, hd)
        return torch.from_numpy(po), torch.from_numpy(pml)

    def merge_fn(go, gml, out):
        m = O.merge(go.numpy(), gml.numpy())
        out.copy_(torch.from_numpy(m.reshape(out.shape)).to(out.dtype))
        return out

    sd = mgpu.ShardedDecode(lengths, nh, nkv, hd, partial_fn=partial_fn, merge_fn=merge_fn)
    out = sd.step(None, out=torch.empty(B, nh, hd, dtype=torch.float32))
    ref = O.attention_batched(q, k, v, offs, np.array(lengths, np.int32), nh, nkv, hd, f64=True)
    err = float(np.abs(out.numpy() - ref).max())
    rows = [list(sd.global_rows(b)) for b in range(B)]
    with open(os.path.join(outdir, f"rank{rank}.json"), "w") as f:
        json.dump({"err": err, "rows": rows, "out0": float(out[0, 0, 0])}, f)
    dist.barrier()
    dist.destroy_process_group()


def max_over_ranks_worker(rank, world, port, repo, outdir):
    sys.path[:0] = [repo]
    dist = _init(rank, world, port)
    import bench
    vals = bench.max_over_ranks([1.0 + rank, 10.0 - rank], dist)
    L = bench.rank_lengths(rank, world, "strong")
    Lw = bench.rank_lengths(rank, world, "weak")
    with open(os.path.join(outdir, f"rank{rank}.json"), "w") as f:
        json.dump({"vals": vals, "strong": [int(x) for x in L], "weak_n": len(Lw),
                   "seeds": bench.seeds_for(rank)}, f)
    dist.barrier()
    dist.destroy_process_group()


def missing_rank_worker(rank, world, port, repo, outdir):
    """Failure detection on the host: rank 1 leaves between steps without posting its
    shard partials (injected on the host, no GPU involved); rank 0's sharded step must
    end with an error once the process group's deadline passes, not hang."""
    sys.path[:0] = [repo]
    import datetime
    import time
    import torch
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    deadline = 3.0
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=deadline))
    mgpu = importlib.import_module("nemotron-webgpu-decode_b200.mgpu")
    B, nh, nkv, hd = 2, 4, 2, 128

    def partial_fn(q):
        return torch.zeros(B, nh, hd), torch.full((B, nh, 2), 1.0)

    def merge_fn(go, gml, out):
        return out

    sd = mgpu.ShardedDecode([300, 77], nh, nkv, hd, partial_fn=partial_fn, merge_fn=merge_fn)
    out = torch.empty(B, nh, hd, dtype=torch.float32)
    sd.step(None, out=out)  # one good step with every rank present
    if rank == world - 1:
        # the failing rank: stays alive but never posts its next partials
        with open(os.path.join(outdir, f"rank{rank}.json"), "w") as f:
            json.dump({"left": True}, f)
        time.sleep(3 * deadline)
        os._exit(0)
    t0 = time.monotonic()
    try:
        sd.step(None, out=out)
        status = "completed"
    except Exception as e:  # the collective's deadline
        status = f"{type(e).__name__}: {str(e)[:160]}"
    elapsed = time.monotonic() - t0
    with open(os.path.join(outdir, f"rank{rank}.json"), "w") as f:
        json.dump({"status": status, "elapsed": elapsed, "deadline": deadline}, f)
    os._exit(0)  # the group is broken: no collective teardown
