"""Decode attention over long contexts (e.g. 4 sequences x 1 048 576 cached rows) sharded across GPUs.

Each sequence's KV rows are split into contiguous shards, shard r on rank r
(one process per GPU).  A decode step is

1. on every rank, the shard partial (m, l, o) of every (sequence, query head)
   over the rank's rows (``nwd_attn_decode_partial``);
2. one all-gather of the partials, packed in one buffer (B*Hq*(128 + 2) floats
   per rank, 66.5 KB for 4 sequences x 32 heads) over NVLink;
3. the log-sum-exp merge in rank order (= row order, deterministic), which
   every rank computes, so every rank holds O (``nwd_attn_merge_packed``).

On GPUs the three run inside the library, ``nwd_mgpu_decode_step`` on an NCCL
communicator the library owns (``Communicator``), with host-side deadlines
that abort the communicator when a peer goes missing; this module only
allocates the buffers and hands the communicator id from rank 0 to the others
through ``torch.distributed`` (any backend).  The exchange is small next to
the KV stream (17 GB per step for 4 x 1M rows), so the step scales with the
shard size.  The reference has no multi-device code; this extends its
single-sequence attention (kernels/sparse_attn.wgsl).

The compute steps are injectable (``partial_fn``, ``merge_fn``) so the host
logic (shard bounds, gather layout and merge order) is tested under gloo on
CPU against the oracle; that path gathers with ``torch.distributed``.
"""
from __future__ import annotations

import ctypes
from typing import Callable, Sequence

import torch
import torch.distributed as dist

from . import _lib


def shard_bounds(length: int, world: int, rank: int) -> tuple[int, int]:
    """Rows [lo, hi) of a sequence of `length` rows held by `rank` (contiguous shards)."""
    return length * rank // world, length * (rank + 1) // world


def _dist_on() -> bool:
    return dist.is_available() and dist.is_initialized()


def gather_partials(part_o: torch.Tensor, part_ml: torch.Tensor, group=None):
    """All-gather [B, Hq, d] / [B, Hq, 2] partials into [world, ...] tensors, rank order."""
    if not _dist_on():  # a single process holds every shard
        return part_o.unsqueeze(0), part_ml.unsqueeze(0)
    world = dist.get_world_size(group)
    go = part_o.new_empty((world,) + tuple(part_o.shape))
    gml = part_ml.new_empty((world,) + tuple(part_ml.shape))
    dist.all_gather(list(go.unbind(0)), part_o.contiguous(), group=group)
    dist.all_gather(list(gml.unbind(0)), part_ml.contiguous(), group=group)
    return go, gml


def gather_packed(packed: torch.Tensor, group=None) -> torch.Tensor:
    """All-gather a rank's packed partials [n] into [world, n], rank order (one collective)."""
    if not _dist_on():
        return packed.unsqueeze(0)
    world = dist.get_world_size(group)
    g = packed.new_empty((world, packed.numel()))
    dist.all_gather(list(g.unbind(0)), packed, group=group)
    return g


def unpack_partials(g: torch.Tensor, batch: int, n_heads: int, head_dim: int):
    """Views (part_o [world, B, Hq, hd], part_ml [world, B, Hq, 2]) of gathered packed partials."""
    n = batch * n_heads * head_dim
    return (g[:, :n].view(-1, batch, n_heads, head_dim),
            g[:, n:].view(-1, batch, n_heads, 2))


def share_unique_id(rank: int, group=None) -> bytes:
    """Rank 0's new communicator id (nwd_mgpu_unique_id), delivered to every rank."""
    lib = _lib.load()
    buf = (ctypes.c_uint8 * 128)()
    if rank == 0:
        _lib.check(lib.nwd_mgpu_unique_id(buf))
    obj = [bytes(buf)]
    if _dist_on() and dist.get_world_size(group) > 1:
        dist.broadcast_object_list(obj, src=0, group=group)
    return obj[0]


class Communicator:
    """An NCCL communicator owned by the library (``nwd_mgpu_*``).

    init_deadline_ms bounds the set-up (every rank must join within it);
    step_deadline_ms bounds each later wait.  After a deadline or an NCCL
    error the library aborts the communicator and every later step raises.
    """

    def __init__(self, unique_id: bytes, world: int, rank: int, device: int,
                 init_deadline_ms: int = 120_000, step_deadline_ms: int = 60_000):
        self.lib = _lib.load()
        self.world, self.rank, self.device = world, rank, device
        uid = (ctypes.c_uint8 * 128).from_buffer_copy(unique_id)
        self.handle = ctypes.c_void_p()
        _lib.check(self.lib.nwd_mgpu_init(uid, world, rank, device, init_deadline_ms,
                                          step_deadline_ms, ctypes.byref(self.handle)))

    def workspace_bytes(self, batch: int, n_heads: int, n_kv_heads: int, head_dim: int) -> int:
        n = ctypes.c_size_t(0)
        _lib.check(self.lib.nwd_mgpu_workspace_size(self.world, batch, n_heads, n_kv_heads,
                                                    head_dim, ctypes.byref(n)))
        return int(n.value)

    def decode_step(self, q, k_pool, v_pool, pool_rows, row_offset, seq_len, o, batch, n_heads,
                    n_kv_heads, head_dim, ws_ptr, ws_bytes, stream, scale: float = 0.0):
        _lib.check(self.lib.nwd_mgpu_decode_step(
            self.handle, q, k_pool, v_pool, pool_rows, row_offset, seq_len, o, batch, n_heads,
            n_kv_heads, head_dim, float(scale), ws_ptr, ws_bytes, stream))

    def sync(self) -> None:
        _lib.check(self.lib.nwd_mgpu_sync(self.handle))

    def set_timing(self, on: bool) -> None:
        _lib.check(self.lib.nwd_mgpu_set_timing(self.handle, int(bool(on))))

    def step_times(self) -> tuple[float, float]:
        """(partial ms, all-gather + merge ms) of the last timed step (after sync)."""
        a, b = ctypes.c_float(), ctypes.c_float()
        _lib.check(self.lib.nwd_mgpu_step_times(self.handle, ctypes.byref(a), ctypes.byref(b)))
        return float(a.value), float(b.value)

    def exchange_mode(self) -> str:
        """"peer" (partials written into every rank's exchange buffer), "nccl"
        (all-gather + merge) or "undecided" (no step yet)."""
        v = ctypes.c_int(0)
        _lib.check(self.lib.nwd_mgpu_exchange_mode(self.handle, ctypes.byref(v)))
        return {1: "peer", -1: "nccl"}.get(int(v.value), "undecided")

    def close(self) -> None:
        if self.handle:
            h, self.handle = self.handle, ctypes.c_void_p()
            _lib.check(self.lib.nwd_mgpu_destroy(h))

    def abort(self) -> None:
        if self.handle:
            h, self.handle = self.handle, ctypes.c_void_p()
            _lib.check(self.lib.nwd_mgpu_abort(h))


class ShardedDecode:
    """One rank's shard of a batch of long sequences, and the sharded step.

    lengths: rows of every sequence (global).  The rank allocates its shard of
    each sequence contiguously in a local pool (plus `extra_rows` of room per
    sequence on the last rank, which receives appended rows).  On a GPU with
    more than one rank the step runs in the library (``Communicator``).
    """

    def __init__(self, lengths: Sequence[int], n_heads: int, n_kv_heads: int,
                 head_dim: int = 128, group=None, device=None, extra_rows: int = 0,
                 partial_fn: Callable | None = None, merge_fn: Callable | None = None,
                 step_deadline_ms: int = 60_000):
        self.group = group
        self.rank = dist.get_rank(group) if _dist_on() else 0
        self.world = dist.get_world_size(group) if _dist_on() else 1
        self.lengths = [int(x) for x in lengths]
        self.B = len(self.lengths)
        self.n_heads, self.n_kv_heads, self.head_dim = n_heads, n_kv_heads, head_dim
        self.device = torch.device(device) if device is not None else torch.device("cpu")
        last = self.rank == self.world - 1
        self.bounds = [shard_bounds(L, self.world, self.rank) for L in self.lengths]
        local = [hi - lo for lo, hi in self.bounds]
        caps = [n + (extra_rows if last else 0) for n in local]
        offs = [0]
        for c in caps[:-1]:
            offs.append(offs[-1] + c)
        self.capacity = caps
        self.pool_rows = max(1, sum(caps))
        self.row_offset = torch.tensor(offs, dtype=torch.int64, device=self.device)
        self.seq_len = torch.tensor(local, dtype=torch.int32, device=self.device)
        shape = (self.pool_rows, n_kv_heads, head_dim)
        self.k_pool = torch.zeros(shape, dtype=torch.float16, device=self.device)
        self.v_pool = torch.zeros_like(self.k_pool)
        # o and (m, l) partials in one buffer (the gloo / single-rank paths)
        n = self.B * n_heads * head_dim
        self.packed = torch.empty(n + self.B * n_heads * 2, dtype=torch.float32,
                                  device=self.device)
        self.part_o = self.packed[:n].view(self.B, n_heads, head_dim)
        self.part_ml = self.packed[n:].view(self.B, n_heads, 2)
        self.comm = None
        self._merge_packed = merge_fn is None
        if partial_fn is None or merge_fn is None:
            from . import ops
            self._ops = ops
            self.workspace = ops.Workspace(self.B, n_heads, n_kv_heads, head_dim, self.device)
        if partial_fn is None and merge_fn is None and self.device.type == "cuda" \
                and self.world > 1:
            uid = share_unique_id(self.rank, group)
            dev = self.device.index if self.device.index is not None else \
                torch.cuda.current_device()
            self.comm = Communicator(uid, self.world, self.rank, dev,
                                     step_deadline_ms=step_deadline_ms)
            nbytes = self.comm.workspace_bytes(self.B, n_heads, n_kv_heads, head_dim)
            self._mws = torch.zeros(nbytes + 256, dtype=torch.uint8, device=self.device)
            self._mws_ptr = (self._mws.data_ptr() + 255) // 256 * 256
            self._mws_bytes = nbytes
        self.partial_fn = partial_fn or self._partial_gpu
        self.merge_fn = merge_fn or self._merge_gpu

    # ---- default compute: the library's kernels ----
    def _partial_gpu(self, q):
        self._ops.attention_partial(q, self.k_pool, self.v_pool, self.row_offset, self.seq_len,
                                    self.part_o, self.part_ml, self.n_heads, self.n_kv_heads,
                                    self.head_dim, workspace=self.workspace)
        return self.part_o, self.part_ml

    def _merge_gpu(self, go, gml, out):
        return self._ops.merge(go, gml, out)

    def global_rows(self, b: int) -> tuple[int, int]:
        """Rows [lo, hi) of sequence b that this rank holds (global row numbers)."""
        return self.bounds[b]

    def append(self, k_new: torch.Tensor, v_new: torch.Tensor) -> None:
        """Append one row per sequence; the last rank holds the sequences' tails."""
        if not hasattr(self, "_ops"):
            raise RuntimeError("append runs the library's kv_append kernel")
        if self.rank == self.world - 1:
            self._ops.kv_append_batched(k_new, v_new, self.k_pool, self.v_pool, self.row_offset,
                                        self.seq_len)
            self.seq_len += 1
        self.lengths = [L + 1 for L in self.lengths]

    def step(self, q: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        """O[b, h] over all shards: local partial, all-gather, merge in rank order."""
        if out is None:
            out = torch.empty(self.B, self.n_heads, self.head_dim, dtype=torch.float16,
                              device=self.device)
        if self.comm is not None:
            ops = self._ops
            self.comm.decode_step(
                ops._h(q, "q"), ops._h(self.k_pool, "k_pool"), ops._h(self.v_pool, "v_pool"),
                self.pool_rows, ops._ptr(self.row_offset, torch.int64, "row_offset"),
                ops._ptr(self.seq_len, torch.int32, "seq_len"), ops._h(out, "o"), self.B,
                self.n_heads, self.n_kv_heads, self.head_dim, self._mws_ptr, self._mws_bytes,
                ops._stream())
            return out
        part_o, part_ml = self.partial_fn(q)
        if part_o.data_ptr() != self.part_o.data_ptr():  # an injected partial_fn
            self.part_o.copy_(part_o)
        if part_ml.data_ptr() != self.part_ml.data_ptr():
            self.part_ml.copy_(part_ml)
        g = gather_packed(self.packed, self.group)
        if self._merge_packed:
            return self._ops.merge_packed(g, out)
        go, gml = unpack_partials(g, self.B, self.n_heads, self.head_dim)
        return self.merge_fn(go, gml, out)

    def sync(self) -> None:
        """Waits for the last step (within the communicator's deadline on GPUs)."""
        if self.comm is not None:
            self.comm.sync()
        elif self.device.type == "cuda":
            torch.cuda.current_stream(self.device).synchronize()

    def close(self) -> None:
        if self.comm is not None:
            self.comm.close()
            self.comm = None
