"""Operator API of the decode-attention path, over torch CUDA tensors.

The names and argument meaning follow the reference's two WGSL kernels:

* ``kv_append(src, cache, KvParams(seq, n_kv, hd))`` — kernels/kv_append.wgsl
  (uniform ``Params{seq, n_kv, hd}``, kernels/kv_append.wgsl:1-6);
* ``attention(q, k_cache, v_cache, o, AttnParams(n_heads, n_kv_heads,
  head_dim, seq))`` — kernels/sparse_attn.wgsl (uniform ``Params{n_heads,
  n_kv_heads, head_dim, seq}``, kernels/sparse_attn.wgsl:12-17).

Differences from the WGSL, all intentional: fp16 storage with fp32
accumulation (the WGSL buffers are f32), no 256-row cap, an optional softmax
``scale`` (0 keeps the reference's inverseSqrt(head_dim)), a caller-visible
workspace for the split-KV partials, and ragged-batch / shard-partial
variants.  Errors raise :class:`NwdError` with the library's message, as the
reference throws ``Error`` (engine/runtime.js:448).

torch is used only to hold device memory and to name the current stream; all
computation runs in ``libnwd.so``.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch

from . import _lib
from ._lib import NwdError, call


@dataclass
class KvParams:
    """kernels/kv_append.wgsl:1-6 ``Params{seq, n_kv, hd}``."""
    seq: int
    n_kv: int
    hd: int


@dataclass
class AttnParams:
    """kernels/sparse_attn.wgsl:12-17 ``Params{n_heads, n_kv_heads, head_dim, seq}``."""
    n_heads: int
    n_kv_heads: int
    head_dim: int
    seq: int


def _stream(stream=None) -> int:
    if stream is None:
        stream = torch.cuda.current_stream()
    return int(stream.cuda_stream) if hasattr(stream, "cuda_stream") else int(stream)


def _ptr(t: torch.Tensor, dtype, name: str) -> int:
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor")
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor")
    if t.dtype != dtype:
        raise TypeError(f"{name} must be {dtype}, got {t.dtype}")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")
    return t.data_ptr()


def _h(t, name):
    return _ptr(t, torch.float16, name)


class Workspace:
    """Device scratch for the split-KV partials and the work queue.

    Sized for ``batch`` sequences of the given head shape on the current
    device and zero-filled once; calls leave it ready for the next call.
    Calls sharing one workspace must be ordered on one stream.
    """

    def __init__(self, batch: int, n_heads: int, n_kv_heads: int, head_dim: int,
                 device=None):
        lib = _lib.load()
        nbytes = ctypes.c_size_t(0)
        device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        with torch.cuda.device(device):
            _lib.check(lib.nwd_attn_decode_workspace_size(batch, n_heads, n_kv_heads, head_dim,
                                                          ctypes.byref(nbytes)))
            self.nbytes = int(nbytes.value)
            # +256 so the base can be rounded up to a 256-byte boundary
            self._buf = torch.zeros(self.nbytes + 256, dtype=torch.uint8, device=device)
        base = self._buf.data_ptr()
        self.ptr = (base + 255) // 256 * 256
        self.shape = (batch, n_heads, n_kv_heads, head_dim)
        self.device = device

    def fits(self, batch: int, n_heads: int, n_kv_heads: int, head_dim: int) -> bool:
        # the library derives the workspace layout from the call's shape, so a
        # workspace serves exactly the shape it was sized (and zeroed) for
        return self.shape == (batch, n_heads, n_kv_heads, head_dim)

    def check(self, stream=None) -> int:
        """Synchronously read and clear the device-side error word (0 = ok)."""
        v = ctypes.c_uint32(0)
        call("nwd_workspace_check", self.ptr, self.nbytes, ctypes.byref(v), _stream(stream))
        return int(v.value)


_ws_cache: dict = {}


def _workspace(batch, n_heads, n_kv, hd, device, ws):
    if ws is not None:
        return ws
    key = (device.index if device.index is not None else torch.cuda.current_device(),
           batch, n_heads, n_kv, hd)
    cur = _ws_cache.get(key)
    if cur is None:
        cur = Workspace(batch, n_heads, n_kv, hd, device)
        _ws_cache[key] = cur
    return cur


# ---------------------------------------------------------------- kv_append

def kv_append(src: torch.Tensor, cache: torch.Tensor, params: KvParams, stream=None) -> None:
    """Write ``src`` ([n_kv*hd] fp16) into row ``params.seq`` of ``cache``.

    ``cache`` is [max_seq, n_kv, hd] (any shape with max_seq rows of n_kv*hd);
    ``seq >= max_seq`` raises NwdError (NWD_ERR_RANGE) without launching.
    """
    n = params.n_kv * params.hd
    if src.numel() < n:
        raise ValueError(f"src has {src.numel()} elements, need {n}")
    cap = cache.numel() // n
    call("nwd_kv_append", _h(src, "src"), _h(cache, "cache"), params.seq, params.n_kv, params.hd,
         cap, _stream(stream))


def kv_append_kv(k_src, v_src, k_cache, v_cache, params: KvParams, stream=None) -> None:
    """Both of the engine's kv_append dispatches (runtime.js:389-390) in one launch."""
    n = params.n_kv * params.hd
    cap = k_cache.numel() // n
    if v_cache.numel() // n != cap:
        raise ValueError("k_cache and v_cache differ in capacity")
    call("nwd_kv_append_kv", _h(k_src, "k_src"), _h(v_src, "v_src"), _h(k_cache, "k_cache"),
         _h(v_cache, "v_cache"), params.seq, params.n_kv, params.hd, cap, _stream(stream))


def kv_append_batched(k_src, v_src, k_pool, v_pool, row_offset, pos, err_count=None,
                      stream=None) -> None:
    """Sequence b writes k_src[b]/v_src[b] into pool row row_offset[b] + pos[b]."""
    batch = pos.numel()
    n_kv, hd = k_src.shape[-2], k_src.shape[-1]
    rows = k_pool.numel() // (n_kv * hd)
    ec = _ptr(err_count, torch.int32, "err_count") if err_count is not None else None
    call("nwd_kv_append_batched", _h(k_src, "k_src"), _h(v_src, "v_src"), _h(k_pool, "k_pool"),
         _h(v_pool, "v_pool"), rows, _ptr(row_offset, torch.int64, "row_offset"),
         _ptr(pos, torch.int32, "pos"), batch, n_kv, hd, ec, _stream(stream))


# ---------------------------------------------------------------- attention

def attention(q, k_cache, v_cache, o, params: AttnParams, scale: float = 0.0, workspace=None,
              stream=None) -> torch.Tensor:
    """One dispatch of kernels/sparse_attn.wgsl: o[h] = softmax(q[h].K^T) V over ``seq`` rows."""
    n = params.n_kv_heads * params.head_dim
    cap = k_cache.numel() // n
    ws = _workspace(1, params.n_heads, params.n_kv_heads, params.head_dim, q.device, workspace)
    call("nwd_attn_decode", _h(q, "q"), _h(k_cache, "k_cache"), _h(v_cache, "v_cache"),
         _h(o, "o"), params.n_heads, params.n_kv_heads, params.head_dim, params.seq, cap,
         float(scale), ws.ptr, ws.nbytes, _stream(stream))
    return o


def kv_append_attention(q, k_new, v_new, k_cache, v_cache, o, params: AttnParams,
                        scale: float = 0.0, workspace=None, stream=None) -> torch.Tensor:
    """The engine's attention-layer step (runtime.js:389-391, uniforms of :451-452):
    write k_new/v_new at row ``params.seq``, then attend over ``params.seq + 1`` rows."""
    n = params.n_kv_heads * params.head_dim
    cap = k_cache.numel() // n
    ws = _workspace(1, params.n_heads, params.n_kv_heads, params.head_dim, q.device, workspace)
    call("nwd_kv_append_attn_decode", _h(q, "q"), _h(k_new, "k_new"), _h(v_new, "v_new"),
         _h(k_cache, "k_cache"), _h(v_cache, "v_cache"), _h(o, "o"), params.n_heads,
         params.n_kv_heads, params.head_dim, params.seq, cap, float(scale), ws.ptr, ws.nbytes,
         _stream(stream))
    return o


def attention_batched(q, k_pool, v_pool, row_offset, seq_len, o, n_heads, n_kv_heads, head_dim,
                      scale: float = 0.0, workspace=None, stream=None) -> torch.Tensor:
    """Ragged batch: q/o [B, n_heads, head_dim]; sequence b attends pool rows
    [row_offset[b], row_offset[b] + seq_len[b])."""
    batch = seq_len.numel()
    rows = k_pool.numel() // (n_kv_heads * head_dim)
    ws = _workspace(batch, n_heads, n_kv_heads, head_dim, q.device, workspace)
    call("nwd_attn_decode_batched", _h(q, "q"), _h(k_pool, "k_pool"), _h(v_pool, "v_pool"), rows,
         _ptr(row_offset, torch.int64, "row_offset"), _ptr(seq_len, torch.int32, "seq_len"),
         _h(o, "o"), batch, n_heads, n_kv_heads, head_dim, float(scale), ws.ptr, ws.nbytes,
         _stream(stream))
    return o


def kv_append_attention_batched(q, k_new, v_new, k_pool, v_pool, row_offset, pos, o, n_heads,
                                n_kv_heads, head_dim, scale: float = 0.0, workspace=None,
                                stream=None) -> torch.Tensor:
    """Batched engine step: sequence b writes its new row at pos[b], attends pos[b] + 1 rows."""
    batch = pos.numel()
    rows = k_pool.numel() // (n_kv_heads * head_dim)
    ws = _workspace(batch, n_heads, n_kv_heads, head_dim, q.device, workspace)
    call("nwd_kv_append_attn_decode_batched", _h(q, "q"), _h(k_new, "k_new"), _h(v_new, "v_new"),
         _h(k_pool, "k_pool"), _h(v_pool, "v_pool"), rows,
         _ptr(row_offset, torch.int64, "row_offset"), _ptr(pos, torch.int32, "pos"), _h(o, "o"),
         batch, n_heads, n_kv_heads, head_dim, float(scale), ws.ptr, ws.nbytes, _stream(stream))
    return o


def attention_partial(q, k_pool, v_pool, row_offset, seq_len, part_o, part_ml, n_heads,
                      n_kv_heads, head_dim, scale: float = 0.0, workspace=None, stream=None):
    """Shard partials: part_o [B, n_heads, hd] f32 (unnormalised), part_ml [B, n_heads, 2]
    f32 = (max in log2 units, sum of 2^(s - max))."""
    batch = seq_len.numel()
    rows = k_pool.numel() // (n_kv_heads * head_dim)
    ws = _workspace(batch, n_heads, n_kv_heads, head_dim, q.device, workspace)
    call("nwd_attn_decode_partial", _h(q, "q"), _h(k_pool, "k_pool"), _h(v_pool, "v_pool"), rows,
         _ptr(row_offset, torch.int64, "row_offset"), _ptr(seq_len, torch.int32, "seq_len"),
         _ptr(part_o, torch.float32, "part_o"), _ptr(part_ml, torch.float32, "part_ml"), batch,
         n_heads, n_kv_heads, head_dim, float(scale), ws.ptr, ws.nbytes, _stream(stream))
    return part_o, part_ml


def merge(part_o, part_ml, o, stream=None) -> torch.Tensor:
    """LSE-merge [shards, B, n_heads, hd] partials into o [B, n_heads, hd] fp16."""
    shards = part_o.shape[0]
    batch, n_heads, hd = o.shape[-3], o.shape[-2], o.shape[-1]
    call("nwd_attn_merge", _ptr(part_o, torch.float32, "part_o"),
         _ptr(part_ml, torch.float32, "part_ml"), _h(o, "o"), shards, batch, n_heads, hd,
         _stream(stream))
    return o


def packed_partials(batch: int, n_heads: int, head_dim: int = 128, device=None):
    """One buffer of B*n_heads*(hd+2) f32 and its (part_o, part_ml) views, the layout
    nwd_attn_merge_packed reads (o first, then the (m, l) pairs)."""
    n = batch * n_heads * head_dim
    buf = torch.empty(n + batch * n_heads * 2, dtype=torch.float32, device=device)
    return buf, buf[:n].view(batch, n_heads, head_dim), buf[n:].view(batch, n_heads, 2)


def merge_packed(packed, o, stream=None) -> torch.Tensor:
    """LSE-merge gathered packed partials [shards, B*n_heads*(hd+2)] into o [B, n_heads, hd]."""
    shards = packed.shape[0]
    batch, n_heads, hd = o.shape[-3], o.shape[-2], o.shape[-1]
    if packed.numel() != shards * batch * n_heads * (hd + 2):
        raise ValueError("packed partials do not match o's shape")
    call("nwd_attn_merge_packed", _ptr(packed, torch.float32, "packed"), _h(o, "o"), shards,
         batch, n_heads, hd, _stream(stream))
    return o


class Scratch:
    """A zeroed 256-byte-aligned device header for calls that only need the
    error word (prefill, multi-row appends)."""

    def __init__(self, device=None):
        device = torch.device(device) if device is not None else torch.device(
            "cuda", torch.cuda.current_device())
        self._buf = torch.zeros(512, dtype=torch.uint8, device=device)
        self.ptr = (self._buf.data_ptr() + 255) // 256 * 256
        self.nbytes = 256

    def check(self, stream=None) -> int:
        v = ctypes.c_uint32(0)
        call("nwd_workspace_check", self.ptr, self.nbytes, ctypes.byref(v), _stream(stream))
        return int(v.value)


_scratch_cache: dict = {}


def _scratch(device, ws):
    if ws is not None:
        return ws
    key = device.index if device.index is not None else torch.cuda.current_device()
    if key not in _scratch_cache:
        _scratch_cache[key] = Scratch(device)
    return _scratch_cache[key]


def kv_append_rows(k_src, v_src, k_pool, v_pool, row_offset, start_pos: int, workspace=None,
                   stream=None) -> None:
    """Prompt-chunk rows [batch, n_rows, n_kv, hd] into pool rows row_offset[b] + start_pos + i."""
    batch, n_rows, n_kv, hd = k_src.shape
    rows = k_pool.numel() // (n_kv * hd)
    ws = _scratch(k_src.device, workspace)
    call("nwd_kv_append_rows", _h(k_src, "k_src"), _h(v_src, "v_src"), _h(k_pool, "k_pool"),
         _h(v_pool, "v_pool"), rows, _ptr(row_offset, torch.int64, "row_offset"), start_pos,
         n_rows, batch, n_kv, hd, ws.ptr, ws.nbytes, _stream(stream))


def attention_prefill(q, k_pool, v_pool, row_offset, o, start_pos: int, n_heads: int,
                      n_kv_heads: int, head_dim: int = 128, scale: float = 0.0, workspace=None,
                      stream=None) -> torch.Tensor:
    """Causal prefill of a chunk: q/o [batch, n_q, n_heads, hd]; token i attends pool rows
    row_offset[b] + [0, start_pos + i] (tcgen05 tensor cores)."""
    batch, n_q = q.shape[0], q.shape[1]
    rows = k_pool.numel() // (n_kv_heads * head_dim)
    ws = _scratch(q.device, workspace)
    call("nwd_attn_prefill", _h(q, "q"), _h(k_pool, "k_pool"), _h(v_pool, "v_pool"), rows,
         _ptr(row_offset, torch.int64, "row_offset"), _h(o, "o"), batch, n_q, start_pos, n_heads,
         n_kv_heads, head_dim, float(scale), ws.ptr, ws.nbytes, _stream(stream))
    return o


@dataclass
class Q4Weights:
    """One q4 matrix in the reference's MatMulNBits layout (what the engine loads):
    b [N, n_blocks, 4] uint32 (int32 storage is accepted), scales [N, n_blocks] f32,
    zp [ceil(N*n_blocks/8)] uint32 (4-bit zero points, 8 per word)."""
    b: torch.Tensor
    scales: torch.Tensor
    zp: torch.Tensor

    @property
    def n(self) -> int:
        return int(self.scales.shape[0])

    @property
    def n_blocks(self) -> int:
        return int(self.scales.shape[1])

    def ptrs(self):
        for t, name in ((self.b, "b"), (self.zp, "zp")):
            if t.dtype not in (torch.int32, torch.uint32):
                raise TypeError(f"q4 {name} must be 32-bit words, got {t.dtype}")
            if not (t.is_cuda and t.is_contiguous()):
                raise ValueError(f"q4 {name} must be a contiguous CUDA tensor")
        return self.b.data_ptr(), _ptr(self.scales, torch.float32, "scales"), self.zp.data_ptr()


def q4_gemv(a: torch.Tensor, w: Q4Weights, y: torch.Tensor | None = None, epilogue: int = 0,
            stream=None) -> torch.Tensor:
    """kernels/matmul_nbits_sg.wgsl: y [N] f32 from a [K] (f32, or fp16 for o_proj).
    epilogue 0 = store, 1 = relu2, 2 = y += result (residual add)."""
    if y is None:
        y = torch.zeros(w.n, dtype=torch.float32, device=a.device)
    K = a.numel()
    bp, sp, zp = w.ptrs()
    if a.dtype == torch.float16:
        call("nwd_q4_gemv_f16a", _h(a, "a"), bp, sp, zp, _ptr(y, torch.float32, "y"), K, w.n,
             w.n_blocks, int(epilogue), _stream(stream))
    else:
        call("nwd_q4_gemv", _ptr(a, torch.float32, "a"), bp, sp, zp, _ptr(y, torch.float32, "y"),
             K, w.n, w.n_blocks, int(epilogue), _stream(stream))
    return y


def q4_qkv_append(h: torch.Tensor, wq: Q4Weights, wk: Q4Weights, wv: Q4Weights,
                  q_out: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, seq: int,
                  stream=None) -> torch.Tensor:
    """The layer's q / k / v projections in one launch; k and v land in cache row `seq`
    ([cap, n_kv, hd] fp16), q in q_out [n_heads, hd] fp16 (runtime.js:321-329, :389-391)."""
    cap, n_kv, hd = k_cache.shape
    n_heads = q_out.numel() // hd
    if wq.n != n_heads * hd or wk.n != n_kv * hd or wv.n != n_kv * hd:
        raise ValueError("q/k/v weight columns do not match the output shapes")
    qb, qs, qz = wq.ptrs()
    kb, ks, kz = wk.ptrs()
    vb, vs, vz = wv.ptrs()
    call("nwd_q4_qkv_append", _ptr(h, torch.float32, "h"), qb, qs, qz, kb, ks, kz, vb, vs, vz,
         _h(q_out, "q_out"), _h(k_cache, "k_cache"), _h(v_cache, "v_cache"), int(seq), cap,
         h.numel(), n_heads, n_kv, hd, _stream(stream))
    return q_out


def selftest_wait_timeout(workspace: "Workspace", stream=None) -> int:
    """Make one of the library's bounded device waits run out (about 2 s) and return the
    workspace's device error word afterwards (NWD_DEVERR_PIPE_TIMEOUT expected); the
    stream stays usable."""
    call("nwd_selftest_wait_timeout", workspace.ptr, workspace.nbytes, _stream(stream))
    return workspace.check(stream)


def prefetch_l2(buffers, stream=None) -> None:
    """Start up to 16 CUDA tensors (e.g. the next projection's q4 weights) on their way
    into L2 on `stream`.  A hint: it never changes a result."""
    buffers = list(buffers)
    for i, t in enumerate(buffers):
        if not isinstance(t, torch.Tensor) or not t.is_cuda or not t.is_contiguous():
            raise ValueError(f"buffer {i} must be a contiguous CUDA tensor")
    n = len(buffers)
    ptrs = (ctypes.c_void_p * max(n, 1))(*[t.data_ptr() for t in buffers])
    sizes = (ctypes.c_uint64 * max(n, 1))(*[t.numel() * t.element_size() for t in buffers])
    call("nwd_prefetch_l2", ctypes.cast(ptrs, ctypes.c_void_p), ctypes.cast(sizes, ctypes.c_void_p),
         n, _stream(stream))


def decode_plan(batch: int, n_heads: int, n_kv_heads: int, seq: int, head_dim: int = 128):
    """How a decode call of this shape runs on the current device (no launch):
    {kernel: "split"|"short", grid, split, cluster, groups} (nwd_attn_decode_plan)."""
    v = [ctypes.c_int() for _ in range(5)]
    call("nwd_attn_decode_plan", batch, n_heads, n_kv_heads, head_dim, seq,
         *[ctypes.byref(x) for x in v])
    k, grid, split, cluster, groups = (int(x.value) for x in v)
    return {"kernel": "short" if k == 1 else "split", "grid": grid, "split": split,
            "cluster": cluster, "groups": groups}


def fill_normal(t: torch.Tensor, seed: int, offset: int = 0, stream=None) -> torch.Tensor:
    """Fill an fp16 tensor with the deterministic N(0,1) stream (bit-identical to the CPU
    generator used by the tests)."""
    call("nwd_fill_normal_f16", _h(t, "t"), t.numel(), int(seed), int(offset), _stream(stream))
    return t


__all__ = [
    "KvParams", "AttnParams", "Workspace", "NwdError", "kv_append", "kv_append_kv",
    "kv_append_batched", "attention", "kv_append_attention", "attention_batched",
    "kv_append_attention_batched", "attention_partial", "merge", "fill_normal", "Scratch",
    "kv_append_rows", "attention_prefill", "packed_partials", "merge_packed", "Q4Weights",
    "q4_gemv", "q4_qkv_append",
]
