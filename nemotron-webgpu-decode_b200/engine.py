"""Attention-layer state of the reference's DecodeEngine, on the B200 library.

``engine/runtime.js`` keeps, per attention layer, two f32 caches of
``maxSeq * kvHeads * headDim`` (runtime.js:170-173), a step counter ``seq``
(runtime.js:66, :467) and two uniforms rewritten every step
(``uKv[0] = seq``, ``uAttn[3] = seq + 1``, runtime.js:451-452).  Each step
dispatches kv_append(K), kv_append(V) and attention (runtime.js:389-391) and
throws once ``seq`` reaches ``maxSeq`` (runtime.js:448).  ``reset()`` wipes the
caches (runtime.js:615-633).

:class:`DecodeAttention` is that slice for one layer, with fp16 caches and the
three dispatches fused into one launch; :class:`BatchedDecodeAttention` is
the same for a ragged batch of independent sequences sharing one KV pool.
"""
from __future__ import annotations

import torch

from . import ops
from ._lib import NWD_ERR_RANGE, NwdError

# engine/config.js:10-12, :24
NANO4B_HEADS = 40
NANO4B_KV_HEADS = 8
NANO4B_HEAD_DIM = 128
NANO4B_MAX_SEQ = 256


class DecodeAttention:
    """One attention layer's KV cache + step (runtime.js:170-173, :389-391, :447-467)."""

    def __init__(self, heads: int = NANO4B_HEADS, kv_heads: int = NANO4B_KV_HEADS,
                 head_dim: int = NANO4B_HEAD_DIM, max_seq: int = NANO4B_MAX_SEQ,
                 device="cuda", scale: float = 0.0):
        self.heads, self.kv_heads, self.head_dim, self.max_seq = heads, kv_heads, head_dim, max_seq
        self.device = torch.device(device)
        self.scale = scale
        self.k_cache = torch.zeros(max_seq, kv_heads, head_dim, dtype=torch.float16,
                                   device=self.device)
        self.v_cache = torch.zeros_like(self.k_cache)
        self.workspace = ops.Workspace(1, heads, kv_heads, head_dim, self.device)
        self.seq = 0

    def step(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
             out: torch.Tensor | None = None, stream=None) -> torch.Tensor:
        """Append this token's k/v at row ``seq`` and attend over ``seq + 1`` rows."""
        if self.seq >= self.max_seq:
            raise NwdError(NWD_ERR_RANGE, f"seq {self.seq} exceeds maxSeq {self.max_seq}")
        if out is None:
            out = torch.empty(self.heads, self.head_dim, dtype=torch.float16, device=self.device)
        params = ops.AttnParams(self.heads, self.kv_heads, self.head_dim, self.seq)
        ops.kv_append_attention(q, k, v, self.k_cache, self.v_cache, out, params,
                                scale=self.scale, workspace=self.workspace, stream=stream)
        self.seq += 1
        return out

    def prefill(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                out: torch.Tensor | None = None, stream=None) -> torch.Tensor:
        """A prompt chunk of n tokens in two launches instead of n steps.

        runtime.js:640-646 feeds a prompt one decode step per token; token i of
        this chunk sees exactly the rows those steps would give it (0 .. seq + i).
        q [n, heads, hd], k / v [n, kv_heads, hd] -> o [n, heads, hd]; the chunk's
        k / v rows land at rows seq .. seq + n - 1 (the kv_append path for many
        rows) and seq advances by n.  A chunk that would run past maxSeq is
        refused before any launch, with the error the first step past it throws.
        """
        n = int(q.shape[0])
        if self.seq + n > self.max_seq:
            raise NwdError(NWD_ERR_RANGE, f"seq {self.max_seq} exceeds maxSeq {self.max_seq}")
        if out is None:
            out = torch.empty(n, self.heads, self.head_dim, dtype=torch.float16,
                              device=self.device)
        if n == 0:
            return out
        if not hasattr(self, "_row0"):
            self._row0 = torch.zeros(1, dtype=torch.int64, device=self.device)
        kv_shape = (1, n, self.kv_heads, self.head_dim)
        ops.kv_append_rows(k.reshape(kv_shape), v.reshape(kv_shape), self.k_cache, self.v_cache,
                           self._row0, self.seq, workspace=self.workspace, stream=stream)
        ops.attention_prefill(q.reshape(1, n, self.heads, self.head_dim), self.k_cache,
                              self.v_cache, self._row0, out.view(1, n, self.heads, self.head_dim),
                              self.seq, self.heads, self.kv_heads, self.head_dim,
                              scale=self.scale, workspace=self.workspace, stream=stream)
        self.seq += n
        return out

    def reset(self) -> None:
        """runtime.js:615-633: seq = 0 and the caches wiped."""
        self.seq = 0
        self.k_cache.zero_()
        self.v_cache.zero_()


class AttentionLayer:
    """One attention layer of the engine with the projections either side of the
    path (runtime.js:321-335 builds it, :385-394 dispatches it): the q / k / v q4
    GEMVs of the normalised hidden state, kv_append of k and v, attention, the
    o_proj q4 GEMV and the residual add into the hidden state.  Here: one launch
    for q/k/v with k/v written straight into the caches, one for attention, one for
    o_proj with the residual add fused.  Weights stay in the MatMulNBits layout
    (:class:`ops.Q4Weights`)."""

    def __init__(self, wq: ops.Q4Weights, wk: ops.Q4Weights, wv: ops.Q4Weights,
                 wo: ops.Q4Weights, heads: int = NANO4B_HEADS, kv_heads: int = NANO4B_KV_HEADS,
                 head_dim: int = NANO4B_HEAD_DIM, max_seq: int = NANO4B_MAX_SEQ, device="cuda",
                 scale: float = 0.0):
        self.attn = DecodeAttention(heads, kv_heads, head_dim, max_seq, device, scale)
        self.wq, self.wk, self.wv, self.wo = wq, wk, wv, wo
        dev = self.attn.device
        self.q = torch.empty(heads, head_dim, dtype=torch.float16, device=dev)
        self.o = torch.empty(heads, head_dim, dtype=torch.float16, device=dev)

    @property
    def seq(self) -> int:
        return self.attn.seq

    def qkv_weights(self) -> list:
        """The q / k / v weight buffers (what the layer's first launch reads)."""
        return [t for w in (self.wq, self.wk, self.wv) for t in (w.b, w.scales, w.zp)]

    def step(self, h_norm: torch.Tensor, h: torch.Tensor, stream=None,
             prefetch=None) -> torch.Tensor:
        """h += o_proj(attention(q, K, V)) for this token; h_norm [hidden] f32 is the
        layer's normalised input, h [hidden] f32 the residual stream (updated in place).

        prefetch = (side_stream, buffers): once the q/k/v launch is done, side_stream
        starts this layer's o_proj weights and `buffers` (e.g. the next layer's
        :meth:`qkv_weights`) into L2 while attention runs; the caller joins
        side_stream before it next needs it.  Results do not change."""
        a = self.attn
        if a.seq >= a.max_seq:
            raise NwdError(NWD_ERR_RANGE, f"seq {a.seq} exceeds maxSeq {a.max_seq}")
        ops.q4_qkv_append(h_norm, self.wq, self.wk, self.wv, self.q, a.k_cache, a.v_cache,
                          a.seq, stream=stream)
        if prefetch is not None:
            side, extra = prefetch
            side.wait_stream(stream if stream is not None else torch.cuda.current_stream())
            ops.prefetch_l2([self.wo.b, self.wo.scales, self.wo.zp] + list(extra), stream=side)
        ops.attention(self.q, a.k_cache, a.v_cache, self.o,
                      ops.AttnParams(a.heads, a.kv_heads, a.head_dim, a.seq + 1),
                      scale=a.scale, workspace=a.workspace, stream=stream)
        ops.q4_gemv(self.o.view(-1), self.wo, y=h, epilogue=2, stream=stream)
        a.seq += 1
        return h

    def reset(self) -> None:
        self.attn.reset()


def step_layers(layers, h_norm: torch.Tensor, h: torch.Tensor, side=None, stream=None):
    """One token through consecutive attention layers (h_norm [n_layers, hidden]).  With a
    side stream, each layer's o_proj weights and the next layer's q/k/v weights are
    prefetched into L2 during its attention launch; the side stream is joined at the end."""
    cur = stream if stream is not None else torch.cuda.current_stream()
    for i, layer in enumerate(layers):
        pf = None
        if side is not None:
            pf = (side, layers[i + 1].qkv_weights() if i + 1 < len(layers) else [])
        layer.step(h_norm[i], h, stream=stream, prefetch=pf)
    if side is not None:
        cur.wait_stream(side)
    return h


class BatchedDecodeAttention:
    """Ragged batch of sequences in one pool: sequence b owns pool rows
    [row_offset[b], row_offset[b] + capacity[b]) and has ``lengths[b]`` rows."""

    def __init__(self, capacities, heads: int, kv_heads: int, head_dim: int = 128,
                 device="cuda", scale: float = 0.0):
        self.device = torch.device(device)
        caps = torch.as_tensor(list(capacities), dtype=torch.int64)
        self.batch = int(caps.numel())
        offs = torch.zeros_like(caps)
        if self.batch > 1:
            offs[1:] = torch.cumsum(caps, 0)[:-1]
        self.capacity = caps
        self.pool_rows = int(caps.sum())
        self.heads, self.kv_heads, self.head_dim = heads, kv_heads, head_dim
        self.scale = scale
        self.k_pool = torch.zeros(self.pool_rows, kv_heads, head_dim, dtype=torch.float16,
                                  device=self.device)
        self.v_pool = torch.zeros_like(self.k_pool)
        self.row_offset = offs.to(self.device)
        self.lengths = torch.zeros(self.batch, dtype=torch.int32, device=self.device)
        self.workspace = ops.Workspace(self.batch, heads, kv_heads, head_dim, self.device)

    def step(self, q, k_new, v_new, out=None, stream=None) -> torch.Tensor:
        """Every sequence appends one row and attends over its rows (fused launch)."""
        if out is None:
            out = torch.empty(self.batch, self.heads, self.head_dim, dtype=torch.float16,
                              device=self.device)
        ops.kv_append_attention_batched(q, k_new, v_new, self.k_pool, self.v_pool,
                                        self.row_offset, self.lengths, out, self.heads,
                                        self.kv_heads, self.head_dim, scale=self.scale,
                                        workspace=self.workspace, stream=stream)
        self.lengths += 1
        return out

    def attend(self, q, out=None, stream=None) -> torch.Tensor:
        if out is None:
            out = torch.empty(self.batch, self.heads, self.head_dim, dtype=torch.float16,
                              device=self.device)
        return ops.attention_batched(q, self.k_pool, self.v_pool, self.row_offset, self.lengths,
                                     out, self.heads, self.kv_heads, self.head_dim,
                                     scale=self.scale, workspace=self.workspace, stream=stream)
