"""numpy front end of the CPU oracle (``oracle/nwd_oracle.c``).

TEST INFRASTRUCTURE ONLY: imported by ``tests/``, ``__graft_entry__.smoke()``
and the CPU-baseline legs of ``bench.py``, as the checker or the timed CPU
baseline.  The product path (``nemotron-webgpu-decode_b200``) never imports it.

The C file restates ``kernels/sparse_attn.wgsl:32-113``,
``kernels/kv_append.wgsl:13-18`` and the q4 GEMV ``kernels/matmul_nbits_sg.wgsl``
(+ ``kernels/add.wgsl``) of the reference; parity is unpinned (the reference has
no tests or golden vectors, and its WGSL cannot run here).
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")

_lib = None

_u16p = np.ctypeslib.ndpointer(np.uint16, flags="C_CONTIGUOUS")
_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_f64p = np.ctypeslib.ndpointer(np.float64, flags="C_CONTIGUOUS")
_i64p = np.ctypeslib.ndpointer(np.int64, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")
_u32p = np.ctypeslib.ndpointer(np.uint32, flags="C_CONTIGUOUS")
_u32 = ctypes.c_uint32
_u64 = ctypes.c_uint64


def build(force: bool = False) -> str:
    """Compile liboracle.so with the committed Makefile (if out of date)."""
    src = os.path.join(HERE, "nwd_oracle.c")
    if force or not os.path.exists(LIB_PATH) or os.path.getmtime(LIB_PATH) < os.path.getmtime(src):
        subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = ctypes.CDLL(LIB_PATH)
        L.oracle_h2f.restype = ctypes.c_float
        L.oracle_h2f.argtypes = [ctypes.c_uint16]
        L.oracle_f2h.restype = ctypes.c_uint16
        L.oracle_f2h.argtypes = [ctypes.c_float]
        L.oracle_h2f_array.argtypes = [_u16p, _f32p, _u64]
        L.oracle_f2h_array.argtypes = [_f32p, _u16p, _u64]
        L.oracle_normal_f16.restype = ctypes.c_uint16
        L.oracle_normal_f16.argtypes = [_u64, _u64]
        L.oracle_fill_normal_f16.argtypes = [_u16p, _u64, _u64, _u64]
        L.oracle_kv_append.argtypes = [_u16p, _u16p, _u32, _u32, _u32]
        L.oracle_attn_f32.argtypes = [_u16p, _u16p, _u16p, _f32p, _u32, _u32, _u32, _u32, ctypes.c_float]
        L.oracle_attn_batched_f32.argtypes = [_u16p, _u16p, _u16p, _i64p, _i32p, _f32p,
                                              _u32, _u32, _u32, _u32, ctypes.c_float]
        L.oracle_attn_batched_f64.argtypes = [_u16p, _u16p, _u16p, _i64p, _i32p, _f64p,
                                              _u32, _u32, _u32, _u32, ctypes.c_double]
        L.oracle_attn_partial.argtypes = [_u16p, _u16p, _u16p, _i64p, _i32p, _f32p, _f32p,
                                          _u32, _u32, _u32, _u32, ctypes.c_float]
        L.oracle_attn_merge.argtypes = [_f32p, _f32p, _f32p, _u32, _u32, _u32]
        L.oracle_attn_prefill_f32.argtypes = [_u16p, _u16p, _u16p, _i64p, _f32p, _u32, _u32, _u32,
                                              _u32, _u32, _u32, ctypes.c_float]
        L.oracle_q4_gemv_f32.argtypes = [_f32p, _u32p, _f32p, _u32p, _f32p, _u32, _u32, _u32]
        L.oracle_q4_gemv_f64.argtypes = [_f32p, _u32p, _f32p, _u32p, _f64p, _u32, _u32]
        L.oracle_fill_q4.argtypes = [_u32p, _f32p, _u32p, _u32, _u32, _u64]
        L.oracle_num_threads.restype = ctypes.c_int
        L.oracle_set_num_threads.argtypes = [ctypes.c_int]
        _lib = L
    return _lib


def _u16(a) -> np.ndarray:
    a = np.ascontiguousarray(a)
    if a.dtype == np.float16:
        a = a.view(np.uint16)
    assert a.dtype == np.uint16, a.dtype
    return a


def f16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    bits = _u16(bits)
    out = np.empty(bits.shape, np.float32)
    lib().oracle_h2f_array(bits.reshape(-1), out.reshape(-1), bits.size)
    return out


def f32_to_f16_bits(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.shape, np.uint16)
    lib().oracle_f2h_array(x.reshape(-1), out.reshape(-1), x.size)
    return out


def normal_f16(n: int, seed: int, offset: int = 0) -> np.ndarray:
    """The deterministic fp16 N(0,1) stream (bit patterns) the GPU generator also makes."""
    out = np.empty(int(n), np.uint16)
    lib().oracle_fill_normal_f16(out, int(n), int(seed), int(offset))
    return out


def kv_append(src, cache, seq: int, n_kv: int, hd: int) -> None:
    """kernels/kv_append.wgsl:13-18, in place on ``cache`` (uint16 bits)."""
    src = _u16(src).reshape(-1)
    assert cache.dtype == np.uint16 and cache.flags["C_CONTIGUOUS"]
    lib().oracle_kv_append(src, cache.reshape(-1), seq, n_kv, hd)


def attention(q, k_cache, v_cache, n_heads: int, n_kv_heads: int, head_dim: int, seq: int,
              scale: float = 0.0) -> np.ndarray:
    """kernels/sparse_attn.wgsl:32-113 on fp16 inputs; returns f32 [n_heads, head_dim]."""
    out = np.empty((n_heads, head_dim), np.float32)
    lib().oracle_attn_f32(_u16(q).reshape(-1), _u16(k_cache).reshape(-1),
                          _u16(v_cache).reshape(-1), out, n_heads, n_kv_heads, head_dim, seq,
                          float(scale))
    return out


def attention_batched(q, k_pool, v_pool, row_offset, seq_len, n_heads: int, n_kv_heads: int,
                      head_dim: int, scale: float = 0.0, f64: bool = False) -> np.ndarray:
    """Ragged batch of the reference kernel; returns [batch, n_heads, head_dim] f32 (or f64)."""
    row_offset = np.ascontiguousarray(row_offset, dtype=np.int64)
    seq_len = np.ascontiguousarray(seq_len, dtype=np.int32)
    batch = len(seq_len)
    if f64:
        out = np.empty((batch, n_heads, head_dim), np.float64)
        lib().oracle_attn_batched_f64(_u16(q).reshape(-1), _u16(k_pool).reshape(-1),
                                      _u16(v_pool).reshape(-1), row_offset, seq_len,
                                      out.reshape(-1), batch, n_heads, n_kv_heads, head_dim,
                                      float(scale))
    else:
        out = np.empty((batch, n_heads, head_dim), np.float32)
        lib().oracle_attn_batched_f32(_u16(q).reshape(-1), _u16(k_pool).reshape(-1),
                                      _u16(v_pool).reshape(-1), row_offset, seq_len,
                                      out.reshape(-1), batch, n_heads, n_kv_heads, head_dim,
                                      float(scale))
    return out


def attention_partial(q, k_pool, v_pool, row_offset, seq_len, n_heads: int, n_kv_heads: int,
                      head_dim: int, scale: float = 0.0):
    """Shard partial (m, l in log2 units; unnormalised o) per (b, h)."""
    row_offset = np.ascontiguousarray(row_offset, dtype=np.int64)
    seq_len = np.ascontiguousarray(seq_len, dtype=np.int32)
    batch = len(seq_len)
    part_o = np.empty((batch, n_heads, head_dim), np.float32)
    part_ml = np.empty((batch, n_heads, 2), np.float32)
    lib().oracle_attn_partial(_u16(q).reshape(-1), _u16(k_pool).reshape(-1),
                              _u16(v_pool).reshape(-1), row_offset, seq_len,
                              part_o.reshape(-1), part_ml.reshape(-1), batch, n_heads,
                              n_kv_heads, head_dim, float(scale))
    return part_o, part_ml


def merge(part_o: np.ndarray, part_ml: np.ndarray) -> np.ndarray:
    """Log-sum-exp merge of [shards, rows, hd] / [shards, rows, 2] partials -> [rows, hd] f32."""
    part_o = np.ascontiguousarray(part_o, dtype=np.float32)
    part_ml = np.ascontiguousarray(part_ml, dtype=np.float32)
    shards = part_o.shape[0]
    hd = part_o.shape[-1]
    rows = part_o.size // (shards * hd)
    out = np.empty((rows, hd), np.float32)
    lib().oracle_attn_merge(part_o.reshape(-1), part_ml.reshape(-1), out.reshape(-1), shards,
                            rows, hd)
    return out


def attention_prefill(q, k_pool, v_pool, row_offset, n_q: int, start_pos: int, n_heads: int,
                      n_kv_heads: int, head_dim: int, scale: float = 0.0) -> np.ndarray:
    """Causal prefill as the reference computes it (one decode step per prompt token):
    q [batch, n_q, n_heads, hd] -> f32 [batch, n_q, n_heads, hd]."""
    row_offset = np.ascontiguousarray(row_offset, dtype=np.int64)
    batch = len(row_offset)
    out = np.empty((batch, n_q, n_heads, head_dim), np.float32)
    lib().oracle_attn_prefill_f32(_u16(q).reshape(-1), _u16(k_pool).reshape(-1),
                                  _u16(v_pool).reshape(-1), row_offset, out.reshape(-1), batch,
                                  n_q, start_pos, n_heads, n_kv_heads, head_dim, float(scale))
    return out


def q4_weights(n: int, n_blocks: int, seed: int):
    """Deterministic synthetic q4 weights: packed [N, n_blocks, 4] u32, scales [N, n_blocks]
    f32, zero points [ceil(N*n_blocks/8)] u32 (the MatMulNBits layout)."""
    B = np.empty((n, n_blocks, 4), np.uint32)
    scales = np.empty((n, n_blocks), np.float32)
    zp = np.empty(((n * n_blocks + 7) // 8,), np.uint32)
    lib().oracle_fill_q4(B.reshape(-1), scales.reshape(-1), zp, n, n_blocks, int(seed))
    return B, scales, zp


def q4_gemv(a, B, scales, zp, epilogue: int = 0, y=None) -> np.ndarray:
    """kernels/matmul_nbits_sg.wgsl: Y [N] f32 from A [K] f32 (epilogue 1 = relu2,
    2 = Y += result, the engine's residual add)."""
    n, n_blocks = scales.shape
    a = np.ascontiguousarray(a, dtype=np.float32)
    assert a.size == 32 * n_blocks
    out = np.zeros(n, np.float32) if y is None else np.array(y, dtype=np.float32, copy=True)
    lib().oracle_q4_gemv_f32(a, np.ascontiguousarray(B, np.uint32).reshape(-1),
                             np.ascontiguousarray(scales, np.float32).reshape(-1),
                             np.ascontiguousarray(zp, np.uint32), out, n, n_blocks, int(epilogue))
    return out


def q4_gemv_f64(a, B, scales, zp) -> np.ndarray:
    n, n_blocks = scales.shape
    out = np.empty(n, np.float64)
    lib().oracle_q4_gemv_f64(np.ascontiguousarray(a, dtype=np.float32),
                             np.ascontiguousarray(B, np.uint32).reshape(-1),
                             np.ascontiguousarray(scales, np.float32).reshape(-1),
                             np.ascontiguousarray(zp, np.uint32), out, n, n_blocks)
    return out


def num_threads() -> int:
    return lib().oracle_num_threads()


def set_num_threads(n: int) -> None:
    lib().oracle_set_num_threads(int(n))
