"""Generates tests/golden/golden.npz.

The reference ships no tests or golden vectors for this path, and its WGSL
cannot run on this machine, so these fixtures come from an independent
restatement: plain float64 numpy (not the C oracle) of
kernels/sparse_attn.wgsl (softmax(scale q.K^T) V per query head, kv head =
h / (n_heads / n_kv_heads), scale = 1/sqrt(head_dim)) on inputs drawn from the
deterministic fp16 N(0,1) generator, which is also restated here in numpy.

Contents:
  gen/<seed>_<offset>: 64 generator outputs (uint16 fp16 bits) — pins the
      generator that the C oracle and the CUDA kernel both implement.
  case/<name>/...: shape, seeds, lengths, row offsets, and the float64
      reference output (stored as float32) of one ragged batch.

Inputs are not stored: tests regenerate them from the pinned generator.
Run:  python tests/golden/make_golden.py
"""
from __future__ import annotations

import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "golden.npz")

_U = np.uint64


def splitmix64(x: np.ndarray) -> np.ndarray:
    with np.errstate(over="ignore"):
        x = x + _U(0x9E3779B97F4A7C15)
        x = (x ^ (x >> _U(30))) * _U(0xBF58476D1CE4E5B9)
        x = (x ^ (x >> _U(27))) * _U(0x94D049BB133111EB)
        return x ^ (x >> _U(31))


def normal_f16(n: int, seed: int, offset: int = 0) -> np.ndarray:
    """fp16 bits of elements offset..offset+n-1 of stream `seed` (Irwin-Hall(12))."""
    with np.errstate(over="ignore"):
        base = splitmix64(np.array([seed], dtype=_U))[0]
        i = np.arange(offset, offset + n, dtype=_U)
        b = base + _U(3) * i
        s = np.zeros(n, dtype=np.int64)
        for j in range(3):
            h = splitmix64(b + _U(j))
            for sh in (0, 16, 32, 48):
                s += ((h >> _U(sh)) & _U(0xFFFF)).astype(np.int64)
    x = (s - 393210).astype(np.float32) * np.float32(1.0 / 65536.0)
    return x.astype(np.float16).view(np.uint16)


def attention_f64(q, k_pool, v_pool, row_offset, seq_len, n_heads, n_kv, hd, scale=None):
    """float64 softmax(scale q.K^T) V per (b, h); zeros for empty sequences."""
    scale = 1.0 / np.sqrt(hd) if scale is None else scale
    group = n_heads // n_kv
    qf = q.view(np.float16).astype(np.float64).reshape(len(seq_len), n_heads, hd)
    kf = k_pool.view(np.float16).astype(np.float64).reshape(-1, n_kv, hd)
    vf = v_pool.view(np.float16).astype(np.float64).reshape(-1, n_kv, hd)
    out = np.zeros((len(seq_len), n_heads, hd))
    for b, (off, L) in enumerate(zip(row_offset, seq_len)):
        if L <= 0:
            continue
        for h in range(n_heads):
            kv = h // group
            s = kf[off:off + L, kv, :] @ qf[b, h] * scale
            p = np.exp(s - s.max())
            p /= p.sum()
            out[b, h] = p @ vf[off:off + L, kv, :]
    return out


# name: (n_heads, n_kv, hd, lengths, capacities, seeds(q, k, v))
CASES = {
    # engine shape (engine/config.js:10-12), the last step of the chat-template trace
    "engine_L151": (40, 8, 128, [151], [256], (1, 2, 3)),
    # config 1 as the benchmark states it (group 4), first decode step
    "g4_L25": (32, 8, 128, [25], [256], (11, 12, 13)),
    # single key: O = V row exactly
    "g4_L1": (32, 8, 128, [1], [8], (21, 22, 23)),
    # smallest config-2 length
    "g5_L1024": (40, 8, 128, [1024], [1024], (31, 32, 33)),
    # group 1 (MHA) and group 8
    "g1_L300": (8, 8, 128, [300], [300], (41, 42, 43)),
    "g8_L97": (16, 2, 128, [97], [128], (51, 52, 53)),
    # ragged batch with an empty sequence and tile edges
    "ragged": (32, 8, 128, [0, 1, 63, 64, 65, 600, 257], [4, 8, 64, 70, 66, 700, 300], (61, 62, 63)),
}


def case_inputs(n_heads, n_kv, hd, lengths, caps, seeds):
    B = len(lengths)
    rows = int(sum(caps))
    offs = np.concatenate([[0], np.cumsum(caps)[:-1]]).astype(np.int64)
    q = normal_f16(B * n_heads * hd, seeds[0])
    k = normal_f16(rows * n_kv * hd, seeds[1])
    v = normal_f16(rows * n_kv * hd, seeds[2])
    return q, k, v, offs, np.asarray(lengths, np.int32), rows


def main():
    data = {}
    for seed in (0, 1, 2, 12345):
        for off in (0, 1000003):
            data[f"gen/{seed}_{off}"] = normal_f16(64, seed, off)
    for name, (nh, nkv, hd, lens, caps, seeds) in CASES.items():
        q, k, v, offs, L, rows = case_inputs(nh, nkv, hd, lens, caps, seeds)
        ref = attention_f64(q, k, v, offs, L, nh, nkv, hd)
        data[f"case/{name}/shape"] = np.array([nh, nkv, hd, rows], np.int64)
        data[f"case/{name}/seeds"] = np.array(seeds, np.int64)
        data[f"case/{name}/lengths"] = L
        data[f"case/{name}/row_offset"] = offs
        data[f"case/{name}/out"] = ref.astype(np.float32)
    np.savez_compressed(OUT, **data)
    print(f"wrote {OUT}: {len(data)} arrays")


if __name__ == "__main__":
    main()
