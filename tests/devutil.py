"""Host <-> device helpers for the GPU tests (fp16 bit patterns <-> torch)."""
from __future__ import annotations

import numpy as np
import torch


def to_dev(bits: np.ndarray, shape=None, device="cuda") -> torch.Tensor:
    a = np.ascontiguousarray(bits).view(np.float16)
    t = torch.from_numpy(a.copy())
    if shape is not None:
        t = t.reshape(shape)
    return t.to(device)


def bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().contiguous().numpy().view(np.uint16)


def vals(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().float().numpy().astype(np.float64)
