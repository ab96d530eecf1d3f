"""B200-native decode-attention path of the Nemotron WebGPU decode engine.

The compute lives in ``libnwd.so`` (hand-written CUDA for sm_100a behind the
C ABI of ``include/nwd.h``).  This package is the host-side mirror of the
reference's operator interface for that path:

* :mod:`.ops`    — ``kv_append`` / ``attention`` with the WGSL ``Params``
  fields, plus batched, fused and shard-partial variants;
* :mod:`.engine` — the attention-layer slice of ``DecodeEngine`` (caches,
  ``seq``, step, reset);
* :mod:`.mgpu`   — the long-context decode sharded over GPUs.

Import with ``importlib.import_module("nemotron-webgpu-decode_b200")``.
"""
from . import _lib
from ._lib import NwdError, version

__all__ = ["NwdError", "version", "ops", "engine", "build_library"]


def build_library(verbose: bool = False) -> str:
    """Compile libnwd.so in-tree (nvcc, sm_100a)."""
    from . import build as _build
    return _build.build(verbose=verbose)


def __getattr__(name):
    if name in ("ops", "engine", "mgpu"):
        import importlib
        return importlib.import_module(f"{__name__}.{name}")
    raise AttributeError(name)
