"""hxinfer_b200 — B200 (sm_100a) KV-cache hot path for the hxinfer engine.

The compute lives in libhxkv.so (CUDA kernels behind the C ABI of
include/hx_kv.h); this package binds it (``_lib``), wraps it over torch
device tensors (``kv``), mirrors its split-K schedule for host-side checks
(``schedule``) and holds the multi-GPU partitioning (``dist``).
"""
from ._lib import HXError, load  # noqa: F401

__all__ = ["HXError", "load"]
