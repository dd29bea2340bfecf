"""Writers of safetensors checkpoints for the loader tests, plus a runner for
tests/cpp/test_loader.

File format (what the reference's SafetensorsReader::load reads,
model_loaders/src/safetensors_loader.cpp:36-81): an 8-byte little-endian
header length, a JSON header {name: {"dtype", "shape", "data_offsets":
[begin, end]}, "__metadata__": {...}} with offsets relative to the end of the
header, then the data.
"""
from __future__ import annotations

import json
import os
import struct
import subprocess

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LOADER_BIN = os.path.join(ROOT, "tests", "cpp", "test_loader")

NP_DTYPE = {"F32": np.float32, "F16": np.float16, "I8": np.int8, "I32": np.int32, "U8": np.uint8,
            "BF16": np.uint16}


def write_safetensors(path: str, tensors, metadata=None, pad_to: int = 8) -> dict:
    """tensors: list of (name, dtype string, shape, raw bytes).  Returns
    {name: (absolute begin, absolute end)}."""
    header = {}
    if metadata is not None:
        header["__metadata__"] = metadata
    off = 0
    for name, dtype, shape, raw in tensors:
        header[name] = {"dtype": dtype, "shape": list(shape), "data_offsets": [off, off + len(raw)]}
        off += len(raw)
    text = json.dumps(header).encode()
    text += b" " * ((-len(text)) % pad_to)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(text)))
        f.write(text)
        for _, _, _, raw in tensors:
            f.write(raw)
    start = 8 + len(text)
    return {name: (start + header[name]["data_offsets"][0], start + header[name]["data_offsets"][1])
            for name, _, _, _ in tensors}


def write_raw(path: str, header_text: bytes, data: bytes = b"", header_len: int | None = None):
    """A file with an arbitrary header (for malformed cases)."""
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(header_text) if header_len is None else header_len))
        f.write(header_text)
        f.write(data)


def fnv1a64(raw: bytes) -> int:
    h = 1469598103934665603
    for b in raw:
        h ^= b
        h = (h * 1099511628211) & 0xFFFFFFFFFFFFFFFF
    return h


def build_loader_bin():
    """libhxkv.so, libhxinfer.so and tests/cpp/test_loader (nvcc, no GPU needed)."""
    from hxinfer_b200 import build
    build.build_cpp()
    subprocess.run(["make", "-s", "-C", os.path.join(ROOT, "tests", "cpp"), "test_loader"], check=True)
    return LOADER_BIN


def run_loader(*args, timeout=600) -> list[str]:
    r = subprocess.run([LOADER_BIN, *map(str, args)], capture_output=True, text=True, timeout=timeout)
    assert r.returncode == 0, r.stdout + r.stderr
    return r.stdout.splitlines()


def random_tensor(rng, dtype: str, shape) -> bytes:
    n = int(np.prod(shape)) if len(shape) else 1
    if dtype == "BF16":
        return rng.integers(0, 1 << 16, n, dtype=np.uint32).astype(np.uint16).tobytes()
    if dtype in ("F32", "F16"):
        return rng.standard_normal(n).astype(NP_DTYPE[dtype]).tobytes()
    return rng.integers(-100, 100, n).astype(NP_DTYPE[dtype]).tobytes()
