"""Generate tests/golden/convert_golden.npz: the checkpoint dtype conversions
of the reference's SafetensorsReader (model_loaders/src/safetensors_loader.cpp:
12-27 bf16_to_fp16, 124-197 the other pairs), computed by the functions those
loops call -- CUDA's host __float2half / __half2float (cuda_fp16.h) -- in
tests/golden/convert_pin.cpp, compiled here with g++.  Run from the repository
root:

    python tests/golden/make_convert_golden.py

Contents (NaN outputs canonicalised to 0x7FFF / 0x7FFFFFFF: compared as NaN,
not by payload):
  bf16_to_f16         uint16[65536]: every BF16 bit pattern -> FP16 bits
  f16_to_f32_sha256   SHA-256 of uint32[65536]: every FP16 bit pattern -> FP32 bits
  f32_edge_in/out     FP32 edge cases (signed zeros, ties to even in the normal
                      and subnormal FP16 ranges, the overflow threshold 65520,
                      infinities, NaNs, FP32 extremes) -> FP16 bits
  f32_rand_seed, f32_rand_n, f32_rand_out_sha256
                      random_f32_bits(seed, n) -> FP16 bits, by SHA-256
"""
import hashlib
import os
import subprocess
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "convert_golden.npz")
CUDA_INCLUDE = "/usr/local/cuda/include"
SEED, N_RAND = 20261202, 1 << 20


def random_f32_bits(seed: int, n: int) -> np.ndarray:
    """Half uniformly random FP32 bit patterns (every exponent, NaNs
    included), half values spread over the FP16 range (|x| up to 2^17, with
    exponents down to 2^-30)."""
    rng = np.random.Generator(np.random.PCG64(seed))
    bits = rng.integers(0, 1 << 32, n // 2, dtype=np.uint64).astype(np.uint32)
    mant = rng.uniform(1.0, 2.0, n - n // 2)
    expo = rng.integers(-30, 18, n - n // 2)
    sign = np.where(rng.integers(0, 2, n - n // 2) == 1, -1.0, 1.0)
    vals = (sign * np.ldexp(mant, expo)).astype(np.float32)
    return np.concatenate([bits, vals.view(np.uint32)])


def f32_edges() -> np.ndarray:
    v = [0.0, -0.0, 1.0, -1.0, 0.5, 65504.0, -65504.0, 65519.99, 65520.0, -65520.0, 65536.0,
         1e30, -1e30, np.inf, -np.inf,
         2.0**-14, 2.0**-14 * (1 - 2.0**-11), 2.0**-24, -2.0**-24, 2.0**-25, 2.0**-25 * 1.0000001,
         3 * 2.0**-25, 5 * 2.0**-25, 2.0**-26, 1e-10, -1e-10,
         1 + 2.0**-11, 1 + 3 * 2.0**-11, 1 + 2.0**-11 + 2.0**-20, 2049.0, 2051.0, -2049.0,
         np.finfo(np.float32).max, -np.finfo(np.float32).max, np.finfo(np.float32).tiny,
         float(np.float32(1.4e-45))]
    bits = np.array(v, dtype=np.float32).view(np.uint32)
    nans = np.array([0x7FC00000, 0xFFC00000, 0x7F800001, 0x7FFFFFFF, 0xFF812345], dtype=np.uint32)
    return np.concatenate([bits, nans])


def canonical(bits: np.ndarray) -> np.ndarray:
    bits = bits.copy()
    if bits.dtype == np.uint16:
        bits[((bits & 0x7C00) == 0x7C00) & ((bits & 0x03FF) != 0)] = 0x7FFF
    else:
        bits[((bits & 0x7F800000) == 0x7F800000) & ((bits & 0x007FFFFF) != 0)] = 0x7FFFFFFF
    return bits


def sha256(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def main() -> int:
    with tempfile.TemporaryDirectory() as tmp:
        exe = os.path.join(tmp, "convert_pin")
        subprocess.run(["g++", "-std=c++17", "-O1", f"-I{CUDA_INCLUDE}",
                        os.path.join(HERE, "convert_pin.cpp"), "-o", exe], check=True)

        def run(mode, x, out_dtype):
            src, dst = os.path.join(tmp, "in.bin"), os.path.join(tmp, "out.bin")
            x.tofile(src)
            subprocess.run([exe, mode, src, dst], check=True)
            return np.fromfile(dst, dtype=out_dtype)

        every16 = np.arange(1 << 16, dtype=np.uint16)
        bf16_to_f16 = canonical(run("bf16_to_f16", every16, np.uint16))
        f16_to_f32 = canonical(run("f16_to_f32", every16, np.uint32))
        edges = f32_edges()
        edge_out = canonical(run("f32_to_f16", edges, np.uint16))
        rand_out = canonical(run("f32_to_f16", random_f32_bits(SEED, N_RAND), np.uint16))
    np.savez_compressed(OUT, bf16_to_f16=bf16_to_f16, f16_to_f32_sha256=sha256(f16_to_f32),
                        f32_edge_in=edges, f32_edge_out=edge_out, f32_rand_seed=SEED,
                        f32_rand_n=N_RAND, f32_rand_out_sha256=sha256(rand_out))
    print(f"wrote {OUT} ({os.path.getsize(OUT)} bytes)")
    return 0


if __name__ == "__main__":
    sys.exit(main())
