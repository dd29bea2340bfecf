"""Build libhxkv.so (the sm_100a kernels + C ABI) in-tree with nvcc.

    python -m hxinfer_b200.build          # or hxinfer_b200.build.build()

Each .cu file under csrc/ is compiled for sm_100a only
(-gencode arch=compute_100a,code=sm_100a) with -lineinfo; the CUDA runtime is
linked statically so the library does not depend on which libcudart the
process already has loaded.  Objects are rebuilt when a source or header is
newer than its object.
"""
from __future__ import annotations

import glob
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
OBJ = os.path.join(PKG, "_build")
LIB = os.path.join(PKG, "libhxkv.so")
CPP = os.path.join(PKG, "cpp")
CPPLIB = os.path.join(PKG, "libhxinfer.so")
CUDA_LIB = "/usr/local/cuda/lib64"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-std=c++17", "-O3", "-lineinfo", "--expt-relaxed-constexpr", "-Xcompiler", "-fPIC",
              "-Xcompiler", "-ffp-contract=off", "-Xptxas", "-warn-spills",
              f"-I{os.path.join(ROOT, 'include')}", f"-I{CSRC}"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _newer(src_files, target) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(s) > t for s in src_files)


def build(verbose: bool = False, ptxas_info: bool = False) -> str:
    os.makedirs(OBJ, exist_ok=True)
    headers = glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h")) + \
        glob.glob(os.path.join(ROOT, "include", "*.h"))
    objs = []
    for src in sorted(glob.glob(os.path.join(CSRC, "*.cu"))):
        obj = os.path.join(OBJ, os.path.basename(src) + ".o")
        objs.append(obj)
        if not (_newer([src] + headers, obj) or ptxas_info):
            continue
        cmd = [nvcc()] + ARCH + NVCC_FLAGS + (["-Xptxas", "-v"] if ptxas_info else []) + \
            ["-c", src, "-o", obj]
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0 or verbose or ptxas_info:
            sys.stderr.write(r.stdout + r.stderr)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src}")
    if _newer(objs, LIB):
        cmd = [nvcc()] + ARCH + ["-shared", "-cudart", "static", "-o", LIB] + objs + ["-lpthread"]
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            sys.stderr.write(r.stdout + r.stderr)
            raise RuntimeError("link of libhxkv.so failed")
    return LIB


def build_cpp(verbose: bool = False) -> str:
    """libhxinfer.so: the C++ interface layer (Tensor, allocators, rope_tensor /
    rope_cuda / attention_score_cuda, AttentionLayer, PrefixCacheManager) over
    libhxkv.so; cuBLAS for the attention projections."""
    build(verbose)
    os.makedirs(OBJ, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CPP, "src", "*.cpp")) + glob.glob(os.path.join(CPP, "src", "*.cu")))
    headers = glob.glob(os.path.join(CPP, "include", "*", "*.h")) + \
        glob.glob(os.path.join(CPP, "src", "*.h")) + glob.glob(os.path.join(ROOT, "include", "*.h"))
    inc = [f"-I{os.path.join(CPP, 'include')}", f"-I{os.path.join(CPP, 'src')}",
           f"-I{os.path.join(ROOT, 'include')}"]
    objs = []
    for src in srcs:
        obj = os.path.join(OBJ, "cpp_" + os.path.basename(src) + ".o")
        objs.append(obj)
        if not _newer([src] + headers, obj):
            continue
        cmd = [nvcc()] + ARCH + ["-std=c++17", "-O2", "-lineinfo", "-Xcompiler", "-fPIC"] + inc + \
            ["-x", "cu" if src.endswith(".cu") else "c++", "-c", src, "-o", obj]
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0 or verbose:
            sys.stderr.write(r.stdout + r.stderr)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src}")
    if _newer(objs + [LIB], CPPLIB):
        cmd = [nvcc()] + ARCH + ["-shared", "-cudart", "static", "-o", CPPLIB] + objs + \
            [f"-L{PKG}", "-lhxkv", f"-L{CUDA_LIB}", "-lcublas", "-Xlinker", "-rpath,$ORIGIN",
             "-Xlinker", f"-rpath,{CUDA_LIB}"]
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            sys.stderr.write(r.stdout + r.stderr)
            raise RuntimeError("link of libhxinfer.so failed")
    return CPPLIB


if __name__ == "__main__":
    build(verbose="-v" in sys.argv, ptxas_info="--ptxas" in sys.argv)
    build_cpp(verbose="-v" in sys.argv)
    print(LIB)
    print(CPPLIB)
