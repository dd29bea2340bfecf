"""The drop-in recipe checked against the reference's own sources, without a GPU.

A maintainer replaces the reference's hot-path headers with this build's, at
the same paths (the reference's layer headers include their siblings by
relative name, so the files themselves must be replaced; an include path
placed first would not shadow them), removes the reference's hot-path
sources, compiles this build's n-row TransformerLayer / SwigluLayer /
CausalLMModel (hxinfer_b200/cpp/engine) in their place, and links the rest
of the engine against libhxinfer.so and libhxkv.so.  This test does exactly that in a scratch directory: every
remaining engine source and the reference's DenseModelLoader
(model_loaders/src/dense_model_loader.cpp, over this build's
SafetensorsMultiReader) are compiled with nvcc and linked into one shared
object with --no-undefined.  Skipped where the reference sources are absent.
"""
import glob
import os
import shutil
import subprocess
import sysconfig
from concurrent.futures import ThreadPoolExecutor

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "hxinfer_b200")
# the reference checkout: HXINFER_REFERENCE, else `reference` beside this repository
REFERENCE = os.environ.get("HXINFER_REFERENCE") or os.path.join(os.path.dirname(ROOT), "reference")
NVCC = "/usr/local/cuda/bin/nvcc"

# this build's header -> the reference header it replaces (same relative path)
REPLACED_HEADERS = ["base/allocator.h", "base/buffer.h", "base/config.h", "tensor/tensor.h",
                    "op/math_ops.h", "layer/layer.h", "layer/attention.h", "cache/prefix_cache.h",
                    "layer/swiglu.h", "layer/transformer.h", "model/causal_lm_model.h"]
REPLACED_LOADER_HEADERS = ["safetensors_loader.h"]
# reference sources whose functions libhxinfer.so provides
REMOVED_SOURCES = ["op/cpu/rope_cpu.cpp", "op/rope_tensor.cpp", "op/cuda/rope_cuda.cu",
                   "op/cuda/attention_score_cuda.cu", "op/cuda/bias_add.cu", "layer/attention.cpp",
                   "base/allocator_cpu.cpp", "base/allocator_cuda.cu", "base/buffer.cpp",
                   "tensor/tensor.cpp", "layer/swiglu.cpp", "layer/transformer.cpp",
                   "model/causal_lm_model.cpp"]
# this build's n-row replacements for the last three, compiled with the engine
ENGINE_SOURCES = sorted(glob.glob(os.path.join(PKG, "cpp", "engine", "*", "*.cpp")))
REMOVED_LOADER_SOURCES = ["safetensors_loader.cpp"]


def nlohmann_include():
    """A directory holding nlohmann/json.hpp (the reference loader's JSON
    library), or None."""
    for base in {sysconfig.get_paths()["purelib"], sysconfig.get_paths()["platlib"]}:
        hits = glob.glob(os.path.join(base, "**", "nlohmann", "json.hpp"), recursive=True)
        if hits:
            return os.path.dirname(os.path.dirname(hits[0]))
    return None


@pytest.mark.skipif(not os.path.isdir(os.path.join(REFERENCE, "hxinfer-engine")),
                    reason="reference sources not present")
@pytest.mark.skipif(not os.path.exists(NVCC), reason="nvcc not present")
def test_reference_engine_builds_and_links_over_this_build(tmp_path):
    from hxinfer_b200 import build
    build.build_cpp()
    inc, ml, obj = tmp_path / "include", tmp_path / "loader_include", tmp_path / "obj"
    shutil.copytree(os.path.join(REFERENCE, "hxinfer-engine", "include"), inc)
    shutil.copytree(os.path.join(REFERENCE, "model_loaders", "include"), ml)
    for h in REPLACED_HEADERS:
        assert os.path.exists(inc / h), h  # replaces an existing reference header
        shutil.copy(os.path.join(PKG, "cpp", "include", h), inc / h)
    for h in REPLACED_LOADER_HEADERS:
        assert os.path.exists(ml / h), h
        shutil.copy(os.path.join(PKG, "cpp", "include", "model_loaders", h), ml / h)
    obj.mkdir()

    src_root = os.path.join(REFERENCE, "hxinfer-engine", "src")
    sources = sorted(os.path.relpath(p, src_root) for p in
                     glob.glob(os.path.join(src_root, "**", "*.cpp"), recursive=True) +
                     glob.glob(os.path.join(src_root, "**", "*.cu"), recursive=True))
    for r in REMOVED_SOURCES:
        assert r in sources, r
    jobs = [(os.path.join(src_root, s), []) for s in sources if s not in REMOVED_SOURCES]
    assert len(ENGINE_SOURCES) == 3, ENGINE_SOURCES
    jobs += [(s, []) for s in ENGINE_SOURCES]
    json_inc = nlohmann_include()
    loader_root = os.path.join(REFERENCE, "model_loaders", "src")
    if json_inc:
        for s in sorted(os.listdir(loader_root)):
            if s.endswith(".cpp") and s not in REMOVED_LOADER_SOURCES:
                jobs.append((os.path.join(loader_root, s), [f"-I{json_inc}"]))

    def compile_one(job):
        src, extra = job
        base = ROOT if src.startswith(PKG) else REFERENCE
        out = obj / (os.path.relpath(src, base).replace(os.sep, "_") + ".o")
        cmd = [NVCC, "-std=c++17", "-O1", "-Xcompiler", "-fPIC", "-x", "cu",
               "-gencode", "arch=compute_100a,code=sm_100a", f"-I{inc}", f"-I{ml}",
               f"-I{os.path.join(ROOT, 'include')}", *extra, "-c", src, "-o", str(out)]
        r = subprocess.run(cmd, capture_output=True, text=True)
        return src, str(out), r.returncode, r.stderr[-2000:]

    with ThreadPoolExecutor(max_workers=os.cpu_count() or 4) as ex:
        results = list(ex.map(compile_one, jobs))
    failed = [(s, err) for s, _, rc, err in results if rc != 0]
    assert not failed, failed[:3]

    lib = tmp_path / "libengine_over_b200.so"
    cmd = [NVCC, "-shared", "-gencode", "arch=compute_100a,code=sm_100a", "-o", str(lib),
           *[o for _, o, _, _ in results], f"-L{PKG}", "-lhxinfer", "-lhxkv",
           "-L/usr/local/cuda/lib64", "-lcudart", "-lcublas", "-Xlinker", "--no-undefined"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr[-3000:]
    if not json_inc:
        pytest.skip("engine linked; nlohmann/json not found, DenseModelLoader not compiled")
