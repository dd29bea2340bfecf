"""The C++ interface layer on the GPU: runs tests/cpp/test_unit_ops, which
repeats the reference's own operator tests (tests/unit/test_unit_ops.cpp:
197-229 RoPE, 292-319 attention) through the kept rope_tensor /
attention_score_cuda, and checks AttentionLayer::forward, GQA attention and
PrefixCacheManager store/lookup/restore against the CPU oracle."""
import os
import subprocess

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_cpp_unit_ops():
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from hxinfer_b200 import build
    build.build_cpp()
    subprocess.run(["make", "-s", "-C", os.path.join(ROOT, "oracle"), "all"], check=True)
    subprocess.run(["make", "-s", "-C", os.path.join(ROOT, "tests", "cpp")], check=True)
    r = subprocess.run([os.path.join(ROOT, "tests", "cpp", "test_unit_ops")], capture_output=True,
                       text=True, timeout=600)
    print(r.stdout[-4000:])
    assert r.returncode == 0, r.stdout[-4000:] + r.stderr[-2000:]
    assert "failed 0" in r.stdout
