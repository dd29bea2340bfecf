"""AttentionLayer::forward on several tokens per call, on the GPU.

Runs tests/cpp/test_layer_tokens: input/output [n, dim] at positions
pos .. pos+n-1 (the reference takes one token per call,
hxinfer-engine/src/layer/attention.cpp:13-88) against the CPU oracle of that
one-token loop.  Appended K/V rows bit-exact (exact signed-permutation
projections); outputs within 2e-3 + 1e-2 |ref|.  Covers the fused projection
(n <= 8, fp16 weights), cuBLAS GEMMs, tcgen05 prefill (head_dim 128), one decode
call per token (head_dim 64), a capacity that is not a multiple of 64 filled to the
end, shape errors, and PrefixCacheManager with host-resident snapshots (a
CPUAllocator, as the reference's callers pass) over caches filled that way.  Collected after the other GPU tests, so that a stop
at the first failure has already run them.
"""
import os
import subprocess

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_attention_layer_multi_token_forward():
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from hxinfer_b200 import build
    build.build_cpp()
    subprocess.run(["make", "-s", "-C", os.path.join(ROOT, "oracle"), "all"], check=True)
    subprocess.run(["make", "-s", "-C", os.path.join(ROOT, "tests", "cpp"), "test_layer_tokens"], check=True)
    r = subprocess.run([os.path.join(ROOT, "tests", "cpp", "test_layer_tokens")], capture_output=True,
                       text=True, timeout=900)
    print(r.stdout[-4000:])
    assert r.returncode == 0, r.stdout[-4000:] + r.stderr[-2000:]
    assert "failed 0" in r.stdout
