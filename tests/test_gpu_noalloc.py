"""hx_decode_attention_noalloc: decode attention for callers that cannot
allocate device memory (inside an allocator or out-of-memory handler, or a
host that reserved all device memory up front), using the library's fixed
scratch array instead of a caller workspace.

Checked through the C ABI against hx_decode_attention (caller workspace) on
two calls in a row, within the attention tolerance of the other tests
(2e-3 absolute + 1e-2 relative); it also passes run alone."""
import ctypes as C
import math

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

ATOL, RTOL = 2e-3, 1e-2


def test_noalloc_matches_workspace_entry_point():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from hxinfer_b200 import _lib, kv
    lib = _lib.load()
    rng = np.random.default_rng(77)
    Hq, Hkv, hd = 28, 4, 128
    lengths = np.array([1025, 3000, 1, 64], np.int32)
    n = len(lengths)
    cache = kv.KVCache(1, Hkv, hd, n, int(lengths.max()))
    for s, L in enumerate(lengths):
        cache.reserve(s, int(L))
    cache.fill_normal(5)
    q = torch.from_numpy(rng.standard_normal((n, Hq * hd)).astype(np.float16)).cuda()
    sid = torch.arange(n, dtype=torch.int32, device="cuda")
    lens = torch.from_numpy(lengths).cuda()
    scale = 1.0 / math.sqrt(hd)
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)

    ws = torch.zeros(cache.workspace_bytes(n, Hq), dtype=torch.uint8, device="cuda")
    want = torch.empty((n, Hq * hd), dtype=torch.float16, device="cuda")
    _lib.check(lib.hx_decode_attention(cache.handle, 0, C.c_void_p(q.data_ptr()), _lib.HX_FP16,
                                       C.c_void_p(sid.data_ptr()), C.c_void_p(lens.data_ptr()), n,
                                       Hq, scale, C.c_void_p(want.data_ptr()), _lib.HX_FP16,
                                       C.c_void_p(ws.data_ptr()), ws.numel(), stream))
    for call in range(2):
        got = torch.full((n, Hq * hd), float("nan"), dtype=torch.float16, device="cuda")
        _lib.check(lib.hx_decode_attention_noalloc(
            cache.handle, 0, C.c_void_p(q.data_ptr()), _lib.HX_FP16, C.c_void_p(sid.data_ptr()),
            C.c_void_p(lens.data_ptr()), n, Hq, scale, C.c_void_p(got.data_ptr()), _lib.HX_FP16,
            stream), f"noalloc call {call}")
        torch.cuda.synchronize()
        g = got.float().cpu().numpy()
        w = want.float().cpu().numpy()
        assert np.isfinite(g).all(), f"call {call}: non-finite output"
        err = np.abs(g - w)
        assert np.all(err <= ATOL + RTOL * np.abs(w)), f"call {call}: max abs err {err.max():.3e}"
    kv.device_status()


def test_noalloc_rejects_oversized_calls():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from hxinfer_b200 import _lib, kv
    lib = _lib.load()
    n, Hq, Hkv = 2048, 32, 8  # workspace > 4 MiB
    cache = kv.KVCache(1, Hkv, 128, n, 64)
    assert cache.workspace_bytes(n, Hq) > (4 << 20)
    dummy = torch.zeros(16, dtype=torch.int32, device="cuda")
    rc = lib.hx_decode_attention_noalloc(cache.handle, 0, C.c_void_p(dummy.data_ptr()),
                                         _lib.HX_FP16, C.c_void_p(dummy.data_ptr()),
                                         C.c_void_p(dummy.data_ptr()), n, Hq, 0.1,
                                         C.c_void_p(dummy.data_ptr()), _lib.HX_FP16,
                                         C.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == _lib.HX_ERR_CAPACITY
    assert b"no-allocation entry point holds at most" in lib.hx_last_error()
