"""Every entry point that launches on a cache, RoPE table or gather endpoint
refuses, before any launch, a call made while another GPU is current: the
cache's TMA tensor maps and block table address its own GPU's memory, and a
kernel on another GPU would read them as peer memory.  Needs two GPUs; every
call here returns HX_ERR_INVALID on the host, so nothing runs on either GPU."""
import ctypes as C

import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu


def test_calls_from_another_device_are_refused():
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs two CUDA devices")
    from hxinfer_b200 import _lib, kv
    lib = _lib.load()
    P = C.c_void_p
    with torch.cuda.device(0):
        cache = kv.KVCache(1, 4, 128, 2, 256)
        cache.reserve(0, 128)
        table = kv.RopeTable(128, 256, 1e6)
        buf = torch.zeros(1 << 20, dtype=torch.uint8, device="cuda:0")
        torch.cuda.synchronize()
    d = P(buf.data_ptr())
    spec = _lib.hx_append_spec(k=d.value, v=d.value, bq=None, bk=None, bv=None,
                               dtype=_lib.HX_FP16, table=table.handle)
    with torch.cuda.device(1):
        s = P(torch.cuda.current_stream().cuda_stream)
        calls = {
            "hx_kv_reserve": lambda: lib.hx_kv_reserve(cache.handle, 1, 64, s),
            "hx_kv_release": lambda: lib.hx_kv_release(cache.handle, 0, s),
            "hx_kv_write": lambda: lib.hx_kv_write(cache.handle, 0, 0, 0, 1, d, d, _lib.HX_FP16, s),
            "hx_kv_read": lambda: lib.hx_kv_read(cache.handle, 0, 0, 0, 1, d, d, s),
            "hx_kv_fill_normal": lambda: lib.hx_kv_fill_normal(cache.handle, 1, s),
            "hx_rope_append": lambda: lib.hx_rope_append(
                cache.handle, 0, d, d, d, _lib.HX_FP16, None, None, None, d, d, 1, 28,
                table.handle, d, _lib.HX_FP16, s),
            "hx_rope_qk": lambda: lib.hx_rope_qk(d, d, _lib.HX_FP16, 1, 28, 4, 128, 3,
                                                 table.handle, s),
            "hx_qkv_rope_append": lambda: lib.hx_qkv_rope_append(
                cache.handle, 0, d, _lib.HX_FP16, 512, d, d, d, _lib.HX_FP16, None, None, None,
                d, d, 1, 28, table.handle, d, _lib.HX_FP16, s),
            "hx_decode_attention": lambda: lib.hx_decode_attention(
                cache.handle, 0, d, _lib.HX_FP16, d, d, 1, 28, 0.1, d, _lib.HX_FP16, d,
                buf.numel(), s),
            "hx_decode_attention_noalloc": lambda: lib.hx_decode_attention_noalloc(
                cache.handle, 0, d, _lib.HX_FP16, d, d, 1, 28, 0.1, d, _lib.HX_FP16, s),
            "hx_append_decode_attention": lambda: lib.hx_append_decode_attention(
                cache.handle, 0, d, C.byref(spec), d, d, 1, 28, 0.1, d, _lib.HX_FP16, d,
                buf.numel(), s),
            "hx_prefill_attention": lambda: lib.hx_prefill_attention(
                cache.handle, 0, d, 0, 0, 16, 28, 0.1, d, _lib.HX_FP16, s),
            "hx_kv_snapshot": lambda: lib.hx_kv_snapshot(cache.handle, 0, 64, d, buf.numel(), s),
            "hx_kv_restore": lambda: lib.hx_kv_restore(cache.handle, 0, 64, d, buf.numel(), s),
        }
        for name, call in calls.items():
            rc = call()
            assert rc == _lib.HX_ERR_INVALID, f"{name} returned {rc}"
            assert b"device" in lib.hx_last_error(), f"{name}: {lib.hx_last_error()!r}"
    with torch.cuda.device(0):
        torch.cuda.synchronize()
        kv.device_status()
        cache.close()
        table.close()
