"""hx_decode_attention_noalloc: decode attention for callers that cannot
allocate device memory.

Some callers cannot call cudaMalloc at the moment they need attention: code
running inside a device-memory allocator or its out-of-memory handler (an
allocation there would recurse or fail), and hosts that reserve all device
memory at start-up and forbid allocations afterwards.  This entry point takes
no workspace; its split-K scratch is a fixed array inside the library, whose
device address is set up when the cache is created.

Checked through the C ABI, for each launch path of the decode (the narrow
split-K kernel with its combine kernel, the wide kernel that merges its own
pieces, the 16-row GQA tile, and the generic kernel of other head sizes):
  * two calls in a row give the same output as hx_decode_attention with a
    caller workspace, bit for bit (the same kernels run on the same
    schedule), and match the CPU oracle within the attention tolerance of
    the other decode tests, 2e-3 absolute + 1e-2 relative;
  * around the second call neither the device's free memory nor torch's
    allocated bytes change.
The file is collected last, so a run that stops at the first failure has
already run every other test; it also passes alone in a fresh process."""
import ctypes as C
import math

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

ATOL, RTOL = 2e-3, 1e-2

# name: (q heads, kv heads, head_dim, lengths)
CASES = {
    "narrow_qwen": (28, 4, 128, [1025, 3000, 1, 64]),
    "wide_folded_llama3": (32, 8, 128,
                           [int(x) for x in np.random.default_rng(5).integers(1, 700, 64)]),
    "group16": (32, 2, 128, [2000, 33]),
    "generic_head_dim_64": (8, 2, 64, [300, 7]),
}


def _ptr(t):
    return C.c_void_p(t.data_ptr())


@pytest.mark.parametrize("name", sorted(CASES))
def test_noalloc_matches_workspace_entry_point_and_oracle(name, oracle):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from hxinfer_b200 import _lib, kv
    lib = _lib.load()
    Hq, Hkv, hd, lengths = CASES[name]
    n = len(lengths)
    rng = np.random.default_rng(77 + n)
    cache = kv.KVCache(1, Hkv, hd, n, max(lengths))
    for s, L in enumerate(lengths):
        cache.reserve(s, L)
    cache.fill_normal(5 + n)
    q = torch.from_numpy(rng.standard_normal((n, Hq * hd)).astype(np.float16)).cuda()
    sid = torch.arange(n, dtype=torch.int32, device="cuda")
    lens = torch.tensor(lengths, dtype=torch.int32, device="cuda")
    scale = 1.0 / math.sqrt(hd)
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)

    ws = torch.zeros(max(cache.workspace_bytes(n, Hq), 16), dtype=torch.uint8, device="cuda")
    want = torch.empty((n, Hq * hd), dtype=torch.float16, device="cuda")
    _lib.check(lib.hx_decode_attention(cache.handle, 0, _ptr(q), _lib.HX_FP16, _ptr(sid),
                                       _ptr(lens), n, Hq, scale, _ptr(want), _lib.HX_FP16,
                                       _ptr(ws), ws.numel(), stream), "hx_decode_attention")
    gots = [torch.full((n, Hq * hd), float("nan"), dtype=torch.float16, device="cuda")
            for _ in range(2)]
    torch.cuda.synchronize()
    mem = []
    for call, got in enumerate(gots):
        if call == 1:
            torch.cuda.synchronize()
            mem.append((torch.cuda.mem_get_info()[0], torch.cuda.memory_allocated()))
        _lib.check(lib.hx_decode_attention_noalloc(cache.handle, 0, _ptr(q), _lib.HX_FP16,
                                                   _ptr(sid), _ptr(lens), n, Hq, scale, _ptr(got),
                                                   _lib.HX_FP16, stream), f"noalloc call {call}")
        torch.cuda.synchronize()
    mem.append((torch.cuda.mem_get_info()[0], torch.cuda.memory_allocated()))
    kv.device_status()
    assert mem[0] == mem[1], f"memory changed around a no-allocation call: {mem}"

    for call, got in enumerate(gots):
        assert torch.equal(got.view(torch.int16), want.view(torch.int16)), \
            f"{name} call {call}: differs from hx_decode_attention"
    g = gots[1].float().cpu().numpy()
    for s, L in enumerate(lengths):
        k, v = cache.read(0, s, 0, L)
        ref = oracle.decode_attention(q[s].float().cpu().numpy(),
                                      k.reshape(L, -1).float().cpu().numpy(),
                                      v.reshape(L, -1).float().cpu().numpy(), Hq, Hkv, hd)
        err = np.abs(g[s] - ref)
        assert np.all(err <= ATOL + RTOL * np.abs(ref)), \
            f"{name} seq {s} (L={L}): max abs err {err.max():.3e} against the oracle"
    cache.close()


def test_noalloc_rejects_oversized_calls():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from hxinfer_b200 import _lib, kv
    lib = _lib.load()
    n, Hq, Hkv = 2048, 32, 8  # workspace > 4 MiB
    cache = kv.KVCache(1, Hkv, 128, n, 64)
    assert cache.workspace_bytes(n, Hq) > (4 << 20)
    dummy = torch.zeros(16, dtype=torch.int32, device="cuda")
    rc = lib.hx_decode_attention_noalloc(cache.handle, 0, _ptr(dummy), _lib.HX_FP16, _ptr(dummy),
                                         _ptr(dummy), n, Hq, 0.1, _ptr(dummy), _lib.HX_FP16,
                                         C.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == _lib.HX_ERR_CAPACITY
    assert b"no-allocation entry point holds at most" in lib.hx_last_error()
    cache.close()
