"""K3 causal prefill (tcgen05) against the CPU oracle.

The cases cover MHA and GQA groups of 2, 3, 4 and 7, lone and partial
query tiles, and continuations after a cached prefix.

Oracle: the reference prefills one token per forward call, so row i is the
decode-step loop of attention.cpp:51-85 over positions [0, start+i]
(oracle.prefill_attention).  Bar: |gpu - oracle| <= 2e-3 + 1e-2*|oracle|."""
import math

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

ATOL, RTOL = 2e-3, 1e-2


@pytest.fixture(scope="module")
def hx():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from hxinfer_b200 import kv
    kv.load()
    kv.device_status(clear=True)
    return kv


def run_prefill(hx, oracle, Hq, Hkv, start, n, seed, out_dtype=torch.float16, layers=2, layer=1,
                qkv=None):
    rng = np.random.default_rng(seed)
    total = start + n
    if qkv is None:
        kc = oracle.f16(rng.standard_normal((total, Hkv * 128)))
        vc = oracle.f16(rng.standard_normal((total, Hkv * 128)))
        q = oracle.f16(rng.standard_normal((n, Hq * 128)))
    else:
        q, kc, vc = qkv
    cache = hx.KVCache(layers, Hkv, 128, 3, total + 64)
    seq = 2  # not the first sequence: exercises the block table
    cache.reserve(0, 64)
    cache.reserve(seq, total)
    cache.write(layer, seq, 0, torch.from_numpy(kc).half().cuda(), torch.from_numpy(vc).half().cuda())
    out = cache.prefill(layer, torch.from_numpy(q).half().cuda(), seq, start, Hq,
                        scale=1.0 / math.sqrt(128), out_dtype=out_dtype)
    torch.cuda.synchronize()
    hx.device_status()
    want = oracle.prefill_attention(q, kc, vc, start, Hq, Hkv, 128)
    got = out.float().cpu().numpy()
    err = np.abs(got - want)
    bad = err > ATOL + RTOL * np.abs(want)
    assert not bad.any(), f"{bad.sum()} of {bad.size} outside tolerance, max abs err {err.max():.3e}"


@pytest.mark.parametrize("n", [1, 5, 128, 129, 300])
def test_prefill_small_mha(hx, oracle, n):
    run_prefill(hx, oracle, 4, 4, 0, n, seed=n)


def test_prefill_llama2_shape_1024(hx, oracle):
    """Config 2's prefill: LLaMA-2-7B MHA (32 heads), 1024 tokens (8 heads here
    for oracle time; the kernel is per head)."""
    run_prefill(hx, oracle, 8, 8, 0, 1024, seed=2)


def test_prefill_qwen_gqa(hx, oracle):
    run_prefill(hx, oracle, 28, 4, 0, 200, seed=3)


@pytest.mark.parametrize("start,n", [(2048, 256), (63, 70), (1, 1), (500, 129)])
def test_prefill_continuation(hx, oracle, start, n):
    """Config 5's continuation: new rows after a cached prefix."""
    run_prefill(hx, oracle, 8, 2, start, n, seed=start + n)


def test_prefill_fp32_out(hx, oracle):
    run_prefill(hx, oracle, 4, 2, 10, 140, seed=9, out_dtype=torch.float32)


@pytest.mark.parametrize("Hq,Hkv,start,n", [(32, 8, 0, 700), (16, 8, 40, 300), (12, 4, 0, 260)])
def test_prefill_gqa_groups(hx, oracle, Hq, Hkv, start, n):
    """GQA groups of 4 (LLaMA-3), 2 and 3, one with a cached prefix."""
    run_prefill(hx, oracle, Hq, Hkv, start, n, seed=Hq + n)


@pytest.mark.parametrize("out_dtype", [torch.float16, torch.float32])
def test_prefill_rows_rescale_apart(hx, oracle, out_dtype):
    """Rows of one warp that move their running max at different key tiles.
    Even query rows are +12u and odd rows -12u for a unit vector u; keys are
    small except that every key from position 128 on is +12u.  At the second
    key tile the even rows' max jumps by about 2^18 (they rescale O) and the
    odd rows' does not, so within each warp some rows rescale and others keep
    their max: the O update must stay warp-collective."""
    rng = np.random.default_rng(11)
    Hq = Hkv = 2
    n = 384
    u = rng.standard_normal(128)
    u /= np.linalg.norm(u)
    q = 0.05 * rng.standard_normal((n, Hq, 128))
    q[0::2] += 12 * u
    q[1::2] -= 12 * u
    kc = 0.05 * rng.standard_normal((n, Hkv, 128))
    kc[128:] += 12 * u
    vc = rng.standard_normal((n, Hkv, 128))
    qkv = tuple(oracle.f16(a.reshape(a.shape[0], -1)) for a in (q, kc, vc))
    run_prefill(hx, oracle, Hq, Hkv, 0, n, seed=0, out_dtype=out_dtype, qkv=qkv)


@pytest.mark.parametrize("out_dtype", [torch.float16, torch.float32])
def test_prefill_writes_only_its_rows(hx, oracle, out_dtype):
    """The output tile is written by tensor-map stores clipped at row n: the
    last, partial query tile leaves the caller's rows past n untouched, and
    an output that starts one row into a buffer leaves the row before it."""
    Hq, Hkv, n = 4, 2, 77
    rng = np.random.default_rng(21)
    kc = oracle.f16(rng.standard_normal((n, Hkv * 128)))
    vc = oracle.f16(rng.standard_normal((n, Hkv * 128)))
    q = oracle.f16(rng.standard_normal((n, Hq * 128)))
    cache = hx.KVCache(1, Hkv, 128, 1, n)
    cache.reserve(0, n)
    cache.write(0, 0, 0, torch.from_numpy(kc).half().cuda(), torch.from_numpy(vc).half().cuda())
    buf = torch.full((n + 130, Hq * 128), 7.0, dtype=out_dtype, device="cuda")
    cache.prefill(0, torch.from_numpy(q).half().cuda(), 0, 0, Hq, scale=1.0 / math.sqrt(128),
                  out=buf[1:n + 1])
    torch.cuda.synchronize()
    hx.device_status()
    assert bool((buf[0] == 7.0).all()) and bool((buf[n + 1:] == 7.0).all())
    want = oracle.prefill_attention(q, kc, vc, 0, Hq, Hkv, 128)
    got = buf[1:n + 1].float().cpu().numpy()
    assert np.all(np.abs(got - want) <= ATOL + RTOL * np.abs(want))
