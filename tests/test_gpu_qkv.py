"""GPU parity of the fused QKV projection + bias + RoPE + append
(hx_qkv_rope_append) against the unfused chain: the projections computed in
fp32 on the CPU and rounded to the projection dtype (what the reference's
cublasGemmEx with CUBLAS_COMPUTE_32F produces, up to accumulation order),
then hx_rope_append (K1, bit-exact against the oracle).

Bar: the two differ only where the fp32 dot products, summed in a different
order, round to neighbouring fp16 values; elementwise |fused - chain| <=
4e-3 + 4e-3 * |chain| (a few fp16 ulps at the values' ~N(0,1) scale), and at
most 2 % of the elements differ at all.
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

ATOL, RTOL, MAX_DIFF_FRAC = 4e-3, 4e-3, 0.02


@pytest.fixture(scope="module")
def hx():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from hxinfer_b200 import kv
    kv.load()
    kv.device_status(clear=True)
    return kv


def compare(got, want, what):
    got = got.double().cpu().numpy()
    want = want.double().cpu().numpy()
    err = np.abs(got - want)
    bad = err > ATOL + RTOL * np.abs(want)
    assert not bad.any(), f"{what}: {bad.sum()} outside tolerance, max err {err.max():.3e}"
    frac = float((err > 0).mean())
    assert frac <= MAX_DIFF_FRAC, f"{what}: {frac:.3%} of elements differ"


@pytest.mark.parametrize("hidden,hq,hkv,n,x_dtype,proj_dtype,with_bias", [
    (3584, 28, 4, 1, torch.float16, torch.float16, True),    # Qwen2.5-7B decode step
    (3584, 28, 4, 3, torch.float32, torch.float16, True),    # fp32 activations
    (4096, 32, 8, 8, torch.float16, torch.float16, False),   # LLaMA-3-8B, a full token group
    (4096, 32, 8, 11, torch.float16, torch.float32, True),   # two token groups, fp32 projections
    (1024, 8, 8, 2, torch.float16, torch.float16, True),     # MHA
    (3584, 28, 4, 5, torch.float16, torch.float16, True),    # tensor-core kernel, 5 of 8 tokens
    (1000, 8, 4, 6, torch.float16, torch.float16, True),     # hidden not a multiple of 32: CUDA cores
])
def test_fused_projection_matches_the_unfused_chain(hx, hidden, hq, hkv, n, x_dtype, proj_dtype,
                                                    with_bias):
    g = torch.Generator().manual_seed(hidden + n)
    hd = 128
    x = torch.randn((n, hidden), generator=g).to(x_dtype)
    wq = (torch.randn((hq * hd, hidden), generator=g) * 0.02).half()
    wk = (torch.randn((hkv * hd, hidden), generator=g) * 0.02).half()
    wv = (torch.randn((hkv * hd, hidden), generator=g) * 0.02).half()
    bias = [(torch.randn((m * hd,), generator=g) * 0.02).to(proj_dtype) if with_bias else None
            for m in (hq, hkv, hkv)]
    seq_ids = torch.tensor([i % 3 for i in range(n)], dtype=torch.int32)
    positions = torch.tensor([5 + 7 * i for i in range(n)], dtype=torch.int32)
    cap = 128
    table = hx.RopeTable(hd, cap, 1e6)

    # unfused: fp32 projections rounded like the reference's q/k/v tensors, then K1
    xf = x.half().float()  # the reference converts fp32 activations to fp16 first
    proj = [(xf @ w.float().T).to(proj_dtype) for w in (wq, wk, wv)]
    ref_cache = hx.KVCache(1, hkv, hd, 3, cap)
    fused_cache = hx.KVCache(1, hkv, hd, 3, cap)
    for c in (ref_cache, fused_cache):
        for s in range(3):
            c.reserve(s, cap)
    dev = torch.device("cuda")
    sid, pos = seq_ids.to(dev), positions.to(dev)
    b_dev = [b.to(dev) if b is not None else None for b in bias]
    q_ref = torch.empty((n, hq * hd), dtype=torch.float16, device=dev)
    ref_cache.rope_append(0, proj[1].to(dev), proj[2].to(dev), sid, pos, q=proj[0].to(dev),
                          num_q_heads=hq, table=table, q_out=q_ref,
                          bq=b_dev[0], bk=b_dev[1], bv=b_dev[2])
    q_fused = fused_cache.qkv_rope_append(0, x.to(dev), wq.to(dev), wk.to(dev), wv.to(dev), sid, pos,
                                          hq, table=table, bq=b_dev[0], bk=b_dev[1], bv=b_dev[2],
                                          proj_dtype=proj_dtype)
    torch.cuda.synchronize()
    hx.device_status()
    compare(q_fused, q_ref, "q")
    for i in range(n):
        s, p = int(seq_ids[i]), int(positions[i])
        kr, vr = ref_cache.read(0, s, p, 1)
        kf, vf = fused_cache.read(0, s, p, 1)
        compare(kf, kr, f"k token {i}")
        compare(vf, vr, f"v token {i}")
    table.close()
    ref_cache.close()
    fused_cache.close()


def test_fused_projection_rejects_unaligned_weights(hx):
    cache = hx.KVCache(1, 4, 128, 1, 16)
    dev = torch.device("cuda")
    x = torch.zeros((1, 512), dtype=torch.float16, device=dev)
    w = torch.zeros((4 * 128 * 512 + 1,), dtype=torch.float16, device=dev)
    wq = w[1:1 + 4 * 128 * 512].view(4 * 128, 512)  # 2-byte offset
    ids = torch.zeros(1, dtype=torch.int32, device=dev)
    from hxinfer_b200._lib import HX_ERR_INVALID, HXError
    with pytest.raises(HXError) as e:
        cache.qkv_rope_append(0, x, wq, wq, wq, ids, ids, 4)
    assert e.value.status == HX_ERR_INVALID
    cache.close()
