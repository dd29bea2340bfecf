"""YaRN RoPE on the GPU.

* hx_rope_table_create(use_yarn = 1) through hx_rope_append (fused bias +
  RoPE + append) and hx_rope_qk equals the oracle's YaRN restatement
  (orc_rope_neox_yarn: rope_cuda.cu:56-68 with the multipliers of
  rope_cuda.cu:13-30 and the attention factor of :32-35, evaluated with the
  host libm) bit for bit: the table holds exactly the oracle's cos/sin.
* The oracle's YaRN restatement is pinned to the reference's own rope_cuda
  (oracle/_ref, run on this GPU).  The reference evaluates powf/cosf/sinf on
  the device, whose results may differ from the host libm by a few units in
  the last place; the angle step * freq carries that relative error, so the
  bound grows with the position:
      |ref - oracle| <= 1e-5 + 1e-6 * step * max|x|.
  At step 1000 with factor 32 the YaRN rotation differs from plain RoPE by
  far more than that bound, so the check does test the YaRN path.
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

# (q heads, kv heads, theta, YaRN settings)
YARN_CASES = {
    "qwen_factor4": (28, 4, 1e6, dict(factor=4.0, beta_fast=32.0, beta_slow=1.0,
                                      orig_max_pos=32768)),
    "llama3_factor32": (32, 8, 5e5, dict(factor=32.0, beta_fast=32.0, beta_slow=1.0,
                                         orig_max_pos=4096)),
    "llama2_factor8_betas": (32, 32, 1e4, dict(factor=8.0, beta_fast=16.0, beta_slow=2.0,
                                               orig_max_pos=2048)),
}


@pytest.fixture(scope="module")
def hx():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from hxinfer_b200 import kv
    kv.load()
    kv.device_status(clear=True)
    return kv


def _oracle_yarn(oracle, x, heads, hd, step, theta, y):
    scale = oracle.yarn_scale(hd, y["factor"], theta, y["beta_fast"], y["beta_slow"],
                              y["orig_max_pos"])
    return oracle.rope_yarn(x, heads, hd, step, theta, scale, oracle.yarn_attn_factor(y["factor"]))


@pytest.mark.parametrize("name", sorted(YARN_CASES))
def test_rope_append_yarn_bit_exact(hx, oracle, name):
    Hq, Hkv, theta, y = YARN_CASES[name]
    hd = 128
    rng = np.random.default_rng(len(name))
    positions = np.array([0, 1, 7, 63, 1000, 4095, 30000], np.int32)
    n = len(positions)
    q = rng.standard_normal((n, Hq * hd)).astype(np.float32)
    k = rng.standard_normal((n, Hkv * hd)).astype(np.float32)
    v = rng.standard_normal((n, Hkv * hd)).astype(np.float32)
    cache = hx.KVCache(1, Hkv, hd, n, 30001)
    seqs = np.arange(n, dtype=np.int32)
    for s in range(n):
        cache.reserve(s, int(positions[s]) + 1)
    table = hx.RopeTable(hd, 30001, theta, yarn=y)
    q_out = torch.empty((n, Hq * hd), dtype=torch.float32, device="cuda")
    cache.rope_append(0, torch.from_numpy(k).cuda(), torch.from_numpy(v).cuda(),
                      torch.from_numpy(seqs).cuda(), torch.from_numpy(positions).cuda(),
                      q=torch.from_numpy(q).cuda(), num_q_heads=Hq, table=table, q_out=q_out)
    torch.cuda.synchronize()
    hx.device_status()
    got_q = q_out.cpu().numpy()
    for i in range(n):
        step = int(positions[i])
        wq = _oracle_yarn(oracle, q[i][None], Hq, hd, step, theta, y)[0]
        wk = _oracle_yarn(oracle, k[i][None], Hkv, hd, step, theta, y)[0]
        assert np.array_equal(got_q[i].view(np.uint32), wq.view(np.uint32)), f"q at {step}"
        ck, cv = cache.read(0, i, step, 1)
        assert np.array_equal(ck.cpu().numpy().reshape(-1).view(np.int16),
                              wk.astype(np.float16).view(np.int16)), f"K at {step}"
        assert np.array_equal(cv.cpu().numpy().reshape(-1).view(np.int16),
                              v[i].astype(np.float16).view(np.int16)), f"V at {step}"
        # hx_rope_qk with the same table: in-place rotation of one row
        tq, tk = torch.from_numpy(q[i][None].copy()).cuda(), torch.from_numpy(k[i][None].copy()).cuda()
        hx.rope_qk(tq, tk, Hq, Hkv, hd, step, table)
        assert np.array_equal(tq.cpu().numpy()[0].view(np.uint32), wq.view(np.uint32))
        assert np.array_equal(tk.cpu().numpy()[0].view(np.uint32), wk.view(np.uint32))
    cache.close()
    table.close()


@pytest.mark.parametrize("name", sorted(YARN_CASES))
def test_oracle_yarn_pinned_to_reference_rope_cuda(hx, oracle, name):
    if not oracle.ref_available():
        pytest.skip("reference library oracle/_ref/libhxref.so not built")
    Hq, Hkv, theta, y = YARN_CASES[name]
    hd = 128
    rng = np.random.default_rng(100 + len(name))
    for step in (0, 1, 7, 100, 1000, 4095, 30000):
        q = rng.standard_normal(Hq * hd).astype(np.float32)
        k = rng.standard_normal(Hkv * hd).astype(np.float32)
        rq, rk = oracle.ref_rope_cuda(q, k, Hq, Hkv, hd, step, theta, yarn=y)
        oq = _oracle_yarn(oracle, q[None], Hq, hd, step, theta, y)[0]
        ok = _oracle_yarn(oracle, k[None], Hkv, hd, step, theta, y)[0]
        for name_, r, o, x in (("q", rq, oq, q), ("k", rk, ok, k)):
            bound = 1e-5 + 1e-6 * step * np.abs(x).max()
            err = np.abs(r - o).max()
            assert err <= bound, f"{name} {name_} step {step}: max diff {err:.3e} > {bound:.3e}"
        if step == 1000 and y["factor"] >= 8:
            plain = oracle.rope(q[None], Hq, hd, step, theta)[0]
            assert np.abs(plain - oq).max() > 10 * (1e-5 + 1e-6 * step * np.abs(q).max())
