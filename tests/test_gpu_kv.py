"""GPU parity of the KV-cache hot path against the CPU oracle.

Bars (stated where they are checked):
  * RoPE, append, snapshot and restore: bit-exact against the oracle
    (the oracle is pinned to the reference's own CPU ops).
  * Attention: |gpu - oracle| <= 2e-3 + 1e-2 * |oracle| elementwise
    (max-abs 2e-3 / max-rel 1e-2 of the fp32 CPU result).
"""
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


def dev(a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a))
    if dtype is not None:
        t = t.to(dtype)
    return t.cuda()


def h16(rng, shape, scale=1.0):
    return (rng.standard_normal(shape) * scale).astype(np.float16)


def u16(t):
    return t.detach().cpu().contiguous().view(torch.int16).numpy()


def assert_close(got, want, what=""):
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    err = np.abs(got - want)
    bad = err > ATOL + RTOL * np.abs(want)
    assert not bad.any(), (f"{what}: {bad.sum()} of {bad.size} outside tolerance; "
                           f"max abs err {err.max():.3e}")


def make_cache(hx, layers, hkv, max_seqs, cap, hd=128):
    return hx.KVCache(layers, hkv, hd, max_seqs, cap)


# ------------------------------------------------------------------ K1

@pytest.mark.parametrize("in_dtype", [np.float16, np.float32])
@pytest.mark.parametrize("with_bias", [False, True])
def test_rope_append_bit_exact(hx, oracle, in_dtype, with_bias):
    """Qwen2.5-7B shape (28 q / 4 kv heads), theta 1e6: rotated q, rotated K
    and V in the cache equal the oracle (rope_cpu + fp16 rounding) bit for bit."""
    rng = np.random.default_rng(10 + with_bias)
    Hq, Hkv, hd, theta = 28, 4, 128, 1e6
    positions = np.array([0, 1, 63, 64, 127, 1024, 4095], np.int32)
    seqs = np.array([0, 1, 2, 0, 1, 2, 3], np.int32)
    n = len(positions)
    q = h16(rng, (n, Hq * hd)).astype(in_dtype)
    k = h16(rng, (n, Hkv * hd)).astype(in_dtype)
    v = h16(rng, (n, Hkv * hd)).astype(in_dtype)
    bq = h16(rng, Hq * hd, 0.02).astype(in_dtype) if with_bias else None
    bk = h16(rng, Hkv * hd, 0.02).astype(in_dtype) if with_bias else None
    bv = h16(rng, Hkv * hd, 0.02).astype(in_dtype) if with_bias else None
    cache = make_cache(hx, 2, Hkv, 4, 4096)
    for s in range(4):
        cache.reserve(s, 4096)
    table = hx.RopeTable(hd, 4096, theta)
    tdt = torch.float16 if in_dtype == np.float16 else torch.float32
    q_out = torch.empty((n, Hq * hd), dtype=tdt, device="cuda")
    cache.rope_append(1, dev(k), dev(v), dev(seqs), dev(positions), q=dev(q), num_q_heads=Hq,
                      table=table, bq=None if bq is None else dev(bq),
                      bk=None if bk is None else dev(bk), bv=None if bv is None else dev(bv),
                      q_out=q_out)
    torch.cuda.synchronize()
    hx.device_status()

    def biased(x, b):
        if b is None:
            return x.astype(np.float32)
        if in_dtype == np.float16:  # __hadd: correctly rounded fp16 sum
            return (x + b).astype(np.float16).astype(np.float32)
        return (x.astype(np.float32) + b.astype(np.float32)).astype(np.float32)

    for i in range(n):
        wq = oracle.rope(biased(q[i], bq)[None], Hq, hd, int(positions[i]), theta)[0]
        wk = oracle.rope(biased(k[i], bk)[None], Hkv, hd, int(positions[i]), theta)[0]
        wv = biased(v[i], bv)
        gq = q_out[i].cpu().numpy()
        if in_dtype == np.float16:
            assert np.array_equal(gq.view(np.int16), wq.astype(np.float16).view(np.int16))
        else:
            assert np.array_equal(gq.view(np.uint32), wq.view(np.uint32))
        ck, cv = cache.read(1, int(seqs[i]), int(positions[i]), 1)
        assert np.array_equal(u16(ck).reshape(-1), wk.astype(np.float16).view(np.int16))
        assert np.array_equal(u16(cv).reshape(-1), wv.astype(np.float16).view(np.int16))


def test_rope_qk_reference_kat(hx):
    """rope_tensor KAT (tests/unit/test_unit_ops.cpp:197-229) through hx_rope_qk, fp32."""
    table = hx.RopeTable(4, 8, 10000.0)
    for step, want in ((0, [1.0, 2.0, 3.0, 4.0]), (1, [-1.9841, None, 2.4624, None])):
        q = torch.tensor([[1.0, 2.0, 3.0, 4.0]], device="cuda")
        k = q.clone()
        hx.rope_qk(q, k, 1, 1, 4, step, table)
        got = q.cpu().numpy()[0]
        for g, w in zip(got, want):
            if w is not None:
                assert abs(g - w) < (1e-5 if step == 0 else 1e-3)


def test_rope_qk_bit_exact_fp32(hx, oracle):
    rng = np.random.default_rng(12)
    Hq, Hkv, hd = 32, 8, 128
    table = hx.RopeTable(hd, 33000, 5e5)
    for step in (0, 17, 32768):
        q = rng.standard_normal((3, Hq * hd)).astype(np.float32)
        k = rng.standard_normal((3, Hkv * hd)).astype(np.float32)
        tq, tk = dev(q), dev(k)
        hx.rope_qk(tq, tk, Hq, Hkv, hd, step, table)
        assert np.array_equal(tq.cpu().numpy().view(np.uint32),
                              oracle.rope(q, Hq, hd, step, 5e5).view(np.uint32))
        assert np.array_equal(tk.cpu().numpy().view(np.uint32),
                              oracle.rope(k, Hkv, hd, step, 5e5).view(np.uint32))


def test_append_out_of_capacity_is_recorded_not_written(hx):
    cache = make_cache(hx, 1, 2, 2, 128)
    cache.reserve(0, 64)  # only the first block is mapped
    k = torch.ones((1, 256), dtype=torch.float16, device="cuda")
    cache.rope_append(0, k, k, dev(np.array([0], np.int32)), dev(np.array([100], np.int32)))
    torch.cuda.synchronize()
    from hxinfer_b200._lib import HXError, HX_ERR_CAPACITY
    with pytest.raises(HXError) as e:
        hx.device_status(clear=True)
    assert e.value.status == HX_ERR_CAPACITY
    hx.device_status(clear=True)  # cleared


# ------------------------------------------------------------------ K2

def oracle_decode_case(oracle, rng, Hq, Hkv, lengths, theta=1e6, hd=128):
    """Caches of N(0,1) fp16 rows, a new token per sequence rotated at
    position L-1; returns inputs and the oracle outputs."""
    cases = []
    for L in lengths:
        kc = oracle.f16(rng.standard_normal((L, Hkv * hd)))
        vc = oracle.f16(rng.standard_normal((L, Hkv * hd)))
        q = oracle.f16(rng.standard_normal(Hq * hd))
        cases.append((kc, vc, q))
    return cases


def run_decode(hx, oracle, Hq, Hkv, lengths, hd=128, out_dtype=torch.float16, seed=0,
               q_dtype=torch.float16):
    rng = np.random.default_rng(seed)
    cases = oracle_decode_case(oracle, rng, Hq, Hkv, lengths, hd=hd)
    cap = max(lengths)
    cache = make_cache(hx, 2, Hkv, len(lengths) + 1, cap, hd)
    # sequence ids deliberately not equal to the batch index
    seq_ids = np.array([(i + 1) % (len(lengths) + 1) for i in range(len(lengths))], np.int32)
    for i, (kc, vc, q) in enumerate(cases):
        cache.reserve(int(seq_ids[i]), lengths[i])
        cache.write(1, int(seq_ids[i]), 0, dev(kc, torch.float16), dev(vc, torch.float16))
    qs = dev(np.stack([c[2] for c in cases]), q_dtype)
    out = cache.decode(1, qs, dev(seq_ids), dev(np.array(lengths, np.int32)), Hq,
                       scale=1.0 / math.sqrt(hd), out_dtype=out_dtype)
    torch.cuda.synchronize()
    hx.device_status()
    got = out.float().cpu().numpy()
    for i, (kc, vc, q) in enumerate(cases):
        want = oracle.decode_attention(q, kc, vc, Hq, Hkv, hd)
        assert_close(got[i], want, f"seq {i} L={lengths[i]} Hq={Hq} Hkv={Hkv} hd={hd}")


@pytest.mark.parametrize("Hq,Hkv", [(28, 4), (32, 8), (32, 32), (32, 2), (4, 4)])
def test_decode_gqa_groups(hx, oracle, Hq, Hkv):
    run_decode(hx, oracle, Hq, Hkv, [1025], seed=Hq + Hkv)


@pytest.mark.parametrize("lengths", [[1], [2], [63], [64], [65], [127, 128, 129], [1, 5000, 64, 3]])
def test_decode_ragged_lengths(hx, oracle, lengths):
    run_decode(hx, oracle, 28, 4, lengths, seed=sum(lengths))


def test_decode_fp32_in_out(hx, oracle):
    run_decode(hx, oracle, 32, 8, [300, 77], out_dtype=torch.float32, q_dtype=torch.float32, seed=3)


def test_decode_qwen_32k(hx, oracle):
    """Single-layer decode at 32k context: Qwen2.5-7B GQA 28/4, 32,769 positions."""
    run_decode(hx, oracle, 28, 4, [32769], seed=32)


def test_decode_batched_llama3(hx, oracle):
    """LLaMA-3-8B shape, 16 sequences of ragged lengths in [512, 8192]."""
    lengths = list(np.random.default_rng(44).integers(512, 8193, 16))
    run_decode(hx, oracle, 32, 8, [int(x) for x in lengths], seed=44)


def test_decode_repeated_calls_share_workspace(hx, oracle):
    """The split-K pieces of a call meet in the workspace: repeated calls on
    one workspace (no clearing in between) give identical outputs."""
    rng = np.random.default_rng(60)
    Hq, Hkv, lengths = 28, 4, [32769, 1025, 70]
    cache = make_cache(hx, 1, Hkv, 3, 32769)
    for s, L in enumerate(lengths):
        cache.reserve(s, L)
    cache.fill_normal(61)
    q = torch.from_numpy(rng.standard_normal((3, Hq * 128)).astype(np.float16)).cuda()
    sid = torch.arange(3, dtype=torch.int32, device="cuda")
    lens = dev(np.array(lengths, np.int32))
    ws = torch.zeros(cache.workspace_bytes(3, Hq), dtype=torch.uint8, device="cuda")
    outs = [cache.decode(0, q, sid, lens, Hq, workspace=ws).clone() for _ in range(3)]
    torch.cuda.synchronize()
    hx.device_status()
    for o in outs[1:]:
        assert torch.equal(o.view(torch.int16), outs[0].view(torch.int16))
    k, v = cache.read(0, 0, 0, lengths[0])
    want = oracle.decode_attention(q[0].float().cpu().numpy(), k.reshape(lengths[0], -1).float().cpu().numpy(),
                                   v.reshape(lengths[0], -1).float().cpu().numpy(), Hq, Hkv, 128)
    assert_close(outs[0][0].float().cpu().numpy(), want, "32k after repeats")


@pytest.mark.parametrize("out_dtype", [torch.float16, torch.float32])
def test_decode_unaligned_out_matches_aligned(hx, out_dtype):
    """An output pointer that is not 16-byte aligned takes the element-wise
    store path; its rows equal the aligned call's bit for bit."""
    rng = np.random.default_rng(65)
    Hq, Hkv, lengths = 32, 8, [3000, 64, 700]
    cache = make_cache(hx, 1, Hkv, 3, 3000)
    for s, L in enumerate(lengths):
        cache.reserve(s, L)
    cache.fill_normal(66)
    q = torch.from_numpy(rng.standard_normal((3, Hq * 128)).astype(np.float16)).cuda()
    sid = torch.arange(3, dtype=torch.int32, device="cuda")
    lens = dev(np.array(lengths, np.int32))
    aligned = cache.decode(0, q, sid, lens, Hq, out_dtype=out_dtype)
    buf = torch.zeros(3 * Hq * 128 + 1, dtype=out_dtype, device="cuda")
    shifted = buf[1:].view(3, Hq * 128)
    assert shifted.data_ptr() % 16 != 0
    cache.decode(0, q, sid, lens, Hq, out=shifted)
    torch.cuda.synchronize()
    hx.device_status()
    assert torch.equal(shifted.cpu(), aligned.cpu())
    assert buf[0].item() == 0


@pytest.mark.parametrize("wide", [False, True])
def test_decode_cuda_graph_replays(hx, oracle, wide):
    """A captured decode replays correctly many times on one workspace.  The
    wide case (128 (sequence, kv head) segments) merges its split-K pieces
    inside the decode kernel through per-segment counters, which every call
    returns to zero."""
    rng = np.random.default_rng(64)
    if wide:
        Hq, Hkv = 32, 8
        lengths = [int(x) for x in rng.integers(1, 3000, 16)]
    else:
        Hq, Hkv, lengths = 28, 4, [32769, 700]
    n = len(lengths)
    cache = make_cache(hx, 1, Hkv, n, max(lengths) + 1)
    for s, L in enumerate(lengths):
        cache.reserve(s, L)
    cache.fill_normal(65)
    q = torch.from_numpy(rng.standard_normal((n, Hq * 128)).astype(np.float16)).cuda()
    sid = torch.arange(n, dtype=torch.int32, device="cuda")
    lens = dev(np.array(lengths, np.int32))
    ws = torch.zeros(cache.workspace_bytes(n, Hq), dtype=torch.uint8, device="cuda")
    out = torch.empty((n, Hq * 128), dtype=torch.float16, device="cuda")
    cache.decode(0, q, sid, lens, Hq, out=out, workspace=ws)  # eager first
    torch.cuda.synchronize()
    want = out.clone()
    stream = torch.cuda.Stream()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        with torch.cuda.graph(g, stream=stream):
            cache.decode(0, q, sid, lens, Hq, out=out, workspace=ws, stream=stream)
    for _ in range(4):
        out.zero_()
        g.replay()
        torch.cuda.synchronize()
        assert torch.equal(out.view(torch.int16), want.view(torch.int16))
    hx.device_status()
    got = want.float().cpu().numpy()
    for s in (0, n - 1):
        k, v = cache.read(0, s, 0, lengths[s])
        ref = oracle.decode_attention(q[s].float().cpu().numpy(),
                                      k.reshape(lengths[s], -1).float().cpu().numpy(),
                                      v.reshape(lengths[s], -1).float().cpu().numpy(), Hq, Hkv, 128)
        assert_close(got[s], ref, f"seq {s} after graph replays")


def test_decode_folded_workspace_reuse_across_batches(hx, oracle):
    """One workspace serves, in turn, a wide call that merges inside the decode
    kernel (64 sequences x 8 kv heads), a narrow call with the combine kernel
    (4 sequences) and the wide call again: the per-segment counters are back
    at zero after every call, so the third call equals the first bit for bit
    and matches the oracle."""
    rng = np.random.default_rng(70)
    Hq, Hkv = 32, 8
    lengths = [int(x) for x in rng.integers(1, 2500, 64)]
    n = len(lengths)
    cache = make_cache(hx, 1, Hkv, n, max(lengths))
    for s, L in enumerate(lengths):
        cache.reserve(s, L)
    cache.fill_normal(71)
    q = torch.from_numpy(rng.standard_normal((n, Hq * 128)).astype(np.float16)).cuda()
    sid = torch.arange(n, dtype=torch.int32, device="cuda")
    lens = dev(np.array(lengths, np.int32))
    ws = torch.zeros(cache.workspace_bytes(n, Hq), dtype=torch.uint8, device="cuda")
    first = cache.decode(0, q, sid, lens, Hq, workspace=ws)
    narrow = cache.decode(0, q[:4].contiguous(), sid[:4].contiguous(), lens[:4].contiguous(), Hq,
                          workspace=ws)
    again = cache.decode(0, q, sid, lens, Hq, workspace=ws)
    torch.cuda.synchronize()
    hx.device_status()
    assert torch.equal(first.view(torch.int16), again.view(torch.int16))
    assert torch.equal(first[:4].view(torch.int16), narrow.view(torch.int16)) or \
        np.allclose(first[:4].float().cpu().numpy(), narrow.float().cpu().numpy(), atol=ATOL, rtol=RTOL)
    got = again.float().cpu().numpy()
    for s in range(0, n, 9):
        k, v = cache.read(0, s, 0, lengths[s])
        ref = oracle.decode_attention(q[s].float().cpu().numpy(),
                                      k.reshape(lengths[s], -1).float().cpu().numpy(),
                                      v.reshape(lengths[s], -1).float().cpu().numpy(), Hq, Hkv, 128)
        assert_close(got[s], ref, f"seq {s} L={lengths[s]}")


def _decode_steps(hx, overlap, graph, layers=4, steps=3, wide=False):
    """rope_append -> decode over `layers` layers for `steps` steps; returns
    every step's outputs."""
    Hq, Hkv, hd = 28, 4, 128
    lengths = np.array([5000, 130, 64], np.int32)
    if wide:  # 20 sequences x 4 kv heads: the decode kernel merges its own pieces
        lengths = np.random.default_rng(98).integers(1, 5000, 20).astype(np.int32)
    n = len(lengths)
    cache = hx.KVCache(layers, Hkv, hd, n, 5100, overlap=overlap)
    for s_, L in enumerate(lengths):
        cache.reserve(s_, int(L) + steps)
    cache.fill_normal(99)
    table = hx.RopeTable(hd, 5200, 1e6)
    g = torch.Generator(device="cuda")
    g.manual_seed(5)
    q = torch.randn((layers, n, Hq * hd), generator=g, device="cuda").half()
    k = torch.randn((layers, n, Hkv * hd), generator=g, device="cuda").half()
    v = torch.randn((layers, n, Hkv * hd), generator=g, device="cuda").half()
    q_rot = torch.empty_like(q)
    out = torch.empty_like(q)
    sid = torch.arange(n, dtype=torch.int32, device="cuda")
    ws = torch.zeros(cache.workspace_bytes(n, Hq), dtype=torch.uint8, device="cuda")
    pos = torch.from_numpy(lengths).cuda()
    lens = pos + 1
    stream = torch.cuda.Stream()

    def one_step():
        for l in range(layers):
            cache.rope_append(l, k[l], v[l], sid, pos, q=q[l], num_q_heads=Hq, table=table,
                              q_out=q_rot[l], stream=stream)
            cache.decode(l, q_rot[l], sid, lens, Hq, out=out[l], workspace=ws, stream=stream)

    results = []
    with torch.cuda.stream(stream):
        if graph:
            one_step()  # warm-up outside capture
            torch.cuda.synchronize()
            gr = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gr, stream=stream):
                one_step()
        for _ in range(steps):
            if graph:
                gr.replay()
            else:
                one_step()
            torch.cuda.synchronize()
            results.append(out.clone())
            pos += 1
            lens += 1
    hx.device_status()
    return results


@pytest.mark.parametrize("graph", [False, True])
@pytest.mark.parametrize("wide", [False, True])
def test_decode_overlap_launch_matches(hx, graph, wide):
    """HX_KV_OVERLAP_LAUNCH (programmatic dependent launch of the
    append -> decode chain) changes timing only: outputs equal the serialised
    launches bit for bit."""
    a = _decode_steps(hx, overlap=False, graph=graph, wide=wide)
    b = _decode_steps(hx, overlap=True, graph=graph, wide=wide)
    for x, y in zip(a, b):
        assert torch.equal(x.view(torch.int16), y.view(torch.int16))


def test_decode_zero_length_sequence(hx, oracle):
    """A sequence with no positions gets zeros and the status word records it;
    its neighbours are unaffected."""
    rng = np.random.default_rng(62)
    Hq, Hkv = 32, 8
    cache = make_cache(hx, 1, Hkv, 3, 256)
    for s in range(3):
        cache.reserve(s, 256)
    cache.fill_normal(63)
    q = torch.from_numpy(rng.standard_normal((3, Hq * 128)).astype(np.float16)).cuda()
    lens = dev(np.array([100, 0, 200], np.int32))
    out = cache.decode(0, q, torch.arange(3, dtype=torch.int32, device="cuda"), lens, Hq)
    torch.cuda.synchronize()
    from hxinfer_b200._lib import HXError
    with pytest.raises(HXError):
        hx.device_status(clear=True)
    assert torch.count_nonzero(out[1]) == 0
    for s, L in ((0, 100), (2, 200)):
        k, v = cache.read(0, s, 0, L)
        want = oracle.decode_attention(q[s].float().cpu().numpy(), k.reshape(L, -1).float().cpu().numpy(),
                                       v.reshape(L, -1).float().cpu().numpy(), Hq, Hkv, 128)
        assert_close(out[s].float().cpu().numpy(), want, f"seq {s}")


@pytest.mark.parametrize("hd", [64, 2])
def test_decode_generic_head_dim(hx, oracle, hd):
    run_decode(hx, oracle, 4, 2, [1, 70, 200], hd=hd, seed=hd)


def test_fused_decode_step_qwen_c1(hx, oracle):
    """Config 1: Qwen2.5-7B layer, cache of 1024 N(0,1) tokens, one new token
    (q/k/v ~ N(0,1)) rotated at position 1024 (theta 1e6), appended, then
    softmax(QK^T/sqrt(128))V over 1025 positions."""
    rng = np.random.default_rng(1)
    Hq, Hkv, hd, theta, P = 28, 4, 128, 1e6, 1024
    kc = oracle.f16(rng.standard_normal((P, Hkv * hd)))
    vc = oracle.f16(rng.standard_normal((P, Hkv * hd)))
    q = h16(rng, (1, Hq * hd))
    k = h16(rng, (1, Hkv * hd))
    v = h16(rng, (1, Hkv * hd))
    cache = make_cache(hx, 1, Hkv, 1, 2048)
    cache.reserve(0, P + 1)
    cache.write(0, 0, 0, dev(kc, torch.float16), dev(vc, torch.float16))
    table = hx.RopeTable(hd, 2048, theta)
    q_out = torch.empty((1, Hq * hd), dtype=torch.float16, device="cuda")
    sid = dev(np.array([0], np.int32))
    cache.rope_append(0, dev(k), dev(v), sid, dev(np.array([P], np.int32)), q=dev(q),
                      num_q_heads=Hq, table=table, q_out=q_out)
    out = cache.decode(0, q_out, sid, dev(np.array([P + 1], np.int32)), Hq)
    torch.cuda.synchronize()
    hx.device_status()
    qr = oracle.rope(q.astype(np.float32), Hq, hd, P, theta)
    kr = oracle.rope(k.astype(np.float32), Hkv, hd, P, theta)
    K = np.concatenate([kc, oracle.f16(kr)])
    V = np.concatenate([vc, v.astype(np.float32)])
    want = oracle.decode_attention(qr[0], K, V, Hq, Hkv, hd)
    assert_close(out.float().cpu().numpy()[0], want, "config-1 step")


def test_wrapped_cache_reference_kat(hx):
    """attention_score_cuda KAT (tests/unit/test_unit_ops.cpp:292-319) through a
    wrapped caller cache: one head, head_dim 2, pos 0 -> out = V = [5, 10]."""
    kbuf = torch.full((10, 2), float("nan"), dtype=torch.float32, device="cuda")
    vbuf = torch.full((10, 2), float("nan"), dtype=torch.float32, device="cuda")
    cache = hx.KVCache.wrap(kbuf, vbuf, 1, 2, 10)
    sid, pos = dev(np.array([0], np.int32)), dev(np.array([0], np.int32))
    k = torch.tensor([[1.0, 0.0]], device="cuda")
    v = torch.tensor([[5.0, 10.0]], device="cuda")
    cache.rope_append(0, k, v, sid, pos)
    q = torch.tensor([[1.0, 0.0]], device="cuda")
    out = cache.decode(0, q, sid, dev(np.array([1], np.int32)), 1, scale=1 / math.sqrt(2),
                       out_dtype=torch.float32)
    torch.cuda.synchronize()
    hx.device_status()
    r = out.cpu().numpy()[0]
    assert abs(r[0] - 5.0) < 1e-3 and abs(r[1] - 10.0) < 1e-3


def test_wrapped_cache_tma_path(hx, oracle):
    """A wrapped head-major cache whose capacity is not a multiple of 64, read
    through the TMA path, with NaN garbage past the sequence end."""
    rng = np.random.default_rng(21)
    Hq, Hkv, hd, cap, L = 8, 2, 128, 100, 90
    kbuf = torch.full((Hkv * cap * hd,), float("nan"), dtype=torch.float16, device="cuda")
    vbuf = torch.full_like(kbuf, float("nan"))
    cache = hx.KVCache.wrap(kbuf, vbuf, Hkv, hd, cap)
    kc = oracle.f16(rng.standard_normal((L, Hkv * hd)))
    vc = oracle.f16(rng.standard_normal((L, Hkv * hd)))
    cache.write(0, 0, 0, dev(kc, torch.float16), dev(vc, torch.float16))
    q = oracle.f16(rng.standard_normal(Hq * hd))
    out = cache.decode(0, dev(q[None], torch.float16), dev(np.array([0], np.int32)),
                       dev(np.array([L], np.int32)), Hq)
    torch.cuda.synchronize()
    hx.device_status()
    assert_close(out.float().cpu().numpy()[0], oracle.decode_attention(q, kc, vc, Hq, Hkv, hd))


# ------------------------------------------------------------------ K4

def test_snapshot_restore_bit_exact(hx):
    """PrefixCacheManager semantics (prefix_cache.h:58-151) on the device: the
    snapshot holds the first prefix_len positions of every layer's K and V;
    restore puts them back and leaves later positions untouched."""
    layers, Hkv, hd, plen, total = 4, 4, 128, 200, 300
    cache = make_cache(hx, layers, Hkv, 3, 512)
    cache.reserve(0, total)
    cache.reserve(2, total)
    cache.fill_normal(1234)
    before = [cache.read(l, 0, 0, total) for l in range(layers)]
    snap = cache.snapshot(0, plen)
    torch.cuda.synchronize()
    # layout [layer][K|V][kv_head][prefix_len][head_dim]
    s = snap.view(torch.float16).view(layers, 2, Hkv, plen, hd)
    for l in range(layers):
        for kv in range(2):
            want = before[l][kv][:plen].permute(1, 0, 2)
            assert torch.equal(s[l, kv].view(torch.int16), want.contiguous().view(torch.int16))
    # overwrite seq 2 with other values, restore seq 0's prefix into it
    other = [cache.read(l, 2, 0, total) for l in range(layers)]
    cache.restore(2, plen, snap)
    torch.cuda.synchronize()
    hx.device_status()
    for l in range(layers):
        k2, v2 = cache.read(l, 2, 0, total)
        assert torch.equal(k2[:plen].view(torch.int16), before[l][0][:plen].view(torch.int16))
        assert torch.equal(v2[:plen].view(torch.int16), before[l][1][:plen].view(torch.int16))
        assert torch.equal(k2[plen:].view(torch.int16), other[l][0][plen:].view(torch.int16))
        assert torch.equal(v2[plen:].view(torch.int16), other[l][1][plen:].view(torch.int16))


@pytest.mark.parametrize("plen", [1, 64, 65, 2048])
def test_snapshot_restore_qwen_shape(hx, plen):
    """Config-5 shape (28 layers, 4 kv heads): the snapshot equals the cache
    rows it covers, and a restore into another sequence reproduces them."""
    layers, Hkv = 28, 4
    cache = make_cache(hx, layers, Hkv, 2, 2048)
    cache.reserve(0, 2048)
    cache.reserve(1, 2048)
    cache.fill_normal(70 + plen)
    snap = cache.snapshot(0, plen)
    cache.restore(1, plen, snap)
    torch.cuda.synchronize()
    hx.device_status()
    s = snap.view(torch.float16).view(layers, 2, Hkv, plen, 128)
    for l in (0, 13, 27):
        k0, v0 = cache.read(l, 0, 0, plen)
        k1, v1 = cache.read(l, 1, 0, plen)
        assert torch.equal(s[l, 0].permute(1, 0, 2).contiguous().view(torch.int16), k0.view(torch.int16))
        assert torch.equal(s[l, 1].permute(1, 0, 2).contiguous().view(torch.int16), v0.view(torch.int16))
        assert torch.equal(k1.view(torch.int16), k0.view(torch.int16))
        assert torch.equal(v1.view(torch.int16), v0.view(torch.int16))


@pytest.mark.parametrize("layers,plen", [(28, 1), (28, 300), (64, 129), (3, 0)])
def test_snapshot_layers_one_launch(hx, layers, plen):
    """hx_kv_snapshot_layers over one-layer wrapped caches (the per-layer
    caches of the model classes) is byte-identical to the per-cache
    snapshots laid end to end; hx_kv_restore_layers puts the prefix back into
    other caches and leaves their later positions untouched."""
    Hkv, hd, cap = 4, 128, 321
    gen = torch.Generator(device="cuda").manual_seed(layers * 1000 + plen)

    def caches():
        out = []
        for _ in range(layers):
            k = torch.randn(Hkv * cap * hd, device="cuda", generator=gen).half()
            v = torch.randn(Hkv * cap * hd, device="cuda", generator=gen).half()
            out.append(hx.KVCache.wrap(k, v, Hkv, hd, cap))
        return out

    src, dst = caches(), caches()
    snap = hx.snapshot_layers(src, plen)
    per = [c.snapshot(0, plen) for c in src]
    torch.cuda.synchronize()
    nb = src[0].snapshot_bytes(plen)
    if plen:
        assert torch.equal(snap[:layers * nb], torch.cat([p[:nb] for p in per]))
    after = [(c._keep[0].clone(), c._keep[1].clone()) for c in dst]
    hx.restore_layers(dst, plen, snap)
    torch.cuda.synchronize()
    hx.device_status()
    for i in range(layers):
        for kv in range(2):
            got = dst[i]._keep[kv].view(Hkv, cap, hd)
            want = src[i]._keep[kv].view(Hkv, cap, hd)
            old = after[i][kv].view(Hkv, cap, hd)
            assert torch.equal(got[:, :plen], want[:, :plen])
            assert torch.equal(got[:, plen:], old[:, plen:])


def test_snapshot_layers_refuses_mixed_caches(hx):
    from hxinfer_b200._lib import HXError
    k = torch.zeros(4 * 128 * 128, device="cuda", dtype=torch.float16)
    a = hx.KVCache.wrap(k, k.clone(), 4, 128, 128)
    b = hx.KVCache.wrap(k.clone(), k.clone(), 2, 128, 128)
    with pytest.raises(HXError):
        hx.snapshot_layers([a, b], 64)
    many = [hx.KVCache.wrap(k, k.clone(), 4, 128, 128) for _ in range(65)]
    with pytest.raises(HXError):
        hx.snapshot_layers(many, 64)
    pooled = make_cache(hx, 2, 4, 1, 128)
    pooled.reserve(0, 128)
    with pytest.raises(HXError):
        hx.snapshot_layers([pooled], 64)


def test_snapshot_rejects_unreserved_prefix(hx):
    cache = make_cache(hx, 1, 1, 1, 256)
    cache.reserve(0, 64)
    from hxinfer_b200._lib import HXError
    with pytest.raises(HXError):
        cache.snapshot(0, 65)


def test_block_allocator_release_and_reuse(hx):
    cache = make_cache(hx, 1, 2, 2, 256)
    info = cache.info()
    assert info["free_blocks"] == 8
    cache.reserve(0, 256)
    cache.reserve(1, 65)
    assert cache.info()["free_blocks"] == 2
    cache.release(0)
    assert cache.info()["free_blocks"] == 6
    from hxinfer_b200._lib import HXError
    with pytest.raises(HXError):
        cache.reserve(1, 257)


# ------------------------------------------------------------------ K1 + K2 in one launch

@pytest.mark.parametrize("name,Hq,Hkv,lens,dtype,bias,rope", [
    ("qwen_batch1_32k", 28, 4, [32769], torch.float16, True, True),
    ("qwen_block_start", 28, 4, [1025, 65, 64, 1], torch.float16, True, True),
    ("llama3_wide_folded", 32, 8, None, torch.float16, False, True),
    ("group16_fp32", 32, 2, [2000, 33, 129], torch.float32, True, True),
    ("mha_no_rope", 8, 8, [300, 7], torch.float16, False, False),
])
def test_append_decode_equals_append_then_decode(hx, name, Hq, Hkv, lens, dtype, bias, rope):
    """hx_append_decode_attention (bias + RoPE + append + decode in one
    launch) against hx_rope_append at positions lengths - 1 followed by
    hx_decode_attention on a copy of the same cache: the appended cache rows
    and the outputs are equal bit for bit, on two steps in a row."""
    if lens is None:
        lens = [int(x) for x in np.random.default_rng(3).integers(1, 3000, 64)]
    n, hd = len(lens), 128
    cap = max(lens) + 2
    caches = [make_cache(hx, 2, Hkv, n, cap) for _ in range(2)]
    for c in caches:
        for s in range(n):
            c.reserve(s, cap)
        c.fill_normal(99)
    table = hx.RopeTable(hd, cap, 1e6) if rope else None
    g = torch.Generator(device="cuda").manual_seed(len(lens))
    sid = torch.arange(n, dtype=torch.int32, device="cuda")
    for step in range(2):
        lengths = torch.tensor(lens, dtype=torch.int32, device="cuda") + step
        q = torch.randn((n, Hq * hd), generator=g, device="cuda").to(dtype)
        k = torch.randn((n, Hkv * hd), generator=g, device="cuda").to(dtype)
        v = torch.randn((n, Hkv * hd), generator=g, device="cuda").to(dtype)
        bq, bk, bv = ((torch.randn((m * hd,), generator=g, device="cuda") * 0.1).to(dtype)
                      for m in (Hq, Hkv, Hkv)) if bias else (None, None, None)
        q_rot = torch.empty((n, Hq * hd), dtype=torch.float16, device="cuda")
        caches[0].rope_append(1, k, v, sid, lengths - 1, q=q, num_q_heads=Hq, table=table,
                              bq=bq, bk=bk, bv=bv, q_out=q_rot)
        want = caches[0].decode(1, q_rot, sid, lengths, Hq)
        got = caches[1].append_decode(1, q, k, v, sid, lengths, Hq, table=table, bq=bq, bk=bk, bv=bv)
        torch.cuda.synchronize()
        hx.device_status()
        assert torch.equal(got.view(torch.int16), want.view(torch.int16)), f"{name} step {step}"
        for s in range(n):
            p0 = lens[s] + step - 1
            k0, v0 = caches[0].read(1, s, p0, 1)
            k1, v1 = caches[1].read(1, s, p0, 1)
            assert torch.equal(k0.view(torch.int16), k1.view(torch.int16)), f"{name} K row {s}"
            assert torch.equal(v0.view(torch.int16), v1.view(torch.int16)), f"{name} V row {s}"


def test_append_decode_refuses_other_head_sizes(hx):
    from hxinfer_b200._lib import HXError
    cache = make_cache(hx, 1, 2, 1, 128, hd=64)
    cache.reserve(0, 128)
    q = torch.zeros((1, 4 * 64), dtype=torch.float16, device="cuda")
    k = torch.zeros((1, 2 * 64), dtype=torch.float16, device="cuda")
    with pytest.raises(HXError):
        cache.append_decode(0, q, k, k.clone(), torch.zeros(1, dtype=torch.int32, device="cuda"),
                            torch.ones(1, dtype=torch.int32, device="cuda"), 4)


def test_append_decode_under_programmatic_launch(hx):
    """The one-launch step with HX_KV_OVERLAP_LAUNCH (each launch a
    programmatic dependent of the previous one, as the benchmark runs it),
    layer after layer and step after step on one stream, against K1 + K2 on
    a copy: outputs and appended rows equal bit for bit."""
    Hq, Hkv, hd, layers, steps = 32, 8, 128, 3, 3
    lens = [int(x) for x in np.random.default_rng(8).integers(100, 2000, 64)]
    n, cap = len(lens), max(lens) + steps + 1
    caches = [hx.KVCache(layers, Hkv, hd, n, cap, overlap=ov) for ov in (False, True)]
    for c in caches:
        for s in range(n):
            c.reserve(s, cap)
        c.fill_normal(5)
    table = hx.RopeTable(hd, cap, 5e5)
    g = torch.Generator(device="cuda").manual_seed(8)
    sid = torch.arange(n, dtype=torch.int32, device="cuda")
    qkv = [[tuple(torch.randn((n, m * hd), generator=g, device="cuda").half() for m in (Hq, Hkv, Hkv))
            for _ in range(layers)] for _ in range(steps)]
    ws = [torch.zeros(c.workspace_bytes(n, Hq), dtype=torch.uint8, device="cuda") for c in caches]
    q_rot = torch.empty((n, Hq * hd), dtype=torch.float16, device="cuda")
    want, got = [], []
    for st in range(steps):
        lengths = torch.tensor(lens, dtype=torch.int32, device="cuda") + st
        for l in range(layers):
            q, k, v = qkv[st][l]
            caches[0].rope_append(l, k, v, sid, lengths - 1, q=q, num_q_heads=Hq, table=table,
                                  q_out=q_rot)
            want.append(caches[0].decode(l, q_rot, sid, lengths, Hq, workspace=ws[0]))
            got.append(caches[1].append_decode(l, q, k, v, sid, lengths, Hq, table=table,
                                               workspace=ws[1]))
    torch.cuda.synchronize()
    hx.device_status()
    for i, (a, b) in enumerate(zip(want, got)):
        assert torch.equal(a.view(torch.int16), b.view(torch.int16)), f"call {i}"
    for l in range(layers):
        for s in (0, 17, 63):
            p0 = lens[s]
            k0, v0 = caches[0].read(l, s, p0 - 1, steps)
            k1, v1 = caches[1].read(l, s, p0 - 1, steps)
            assert torch.equal(k0.view(torch.int16), k1.view(torch.int16))
            assert torch.equal(v0.view(torch.int16), v1.view(torch.int16))
