"""The CPU oracle against the reference: its known-answer tests, the golden
vectors the reference produced (tests/golden/make_golden.py), and, where the
reference library is built (oracle/_ref), fresh seeded inputs."""
import numpy as np
import pytest


def bits(a):
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


# --------------------------------------------------------------- reference KATs

def test_rope_kat_identity_at_pos0(oracle):
    # tests/unit/test_unit_ops.cpp:197-217: at pos 0 RoPE is the identity
    x = np.array([[1.0, 2.0, 3.0, 4.0]], np.float32)
    y = oracle.rope(x, 1, 4, 0, 10000.0)
    assert np.allclose(y, x, atol=1e-5)


def test_rope_kat_pos1(oracle):
    # tests/unit/test_unit_ops.cpp:219-228: Q[0]' = -1.9841, Q[2]' = 2.4624 (tol 1e-3)
    x = np.array([[1.0, 2.0, 3.0, 4.0]], np.float32)
    y = oracle.rope(x, 1, 4, 1, 10000.0)[0]
    assert abs(y[0] - (-1.9841)) < 1e-3
    assert abs(y[2] - 2.4624) < 1e-3


def test_attention_kat_single_position(oracle):
    # tests/unit/test_unit_ops.cpp:292-319: one position -> softmax = 1 -> out = V
    out = oracle.decode_attention(np.array([1.0, 0.0], np.float32),
                                  np.array([[1.0, 0.0]], np.float32),
                                  np.array([[5.0, 10.0]], np.float32), 1, 1, 2)
    assert abs(out[0] - 5.0) < 1e-3 and abs(out[1] - 10.0) < 1e-3


# --------------------------------------------------------------- golden vectors

def test_rope_golden(oracle, golden):
    kat = golden["rope_kat_in"]
    for step in (0, 1):
        assert np.array_equal(bits(oracle.rope(kat, 1, 4, step, 10000.0)),
                              bits(golden[f"rope_kat_q_step{step}"]))
    for name in ("qwen", "llama"):
        hq, hkv, step, theta = golden[f"rope_{name}_meta"]
        q = oracle.rope(golden[f"rope_{name}_q_in"], int(hq), 128, int(step), float(theta))
        k = oracle.rope(golden[f"rope_{name}_k_in"], int(hkv), 128, int(step), float(theta))
        assert np.array_equal(bits(q), bits(golden[f"rope_{name}_q_out"]))
        assert np.array_equal(bits(k), bits(golden[f"rope_{name}_k_out"]))


def test_softmax_golden(oracle, golden):
    assert np.array_equal(bits(oracle.softmax(golden["softmax_in"])), bits(golden["softmax_out"]))


def test_attention_layer_golden(oracle, golden):
    """The oracle's RoPE + append + attention loop reproduces the reference
    AttentionLayer CPU branch bit for bit (exact signed-permutation projections)."""
    head, hd, npos, theta = golden["attn_meta"]
    head, hd, npos = int(head), int(hd), int(npos)
    wq, wk, wv, wo = golden["attn_w"]
    x = golden["attn_x"]
    dim = head * hd
    K = np.zeros((npos, dim), np.float32)
    V = np.zeros((npos, dim), np.float32)
    outs = []
    for p in range(npos):
        q = oracle.rope((wq @ x[p])[None].astype(np.float32), head, hd, p, float(theta))[0]
        K[p] = oracle.rope((wk @ x[p])[None].astype(np.float32), head, hd, p, float(theta))[0]
        V[p] = (wv @ x[p]).astype(np.float32)
        a = oracle.decode_attention(q, K[:p + 1], V[:p + 1], head, head, hd)
        outs.append((wo @ a).astype(np.float32))
    assert np.array_equal(bits(np.stack(outs)), bits(golden["attn_out"]))


def test_hash_golden(oracle, golden):
    toks, lens, want = golden["hash_tokens"], golden["hash_lens"], golden["hash_out"]
    off = 0
    for n, h in zip(lens, want):
        assert oracle.fnv1a64(toks[off:off + n]) == int(h)
        off += n


def test_prefix_cache_semantics_golden(oracle, golden):
    """PrefixCacheManager (prefix_cache.h:58-151): restore puts back the first
    prefix_len rows of every layer's K and V, leaves later rows alone; a miss
    changes nothing; lookup returns prefix_len on a hit and 0 on a miss."""
    layers, dim, head, seq_len, plen = [int(v) for v in golden["prefix_meta"]]
    init, over = golden["prefix_init_kv"], golden["prefix_over_kv"]
    expect = over.copy()
    expect[:, :, :plen, :] = init[:, :, :plen, :]
    assert np.array_equal(golden["prefix_after_restore"], expect)
    assert np.array_equal(golden["prefix_after_miss"], over)
    assert list(golden["prefix_hits"]) == [plen, 0, 1]
    assert oracle.fnv1a64(golden["prefix_tokens"]) != oracle.fnv1a64(golden["prefix_probe"])


# --------------------------------------------------------------- oracle properties

def test_rope_table_reproduces_rope(oracle):
    """The cos/sin table the kernels rotate with holds exactly rope_cpu's values."""
    rng = np.random.default_rng(5)
    tab = oracle.rope_table(2100, 128, 1e6)
    for step in (0, 1, 63, 64, 1024, 2099):
        x = oracle.f16(rng.standard_normal((1, 4 * 128)))
        want = oracle.rope(x, 4, 128, step, 1e6)
        y = x.reshape(4, 128).copy()
        c, s = tab[step, :, 0], tab[step, :, 1]
        x1, x2 = y[:, :64].copy(), y[:, 64:].copy()
        y[:, :64] = x1 * c - x2 * s
        y[:, 64:] = x2 * c + x1 * s
        assert np.array_equal(bits(y.reshape(1, -1)), bits(want))


def test_yarn_identity_when_factor_one(oracle):
    scale = oracle.yarn_scale(128, 1.0, 1e6, 32.0, 1.0, 4096)
    assert np.all(scale == 1.0)
    assert oracle.yarn_attn_factor(1.0) == 1.0
    rng = np.random.default_rng(6)
    x = oracle.f16(rng.standard_normal((2, 256)))
    assert np.array_equal(bits(oracle.rope_yarn(x, 2, 128, 77, 1e6, scale, 1.0)),
                          bits(oracle.rope(x, 2, 128, 77, 1e6)))


def test_batch_attention_is_thread_count_invariant(oracle):
    rng = np.random.default_rng(7)
    Hq, Hkv, hd = 8, 2, 128
    lens = [1, 5, 64, 130]
    q = oracle.f16(rng.standard_normal((len(lens), Hq * hd)))
    ks = [oracle.f16(rng.standard_normal((L, Hkv * hd))) for L in lens]
    vs = [oracle.f16(rng.standard_normal((L, Hkv * hd))) for L in lens]
    a = oracle.decode_attention_batch(q, ks, vs, Hq, Hkv, hd, nthreads=1)
    b = oracle.decode_attention_batch(q, ks, vs, Hq, Hkv, hd, nthreads=3)
    assert np.array_equal(bits(a), bits(b))
    for i in range(len(lens)):
        assert np.array_equal(bits(a[i]), bits(oracle.decode_attention(q[i], ks[i], vs[i], Hq, Hkv, hd)))


def test_prefill_equals_decode_steps(oracle):
    rng = np.random.default_rng(8)
    Hq, Hkv, hd, n = 4, 2, 128, 9
    q = oracle.f16(rng.standard_normal((n, Hq * hd)))
    k = oracle.f16(rng.standard_normal((n, Hkv * hd)))
    v = oracle.f16(rng.standard_normal((n, Hkv * hd)))
    out = oracle.prefill_attention(q, k, v, 0, Hq, Hkv, hd)
    for i in range(n):
        assert np.array_equal(bits(out[i]), bits(oracle.decode_attention(q[i], k[:i + 1], v[:i + 1], Hq, Hkv, hd)))


# --------------------------------------------------------------- against the built reference

@pytest.fixture(scope="module")
def ref(oracle):
    if not oracle.ref_available():
        pytest.skip("oracle/_ref/libhxref.so not built")
    return oracle


@pytest.mark.parametrize("hq,hkv,step,theta", [(28, 4, 1024, 1e6), (32, 8, 32768, 5e5),
                                                (32, 32, 0, 1e4), (2, 1, 4095, 1e4)])
def test_rope_matches_reference_fresh(ref, hq, hkv, step, theta):
    rng = np.random.default_rng(hq * 1000 + step)
    q = ref.f16(rng.standard_normal((2, hq * 128)))
    k = ref.f16(rng.standard_normal((2, hkv * 128)))
    rq, rk = ref.ref_rope(q, k, hq, hkv, 128, step, theta)
    assert np.array_equal(bits(ref.rope(q, hq, 128, step, theta)), bits(rq))
    assert np.array_equal(bits(ref.rope(k, hkv, 128, step, theta)), bits(rk))


def test_attention_layer_matches_reference_fresh(ref):
    rng = np.random.default_rng(99)
    head, hd, npos, theta = 4, 32, 12, 1e4
    dim = head * hd
    ws = []
    for i in range(4):
        w = np.zeros((dim, dim), np.float32)
        w[np.arange(dim), rng.permutation(dim)] = rng.choice([-1.0, 0.5, 1.0, 2.0], dim)
        ws.append(w)
    x = ref.f16(rng.standard_normal((npos, dim)))
    want = ref.ref_attention_layer(dim, head, theta, *ws, x)
    K = np.zeros((npos, dim), np.float32)
    V = np.zeros((npos, dim), np.float32)
    for p in range(npos):
        q = ref.rope((ws[0] @ x[p])[None].astype(np.float32), head, hd, p, theta)[0]
        K[p] = ref.rope((ws[1] @ x[p])[None].astype(np.float32), head, hd, p, theta)[0]
        V[p] = (ws[2] @ x[p]).astype(np.float32)
        got = (ws[3] @ ref.decode_attention(q, K[:p + 1], V[:p + 1], head, head, hd)).astype(np.float32)
        assert np.array_equal(bits(got), bits(want[p]))


def test_hash_matches_reference_fresh(ref):
    rng = np.random.default_rng(3)
    for n in (0, 1, 7, 300):
        t = rng.integers(-5, 152064, n).astype(np.int32)
        assert ref.fnv1a64(t) == ref.ref_hash(t)


# --------------------------------------------------------------- random inputs against the built reference

from hypothesis import HealthCheck, given, settings  # noqa: E402
from hypothesis import strategies as st  # noqa: E402
from hypothesis.extra.numpy import arrays  # noqa: E402

_SETTINGS = settings(max_examples=60, deadline=None,
                     suppress_health_check=[HealthCheck.function_scoped_fixture])


@_SETTINGS
@given(hkv=st.sampled_from([1, 2, 4, 8]), group=st.sampled_from([1, 2, 4, 7]),
       hd=st.sampled_from([64, 128, 256]), rows=st.integers(1, 3), step=st.integers(0, 131071),
       theta=st.sampled_from([1e4, 5e5, 1e6]) | st.floats(100.0, 1e7, width=32),
       seed=st.integers(0, 2**31 - 1), scale=st.sampled_from([1.0, 1e-3, 300.0]))
def test_rope_matches_reference_on_random_inputs(ref, hkv, group, hd, rows, step, theta, seed, scale):
    """Bit-exact RoPE for random head layouts, positions, bases and magnitudes."""
    hq = hkv * group
    rng = np.random.default_rng(seed)
    q = ref.f16(rng.standard_normal((rows, hq * hd)) * scale)
    k = ref.f16(rng.standard_normal((rows, hkv * hd)) * scale)
    rq, rk = ref.ref_rope(q, k, hq, hkv, hd, step, float(theta))
    assert np.array_equal(bits(ref.rope(q, hq, hd, step, float(theta))), bits(rq))
    assert np.array_equal(bits(ref.rope(k, hkv, hd, step, float(theta))), bits(rk))


@_SETTINGS
@given(x=arrays(np.float32, st.integers(1, 5000),
                elements=st.floats(-80.0, 80.0, width=32, allow_nan=False)))
def test_softmax_matches_reference_on_random_inputs(ref, x):
    """Bit-exact safe softmax (max-subtracted exponentials over their sum)."""
    assert np.array_equal(bits(ref.softmax(x)), bits(ref.ref_softmax(x)))


@_SETTINGS
@given(t=arrays(np.int32, st.integers(0, 2000), elements=st.integers(-2**31, 2**31 - 1)))
def test_hash_matches_reference_on_random_inputs(ref, t):
    assert ref.fnv1a64(t) == ref.ref_hash(t)


@settings(max_examples=25, deadline=None, suppress_health_check=[HealthCheck.function_scoped_fixture])
@given(head=st.integers(1, 6), hd=st.sampled_from([32, 64, 128]), npos=st.integers(1, 24),
       theta=st.sampled_from([1e4, 1e6]), seed=st.integers(0, 2**31 - 1))
def test_attention_layer_matches_reference_on_random_inputs(ref, head, hd, npos, theta, seed):
    """The reference's CPU AttentionLayer (one token per forward) against the
    oracle's RoPE + decode attention, bit-exact, with exact signed-permutation
    projections."""
    rng = np.random.default_rng(seed)
    dim = head * hd
    ws = []
    for _ in range(4):
        w = np.zeros((dim, dim), np.float32)
        w[np.arange(dim), rng.permutation(dim)] = rng.choice([-1.0, 0.5, 1.0, 2.0], dim)
        ws.append(w)
    x = ref.f16(rng.standard_normal((npos, dim)))
    want = ref.ref_attention_layer(dim, head, theta, *ws, x)
    K = np.zeros((npos, dim), np.float32)
    V = np.zeros((npos, dim), np.float32)
    for p in range(npos):
        q = ref.rope((ws[0] @ x[p])[None].astype(np.float32), head, hd, p, theta)[0]
        K[p] = ref.rope((ws[1] @ x[p])[None].astype(np.float32), head, hd, p, theta)[0]
        V[p] = (ws[2] @ x[p]).astype(np.float32)
        got = (ws[3] @ ref.decode_attention(q, K[:p + 1], V[:p + 1], head, head, hd)).astype(np.float32)
        assert np.array_equal(bits(got), bits(want[p])), p
