"""Weight loading on the GPU.

hx_convert (the device-side checkpoint dtype conversion) is checked against
the oracle's restatement of the reference's CPU loops
(model_loaders/src/safetensors_loader.cpp:12-27, 124-197), itself pinned to
CUDA's host __float2half / __half2float by tests/golden/convert_golden.npz.
SafetensorsReader::get_tensor_gpu and AttentionLoader::load_layers
run end to end through tests/cpp/test_loader.  Bar: bit-exact, NaN outputs
compared as NaN (not by payload).  Collected after the other GPU tests, so
that a stop at the first failure has already run them.
"""
import json
import os
import sys

import numpy as np
import pytest

torch = pytest.importorskip("torch")

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
sys.path.insert(0, os.path.join(HERE, "golden"))

import make_convert_golden as G  # noqa: E402
from safetensors_files import build_loader_bin, random_tensor, run_loader, write_safetensors  # noqa: E402

pytestmark = pytest.mark.gpu

GOLDEN = np.load(os.path.join(HERE, "golden", "convert_golden.npz"))
TARGET = {"fp16": "FP16", "fp32": "FP32", "int8": "Int8"}
NP_OUT = {"fp16": np.float16, "fp32": np.float32, "int8": np.int8}


@pytest.fixture(scope="module")
def hx():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from hxinfer_b200 import kv
    kv.load()
    kv.device_status(clear=True)
    return kv


@pytest.fixture(scope="module")
def loader_bin():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return build_loader_bin()


def host_bits(oracle, t: torch.Tensor) -> np.ndarray:
    return oracle.canonical_nan_bits(t.cpu().numpy())


def every_bf16() -> torch.Tensor:
    return torch.from_numpy(np.arange(1 << 16, dtype=np.uint16).view(np.int16).copy()).view(torch.bfloat16)


def every_fp16() -> torch.Tensor:
    return torch.from_numpy(np.arange(1 << 16, dtype=np.uint16).view(np.int16).copy()).view(torch.float16)


def want_bits(oracle, raw: np.ndarray, src: str, dst: str) -> np.ndarray:
    return oracle.canonical_nan_bits(oracle.convert(raw.view(np.uint8), src, dst))


# ---------------------------------------------------------------- hx_convert

def test_bf16_to_fp16_every_bit_pattern(hx, oracle):
    src = every_bf16().cuda()
    want = want_bits(oracle, np.arange(1 << 16, dtype=np.uint16), "BF16", "FP16")
    dst = torch.empty(1 << 16, dtype=torch.float16, device="cuda")
    hx.convert(dst, src)
    assert np.array_equal(host_bits(oracle, dst), want)
    buf = src.clone()  # in place: the FP16 result over the BF16 input
    hx.convert(buf.view(torch.float16), buf)
    assert np.array_equal(host_bits(oracle, buf.view(torch.float16)), want)
    hx.device_status(clear=True)


def test_widening_every_bit_pattern(hx, oracle):
    every = np.arange(1 << 16, dtype=np.uint16)
    for src, name in ((every_bf16().cuda(), "BF16"), (every_fp16().cuda(), "F16")):
        dst = torch.empty(1 << 16, dtype=torch.float32, device="cuda")
        hx.convert(dst, src)
        assert np.array_equal(host_bits(oracle, dst), want_bits(oracle, every, name, "FP32")), name


def test_fp32_to_fp16_edges_and_random(hx, oracle):
    for bits in (GOLDEN["f32_edge_in"], G.random_f32_bits(11, 1 << 20)):
        src = torch.from_numpy(bits.view(np.int32).copy()).view(torch.float32).cuda()
        dst = torch.empty(bits.size, dtype=torch.float16, device="cuda")
        hx.convert(dst, src)
        assert np.array_equal(host_bits(oracle, dst), want_bits(oracle, bits, "F32", "FP16"))
    edge = torch.from_numpy(GOLDEN["f32_edge_in"].view(np.int32).copy()).view(torch.float32).cuda()
    dst = torch.empty(edge.numel(), dtype=torch.float16, device="cuda")
    hx.convert(dst, edge)
    assert np.array_equal(host_bits(oracle, dst), GOLDEN["f32_edge_out"])  # the golden itself


@pytest.mark.parametrize("n,src_off,dst_off", [
    (65533, 1, 3),        # 2-byte aligned only: element path throughout
    (8 * 5000 + 5, 0, 0),  # 16-byte aligned: 8-element groups plus a 5-element tail
    (7, 0, 0),            # shorter than one group
    (50_000_003, 0, 0),   # many grid-stride rounds
])
def test_alignment_tails_and_size(hx, oracle, n, src_off, dst_off):
    rng = np.random.default_rng(n)
    bits = rng.integers(0, 1 << 16, n + 16, dtype=np.uint32).astype(np.uint16)
    src_all = torch.from_numpy(bits.view(np.int16)).view(torch.bfloat16).cuda()
    dst_all = torch.empty(n + 16, dtype=torch.float16, device="cuda")
    src, dst = src_all[src_off:src_off + n], dst_all[dst_off:dst_off + n]
    hx.convert(dst, src)
    assert np.array_equal(host_bits(oracle, dst), want_bits(oracle, bits[src_off:src_off + n], "BF16", "FP16"))
    f32_all = torch.empty(n + 16, dtype=torch.float32, device="cuda")
    f32 = f32_all[dst_off:dst_off + n]
    hx.convert(f32, src)
    assert np.array_equal(host_bits(oracle, f32), want_bits(oracle, bits[src_off:src_off + n], "BF16", "FP32"))


def test_same_dtype_copy_and_refusals(hx):
    from hxinfer_b200 import _lib
    lib = _lib.load()
    s = torch.cuda.current_stream().cuda_stream
    a = torch.randn(1000, device="cuda").half()
    b = torch.empty_like(a)
    hx.convert(b, a)
    assert torch.equal(a, b)
    p = a.data_ptr()
    assert lib.hx_convert(p, _lib.HX_FP16, p + 2, _lib.HX_FP16, 100, s) == _lib.HX_ERR_INVALID  # overlap
    assert lib.hx_convert(p, _lib.HX_FP16, p, _lib.HX_FP32, 100, s) == _lib.HX_ERR_INVALID  # in place, 4 -> 2 bytes
    assert lib.hx_convert(p, _lib.HX_BF16, b.data_ptr(), _lib.HX_FP16, 10, s) == _lib.HX_ERR_INVALID  # BF16 target
    assert lib.hx_convert(p, _lib.HX_FP16, b.data_ptr(), 99, 10, s) == _lib.HX_ERR_INVALID
    assert lib.hx_convert(p + 1, _lib.HX_FP16, b.data_ptr(), _lib.HX_BF16, 10, s) == _lib.HX_ERR_INVALID
    assert lib.hx_convert(None, _lib.HX_FP16, None, _lib.HX_BF16, 0, s) == _lib.HX_OK  # nothing to do
    assert lib.hx_convert(None, _lib.HX_FP16, b.data_ptr(), _lib.HX_BF16, 10, s) == _lib.HX_ERR_INVALID
    hx.device_status(clear=True)


# ---------------------------------------------------------------- SafetensorsReader::get_tensor_gpu

def fetch(path, out_dir, requests):
    lines = run_loader("fetch", path, out_dir, *[f"{n}:{d}" for n, d in requests])
    return {int(ln.split()[1]): ln.split()[2:] for ln in lines if ln.startswith("r ")}


def test_get_tensor_gpu_matches_the_oracle(loader_bin, oracle, tmp_path):
    rng = np.random.default_rng(7)
    spec = [("big.bf16", "BF16", (8388613,)),  # two 16 MB staging chunks and a 5-element tail
            ("big.f32", "F32", (4194307,)),    # two chunks, converted out of a device temporary
            ("w.f16", "F16", (37, 29)), ("w.i8", "I8", (33,)), ("empty", "BF16", (0, 8)),
            ("scalar", "F32", ()), ("odd.bf16", "BF16", (3,))]
    tensors = [(n, d, s, random_tensor(rng, d, s)) for n, d, s in spec]
    path = str(tmp_path / "w.safetensors")
    write_safetensors(path, tensors)
    ok = [("big.bf16", "fp16"), ("big.bf16", "fp32"), ("big.f32", "fp16"), ("big.f32", "fp32"),
          ("w.f16", "fp16"), ("w.f16", "fp32"), ("w.i8", "int8"), ("empty", "fp16"),
          ("scalar", "fp16"), ("odd.bf16", "fp16")]
    refused = [("w.f16", "int8"), ("w.i8", "fp16"), ("no.such.tensor", "fp16")]
    res = fetch(path, str(tmp_path), ok + refused)
    raw = {n: (d, np.frombuffer(r, np.uint8)) for n, d, _, r in tensors}
    for i, (name, dt) in enumerate(ok):
        src, data = raw[name]
        want = oracle.convert(data, src, TARGET[dt])
        assert res[i] == ["ok", str(want.nbytes), "1"], (name, dt, res[i])
        got = np.fromfile(str(tmp_path / f"{i}.bin"), dtype=NP_OUT[dt])
        if dt == "int8":
            assert np.array_equal(got, want), name
        else:
            assert np.array_equal(oracle.canonical_nan_bits(got), oracle.canonical_nan_bits(want)), (name, dt)
    for j in range(len(refused)):
        assert res[len(ok) + j] == ["null"], refused[j]


def test_multi_reader_takes_the_first_shard(loader_bin, oracle, tmp_path):
    rng = np.random.default_rng(8)
    d = tmp_path / "shards"
    d.mkdir()
    first = random_tensor(rng, "BF16", (64,))
    write_safetensors(str(d / "model-00001-of-00002.safetensors"), [("shared", "BF16", (64,), first)])
    write_safetensors(str(d / "model-00002-of-00002.safetensors"),
                      [("shared", "BF16", (64,), random_tensor(rng, "BF16", (64,))),
                       ("only2", "F32", (10,), random_tensor(rng, "F32", (10,)))])
    res = fetch(str(d), str(tmp_path), [("shared", "fp16"), ("only2", "fp32"), ("missing", "fp16")])
    assert res[0][0] == "ok" and res[1][0] == "ok" and res[2] == ["null"]
    got = np.fromfile(str(tmp_path / "0.bin"), dtype=np.float16)
    want = oracle.convert(np.frombuffer(first, np.uint8), "BF16", "FP16")
    assert np.array_equal(oracle.canonical_nan_bits(got), oracle.canonical_nan_bits(want))


# ---------------------------------------------------------------- AttentionLoader::load_layers

def bf16_bytes(x: np.ndarray) -> bytes:
    """fp32 -> BF16 bits, round to nearest even (finite inputs)."""
    b = x.astype(np.float32).view(np.uint32).astype(np.uint64)
    return ((b + 0x7FFF + ((b >> 16) & 1)) >> 16).astype(np.uint16).tobytes()


def make_model(oracle, model_dir, ref_dir, *, layers, hq, hkv, bias, seed):
    """A small dense checkpoint in two shards (BF16, as Qwen2 / LLaMA ship)
    plus the weights it should load to -- FP16 weights and FP32 biases, the
    ModelConfig defaults -- converted by the oracle, for the reference layers."""
    rng = np.random.default_rng(seed)
    hd = 128
    dim, kv = hq * hd, hkv * hd
    (model_dir / "config.json").write_text(json.dumps({
        "hidden_size": dim, "intermediate_size": 2 * dim, "num_hidden_layers": layers,
        "num_attention_heads": hq, "num_key_value_heads": hkv, "vocab_size": 1000,
        "rope_theta": 1000000.0, "rope_scaling": None}))
    names = [("q_proj.weight", "wq", (dim, dim)), ("k_proj.weight", "wk", (kv, dim)),
             ("v_proj.weight", "wv", (kv, dim)), ("o_proj.weight", "wo", (dim, dim))]
    if bias:
        names += [("q_proj.bias", "bq", (dim,)), ("k_proj.bias", "bk", (kv,)), ("v_proj.bias", "bv", (kv,))]
    shards = [[], []]
    shards[0].append(("model.embed_tokens.weight", "BF16", (1000, dim),
                      bf16_bytes(rng.standard_normal((1000, dim)))))  # not attention: never read
    for layer in range(layers):
        for suffix, key, shape in names:
            scale = 0.05 if suffix.endswith("weight") else 0.02
            raw = bf16_bytes(rng.standard_normal(shape) * scale)
            shards[layer % 2].append((f"model.layers.{layer}.self_attn.{suffix}", "BF16", shape, raw))
            target = "FP16" if suffix.endswith("weight") else "FP32"
            oracle.convert(np.frombuffer(raw, np.uint8), "BF16", target).tofile(str(ref_dir / f"{layer}.{key}.bin"))
        shards[layer % 2].append((f"model.layers.{layer}.mlp.gate_proj.weight", "BF16", (4, dim),
                                  bf16_bytes(rng.standard_normal((4, dim)))))
    for i, s in enumerate(shards):
        write_safetensors(str(model_dir / f"model-0000{i + 1}-of-00002.safetensors"), s)


@pytest.mark.parametrize("hq,hkv,bias", [(2, 1, True), (4, 4, False)])
def test_loaded_attention_layers_match_layers_built_from_the_oracle_weights(loader_bin, oracle, tmp_path,
                                                                           hq, hkv, bias):
    model_dir, ref_dir = tmp_path / "model", tmp_path / "ref"
    model_dir.mkdir()
    ref_dir.mkdir()
    make_model(oracle, model_dir, ref_dir, layers=2, hq=hq, hkv=hkv, bias=bias, seed=hq + hkv)
    out = run_loader("layers", str(model_dir), str(ref_dir), 70)
    assert "loaded 2" in out, out
    rows = [ln.split() for ln in out if ln.startswith("layer ")]
    assert len(rows) == 2, out
    for r in rows:
        # layer <l> bias <0|1> mismatches <n> max_abs <x> cuda <ok>
        assert r[3] == str(int(bias)) and r[5] == "0" and r[9] == "ok", r
        assert float(r[7]) > 0.0, r
