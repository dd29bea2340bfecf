"""Checkpoint loading without a GPU: the oracle's dtype conversions pinned to
the golden vectors of CUDA's host __float2half / __half2float (the functions
the reference's SafetensorsReader loops call), and the C++ SafetensorsReader /
SafetensorsMultiReader / AttentionLoader::load_config on headers, shard
directories and config.json files, and its JSON reader against Python's
(tests/cpp/test_loader, CPU subcommands only).  The reference has no tests for its loader; the cases follow its code
(model_loaders/src/safetensors_loader.cpp:36-268,
model_loaders/src/dense_model_loader.cpp:27-52) and the safetensors format."""
import json
import os
import sys

import numpy as np
import pytest
from hypothesis import HealthCheck, given, settings
from hypothesis import strategies as st

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
sys.path.insert(0, ROOT)
sys.path.insert(0, HERE)
sys.path.insert(0, os.path.join(HERE, "golden"))

from oracle import oracle as O  # noqa: E402
import make_convert_golden as G  # noqa: E402
from safetensors_files import (build_loader_bin, fnv1a64, random_tensor, run_loader,  # noqa: E402
                               write_raw, write_safetensors)

GOLDEN = np.load(os.path.join(HERE, "golden", "convert_golden.npz"))


# ---------------------------------------------------------------- oracle pin

def test_oracle_bf16_to_fp16_matches_golden_on_every_bit_pattern():
    every = np.arange(1 << 16, dtype=np.uint16)
    got = O.canonical_nan_bits(O.convert(every.view(np.uint8), "BF16", "FP16"))
    bad = np.nonzero(got != GOLDEN["bf16_to_f16"])[0]
    assert bad.size == 0, [(hex(i), hex(got[i]), hex(GOLDEN["bf16_to_f16"][i])) for i in bad[:8]]


def test_oracle_fp16_to_fp32_matches_golden_on_every_bit_pattern():
    every = np.arange(1 << 16, dtype=np.uint16)
    got = O.canonical_nan_bits(O.convert(every.view(np.uint8), "F16", "FP32"))
    assert G.sha256(got) == str(GOLDEN["f16_to_f32_sha256"])


def test_oracle_fp32_to_fp16_matches_golden_edges_and_random():
    edges = GOLDEN["f32_edge_in"]
    got = O.canonical_nan_bits(O.convert(edges.view(np.uint8), "F32", "FP16"))
    bad = np.nonzero(got != GOLDEN["f32_edge_out"])[0]
    assert bad.size == 0, [(hex(edges[i]), hex(got[i]), hex(GOLDEN["f32_edge_out"][i])) for i in bad]
    rnd = G.random_f32_bits(int(GOLDEN["f32_rand_seed"]), int(GOLDEN["f32_rand_n"]))
    got = O.canonical_nan_bits(O.convert(rnd.view(np.uint8), "F32", "FP16"))
    assert G.sha256(got) == str(GOLDEN["f32_rand_out_sha256"])


def test_oracle_exact_pairs_and_refusals():
    rng = np.random.default_rng(5)
    bits = rng.integers(0, 1 << 16, 1000).astype(np.uint16)
    f32 = O.convert(bits.view(np.uint8), "BF16", "FP32")
    assert np.array_equal(f32.view(np.uint32) >> 16, bits.astype(np.uint32))
    assert np.array_equal(f32.view(np.uint32) & 0xFFFF, np.zeros(1000, np.uint32))
    x = rng.standard_normal(100).astype(np.float32)
    assert np.array_equal(O.convert(x.view(np.uint8), "F32", "FP32"), x)
    i8 = rng.integers(-128, 128, 50).astype(np.int8)
    assert np.array_equal(O.convert(i8.view(np.uint8), "I8", "Int8"), i8)
    for src, dst in [("F16", "Int8"), ("I32", "FP32"), ("I8", "FP16"), ("BF16", "Int8")]:
        with pytest.raises(ValueError):
            O.convert(np.zeros(8, np.uint8), src, dst)


# ---------------------------------------------------------------- C++ reader (no CUDA calls)

@pytest.fixture(scope="module")
def loader_bin():
    return build_loader_bin()


def parse_info(lines):
    out = {"load": lines[0].split()[1], "tensors": {}}
    for ln in lines[1:]:
        f = ln.split(" ")
        if f[0] == "n":
            out["n"] = int(f[1])
        elif f[0] == "t":
            out["tensors"][f[1]] = dict(dtype=f[2], shape=f[3], begin=int(f[4]), end=int(f[5]),
                                        fnv=int(f[6], 16), has=int(f[7]))
        elif f[0] == "absent":
            out["absent"] = int(f[1])
    return out


def test_reader_parses_header_offsets_and_bytes(loader_bin, tmp_path):
    rng = np.random.default_rng(1)
    tensors = [
        ("model.layers.0.self_attn.q_proj.weight", "BF16", (6, 5), None),
        ("w.f32", "F32", (3, 4), None),
        ("w.f16", "F16", (5,), None),
        ("w.i8", "I8", (7,), None),
        ("w.i32", "I32", (2,), None),
        ("empty", "F16", (0, 4), None),
        ("scalar", "F32", (), None),
        ("layer.ä中\U0001F600", "F16", (2,), None),  # non-ASCII name: \u escapes in the JSON
    ]
    tensors = [(n, d, s, random_tensor(rng, d, s)) for n, d, s, _ in tensors]
    path = str(tmp_path / "a.safetensors")
    offs = write_safetensors(path, tensors, metadata={"format": "pt", "note": "q\"uote\\"})
    info = parse_info(run_loader("info", path))
    assert info["load"] == "ok" and info["n"] == len(tensors) and info["absent"] == 1
    for name, dtype, shape, raw in tensors:
        t = info["tensors"][name]
        assert t["dtype"] == dtype and t["has"] == 1
        assert t["shape"] == (",".join(map(str, shape)) or "-")
        assert (t["begin"], t["end"]) == offs[name]
        assert t["fnv"] == fnv1a64(raw)


def test_reader_accepts_padding_empty_header_and_unknown_dtypes(loader_bin, tmp_path):
    p = str(tmp_path / "meta_only.safetensors")
    write_raw(p, b'{"__metadata__": {"format": "pt"}}      ')
    info = parse_info(run_loader("info", p))
    assert info["load"] == "ok" and info["n"] == 0
    p = str(tmp_path / "unknown.safetensors")
    write_raw(p, json.dumps({"x": {"dtype": "X9", "shape": [3], "data_offsets": [0, 5]},
                             "f8": {"dtype": "F8_E4M3", "shape": [2, 2], "data_offsets": [5, 9]}}).encode(),
              bytes(range(9)))
    info = parse_info(run_loader("info", p))
    assert info["load"] == "ok" and info["tensors"]["x"]["dtype"] == "X9"
    assert info["tensors"]["f8"]["end"] - info["tensors"]["f8"]["begin"] == 4


def _hdr(d):
    return json.dumps(d).encode()


MALFORMED = {
    "short_file": lambda p: open(p, "wb").write(b"\x01\x00\x00"),
    "header_len_past_end": lambda p: write_raw(p, b"{}", header_len=1000),
    "header_len_huge": lambda p: write_raw(p, b"{}", header_len=(1 << 64) - 1),
    "truncated_json": lambda p: write_raw(p, b'{"a": {"dtype": "F16", "shape": [1], "data_off'),
    "not_an_object": lambda p: write_raw(p, b"[1, 2, 3]"),
    "trailing_garbage": lambda p: write_raw(p, b"{} x"),
    "missing_offsets": lambda p: write_raw(p, _hdr({"a": {"dtype": "F16", "shape": [1]}}), b"\0\0"),
    "offsets_past_data": lambda p: write_raw(
        p, _hdr({"a": {"dtype": "F16", "shape": [2], "data_offsets": [0, 4]}}), b"\0\0"),
    "begin_after_end": lambda p: write_raw(
        p, _hdr({"a": {"dtype": "F16", "shape": [0], "data_offsets": [2, 0]}}), b"\0\0"),
    "size_mismatch": lambda p: write_raw(
        p, _hdr({"a": {"dtype": "F32", "shape": [3], "data_offsets": [0, 8]}}), bytes(8)),
    "negative_dim": lambda p: write_raw(
        p, _hdr({"a": {"dtype": "F16", "shape": [-1], "data_offsets": [0, 0]}})),
    "fractional_dim": lambda p: write_raw(
        p, _hdr({"a": {"dtype": "F16", "shape": [1.5], "data_offsets": [0, 2]}}), b"\0\0"),
    "dim_over_int_max": lambda p: write_raw(
        p, _hdr({"a": {"dtype": "U8", "shape": [1 << 31], "data_offsets": [0, 1]}}), b"\0"),
    "element_count_overflow": lambda p: write_raw(
        p, _hdr({"a": {"dtype": "F32", "shape": [2**31 - 1] * 3, "data_offsets": [0, 4]}}), bytes(4)),
    "duplicate_name": lambda p: write_raw(
        p, b'{"a": {"dtype": "U8", "shape": [1], "data_offsets": [0, 1]}, '
           b'"a": {"dtype": "U8", "shape": [1], "data_offsets": [0, 1]}}', b"\0"),
    "dtype_not_string": lambda p: write_raw(
        p, _hdr({"a": {"dtype": 7, "shape": [1], "data_offsets": [0, 1]}}), b"\0"),
    "control_char_in_name": lambda p: write_raw(p, b'{"a\x01": {}}'),
    "lone_surrogate": lambda p: write_raw(p, b'{"\\ud800": {}}'),
    "deep_nesting": lambda p: write_raw(p, b"[" * 100 + b"]" * 100),
}


@pytest.mark.parametrize("case", sorted(MALFORMED))
def test_reader_rejects_malformed_files(loader_bin, tmp_path, case):
    p = str(tmp_path / f"{case}.safetensors")
    MALFORMED[case](p)
    assert run_loader("info", p)[0] == "load fail"


def test_reader_rejects_missing_file_and_directory(loader_bin, tmp_path):
    assert run_loader("info", str(tmp_path / "none.safetensors"))[0] == "load fail"
    assert run_loader("info", str(tmp_path))[0] == "load fail"


def test_multi_reader_directory(loader_bin, tmp_path):
    rng = np.random.default_rng(2)
    d = tmp_path / "model"
    d.mkdir()
    t = lambda n: (n, "F16", (4,), random_tensor(rng, "F16", (4,)))  # noqa: E731
    write_safetensors(str(d / "model-00002-of-00002.safetensors"), [t("b"), t("shared")])
    write_safetensors(str(d / "model-00001-of-00002.safetensors"), [t("a"), t("shared")])
    write_safetensors(str(d / ".hidden.safetensors"), [t("hidden")])
    write_raw(str(d / "broken.safetensors"), b"{not json")
    write_safetensors(str(d / "notes.bin"), [t("other")])
    out = run_loader("multi", str(d), "a", "b", "shared", "hidden", "other")
    assert out[0] == "load ok"
    assert out[1] == "n 4"  # per-shard counts summed, as the reference does
    assert [ln for ln in out if ln.startswith("m ")] == ["m a", "m b", "m shared"]
    assert [ln for ln in out if ln.startswith("has ")] == ["has a 1", "has b 1", "has shared 1",
                                                          "has hidden 0", "has other 0"]
    e = tmp_path / "empty"
    e.mkdir()
    assert run_loader("multi", str(e))[:2] == ["load fail", "n 0"]


def _config(tmp_path, name, cfg):
    d = tmp_path / name
    d.mkdir()
    (d / "config.json").write_text(cfg if isinstance(cfg, str) else json.dumps(cfg))
    return str(d)


QWEN_CFG = {"architectures": ["Qwen2ForCausalLM"], "hidden_size": 3584, "intermediate_size": 18944,
            "num_hidden_layers": 28, "num_attention_heads": 28, "num_key_value_heads": 4,
            "vocab_size": 152064, "rope_theta": 1000000.0, "rope_scaling": None,
            "torch_dtype": "bfloat16"}


def test_load_config_reads_the_reference_keys(loader_bin, tmp_path):
    out = run_loader("config", _config(tmp_path, "qwen", QWEN_CFG))
    assert out == ["config dim=3584 hidden_dim=18944 layer=28 head=28 kv_head=4 vocab=152064 "
                   "seq_len=4096 theta=1000000 yarn=0 factor=1 orig=4096 beta_fast=32 beta_slow=1"]
    llama = dict(QWEN_CFG, hidden_size=4096, num_attention_heads=32, rope_theta=500000)
    del llama["num_key_value_heads"], llama["rope_scaling"]
    out = run_loader("config", _config(tmp_path, "llama", llama))
    assert "head=32 kv_head=32" in out[0] and "theta=500000" in out[0]
    yarn = dict(QWEN_CFG, rope_scaling={"type": "yarn", "factor": 4.0,
                                        "original_max_position_embeddings": 32768})
    out = run_loader("config", _config(tmp_path, "yarn", yarn))
    assert "yarn=1 factor=4 orig=32768 beta_fast=32 beta_slow=1" in out[0]
    yarn2 = dict(QWEN_CFG, rope_scaling={"rope_type": "yarn", "factor": 2, "beta_fast": 16,
                                         "beta_slow": 2})
    out = run_loader("config", _config(tmp_path, "yarn2", yarn2))
    assert "yarn=1 factor=2 orig=4096 beta_fast=16 beta_slow=2" in out[0]
    linear = dict(QWEN_CFG, rope_scaling={"type": "linear", "factor": 2.0})
    assert "yarn=0 factor=1" in run_loader("config", _config(tmp_path, "linear", linear))[0]


def test_load_config_errors(loader_bin, tmp_path):
    assert run_loader("config", str(tmp_path / "nowhere"))[0].startswith("error config.json not found")
    bad = dict(QWEN_CFG)
    del bad["hidden_size"]
    assert "hidden_size" in run_loader("config", _config(tmp_path, "nohidden", bad))[0]
    assert run_loader("config", _config(tmp_path, "garbage", "{oops"))[0].startswith("error")



# ---------------------------------------------------------------- the JSON reader

def _json_lines(loader_bin, tmp_path, docs):
    p = tmp_path / "docs.jsonl"
    p.write_bytes(b"\n".join(d.encode() if isinstance(d, str) else d for d in docs) + b"\n")
    out = run_loader("json", str(p))
    assert len(out) == len(docs)
    return out


_JSON_SCALARS = (st.none() | st.booleans() | st.integers(-(2**63), 2**63 - 1) |
                 st.floats(allow_nan=False, allow_infinity=False) |
                 st.text(alphabet=st.characters(blacklist_categories=("Cs",)), max_size=12))
_JSON_VALUES = st.recursive(
    _JSON_SCALARS,
    lambda inner: st.lists(inner, max_size=5) |
    st.dictionaries(st.text(alphabet=st.characters(blacklist_categories=("Cs",)), max_size=8), inner,
                    max_size=5),
    max_leaves=25)


@settings(max_examples=1, deadline=None, suppress_health_check=[HealthCheck.function_scoped_fixture])
@given(st.lists(st.tuples(_JSON_VALUES, st.booleans()), min_size=300, max_size=300))
def test_json_reader_round_trips_random_documents(loader_bin, tmp_path, docs):
    """Random documents (escaped or raw UTF-8) read by json_lite and written
    back canonically load to the same Python values."""
    texts = [json.dumps(v, ensure_ascii=a) for v, a in docs]
    out = _json_lines(loader_bin, tmp_path, texts)
    for (v, _), text, line in zip(docs, texts, out):
        assert line.startswith("ok "), text
        assert json.loads(line[3:]) == v, text


def test_json_reader_rejects_what_rfc8259_rejects(loader_bin, tmp_path):
    invalid = ["{", "[1,]", '{"a":}', "01", "1.", ".5", "-", "+1", "tru", "nul", '"\\x"', '"abc',
               "[1 2]", '{"a" 1}', "{1:2}", "1e", "1e+", "--1", '"\t"', "[]]", "{} {}", "",
               "NaN", "Infinity", "-Infinity", '"\\ud800"', '"\\udc00x"', '"\\u12"', "[" * 70 + "]" * 70]
    out = _json_lines(loader_bin, tmp_path, invalid)
    assert [d for d, line in zip(invalid, out) if line != "error"] == []
    for d in invalid[:21]:  # Python's reader rejects these too
        with pytest.raises(ValueError):
            json.loads(d)


def test_json_reader_keeps_int64_exact(loader_bin, tmp_path):
    docs = ["9223372036854775807", "-9223372036854775808", "[0, -0, 18446744073709551615]",
            '{"data_offsets": [4294967296, 1099511627776]}']
    out = _json_lines(loader_bin, tmp_path, docs)
    assert out[0] == "ok 9223372036854775807" and out[1] == "ok -9223372036854775808"
    assert out[2] == "ok [0,0,1.8446744073709552e+19]"  # past int64: a double
    assert out[3] == 'ok {"data_offsets":[4294967296,1099511627776]}'


def test_json_reader_numbers_at_the_double_range_edges(loader_bin, tmp_path):
    docs = ["5e-324", "1e-310", "-4.9406564584124654e-324", "2.2250738585072014e-308",
            "1.7976931348623157e308", "0.1", "-0.0", "1E+2", "123456789012345678901234"]
    out = _json_lines(loader_bin, tmp_path, docs)
    for d, line in zip(docs, out):
        want = json.loads(d)
        if isinstance(want, int) and not -2**63 <= want < 2**63:
            want = float(want)  # integers past int64 become the nearest double
        assert line.startswith("ok ") and json.loads(line[3:]) == want, (d, line)
    over = _json_lines(loader_bin, tmp_path, ["1e999", "-1e999", "1e-400", "-1e-400"])
    assert over == ["ok inf", "ok -inf", "ok 0", "ok -0"]
