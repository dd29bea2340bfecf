"""The checkpoint reader on hostile input, under AddressSanitizer and
UndefinedBehaviorSanitizer, without a GPU.

Checkpoint files are untrusted.  tests/cpp/fuzz_reader (the reader's and the
JSON reader's sources built with g++ -fsanitize=address,undefined) loads
generated files and reads every byte of every tensor it accepts; it must
finish with no sanitizer report, whatever the bytes.  Inputs: headers built
from random JSON values in the safetensors shape (random dtypes, shapes,
offsets, metadata), valid files with flipped, truncated or appended bytes,
random header lengths, and random JSON lines."""
import json
import os
import random
import struct
import subprocess
import sys

import pytest
from hypothesis import HealthCheck, given, settings
from hypothesis import strategies as st

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
sys.path.insert(0, HERE)

from safetensors_files import write_raw, write_safetensors  # noqa: E402

FUZZ_BIN = os.path.join(HERE, "cpp", "fuzz_reader")
ENV = dict(os.environ, ASAN_OPTIONS="detect_leaks=0:abort_on_error=0:halt_on_error=1",
           UBSAN_OPTIONS="halt_on_error=1:print_stacktrace=1")


@pytest.fixture(scope="module")
def fuzz_bin():
    from hxinfer_b200 import build
    build.build()
    r = subprocess.run(["make", "-s", "-C", os.path.join(HERE, "cpp"), "fuzz_reader"],
                       capture_output=True, text=True)
    if r.returncode != 0:
        pytest.skip("sanitizer build unavailable: " + r.stderr[-300:])
    return FUZZ_BIN


def run_fuzz(*args):
    r = subprocess.run([FUZZ_BIN, *map(str, args)], capture_output=True, text=True, env=ENV,
                       timeout=600)
    report = r.stderr
    assert "AddressSanitizer" not in report and "runtime error" not in report, report[-4000:]
    assert r.returncode == 0, report[-4000:]
    return r.stdout


_INTS = st.integers(-5, 70) | st.integers(-2**63, 2**64) | st.sampled_from([0, 1, 2**31, 2**32 - 1])
_DTYPES = st.sampled_from(["F32", "F16", "BF16", "I8", "U8", "I32", "I64", "F64", "BOOL", "F8_E4M3",
                           "X9", ""]) | st.integers(0, 9) | st.none()
_ENTRY = st.fixed_dictionaries(
    {}, optional={"dtype": _DTYPES,
                  "shape": st.lists(_INTS, max_size=4) | st.integers() | st.text(max_size=3),
                  "data_offsets": st.lists(_INTS, max_size=3) | st.none() | st.floats(allow_nan=False)})
_HEADER = st.dictionaries(st.text(max_size=6), _ENTRY | st.integers() | st.lists(st.integers(), max_size=2),
                          max_size=5)


@settings(max_examples=3, deadline=None, suppress_health_check=[HealthCheck.function_scoped_fixture])
@given(headers=st.lists(st.tuples(_HEADER, st.integers(0, 300), st.integers(-8, 8)), min_size=150,
                        max_size=150))
def test_reader_survives_random_headers(fuzz_bin, tmp_path, headers):
    paths = []
    for i, (h, data_len, len_skew) in enumerate(headers):
        text = json.dumps(h).encode()
        p = tmp_path / f"h{i}.safetensors"
        write_raw(str(p), text, os.urandom(data_len), header_len=max(0, len(text) + len_skew))
        paths.append(str(p))
    out = run_fuzz("files", *paths)
    assert out.startswith("files loaded")


def _valid_file(path, rng):
    tensors = []
    for j in range(rng.randint(1, 4)):
        dtype = rng.choice(["F32", "F16", "BF16", "I8"])
        shape = [rng.randint(0, 5) for _ in range(rng.randint(0, 3))]
        n = 1
        for d in shape:
            n *= d
        size = {"F32": 4, "F16": 2, "BF16": 2, "I8": 1}[dtype] * n
        tensors.append((f"t{j}", dtype, shape, os.urandom(size)))
    write_safetensors(path, tensors, metadata={"format": "pt"})


def test_reader_survives_mutated_files(fuzz_bin, tmp_path):
    rng = random.Random(20261202)
    paths = []
    for i in range(400):
        p = str(tmp_path / f"m{i}.safetensors")
        _valid_file(p, rng)
        data = bytearray(open(p, "rb").read())
        kind = i % 5
        if kind == 0:  # flip bytes anywhere in the header length and header
            for _ in range(rng.randint(1, 6)):
                k = rng.randrange(min(len(data), 8 + 200))
                data[k] = rng.randrange(256)
        elif kind == 1:  # truncate
            data = data[:rng.randrange(len(data) + 1)]
        elif kind == 2:  # random header length
            data[:8] = struct.pack("<Q", rng.choice([0, 1, 7, len(data), 2**63, 2**64 - 1,
                                                     rng.randrange(2 * len(data) + 1)]))
        elif kind == 3:  # append garbage after the data
            data += os.urandom(rng.randint(1, 64))
        else:  # random bytes of a random length
            data = bytearray(os.urandom(rng.randint(0, 64)))
        open(p, "wb").write(bytes(data))
        paths.append(p)
    out = run_fuzz("files", *paths)
    assert out.startswith("files loaded")


def test_json_reader_survives_random_lines(fuzz_bin, tmp_path):
    rng = random.Random(7)
    alphabet = b'{}[]",:0123456789-+.eEtrufalsn \\/u\x00\x01\xff\xc3\xa4'
    lines = [bytes(rng.choice(alphabet) for _ in range(rng.randint(0, 80))).replace(b"\n", b" ")
             for _ in range(3000)]
    lines += [b"[" * 200, b"{" * 200, b'"\\ud800\\udc00"', b'"' + b"\\" * 99 + b'"']
    p = tmp_path / "lines.jsonl"
    p.write_bytes(b"\n".join(lines) + b"\n")
    out = run_fuzz("json", str(p))
    assert out.startswith("json ok")
