"""libhxkv.so loads without a GPU and exports every function include/*.h
declares; host-only entry points behave without touching a device."""
import glob
import os
import re

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    names = set()
    for hdr in glob.glob(os.path.join(ROOT, "include", "*.h")):
        text = open(hdr).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        text = re.sub(r"//[^\n]*", "", text)
        for m in re.finditer(r"\b(hx_[a-z0-9_]+)\s*\(", text):
            names.add(m.group(1))
    return names


def test_library_exports_every_declared_symbol(hxlib):
    names = declared_functions()
    assert len(names) >= 20
    missing = [n for n in sorted(names) if not hasattr(hxlib, n)]
    assert not missing, f"not exported: {missing}"


def test_python_binding_covers_the_header():
    from hxinfer_b200 import _lib
    assert declared_functions() <= set(_lib.SIGNATURES), \
        sorted(declared_functions() - set(_lib.SIGNATURES))


def test_prefix_hash_matches_oracle(hxlib, oracle):
    from hxinfer_b200 import kv
    rng = np.random.default_rng(11)
    for n in (0, 1, 5, 2048):
        toks = rng.integers(-3, 152064, n).astype(np.int32)
        assert kv.prefix_hash(toks.tolist()) == oracle.fnv1a64(toks)


def test_status_strings(hxlib):
    assert hxlib.hx_status_string(0) == b"ok"
    assert hxlib.hx_status_string(2) == b"capacity exceeded"
    assert hxlib.hx_status_string(999) == b"unknown status"


def test_null_arguments_are_rejected_without_a_device(hxlib):
    import ctypes as C
    from hxinfer_b200 import _lib
    out = C.c_void_p()
    assert hxlib.hx_kv_create(None, C.byref(out)) == _lib.HX_ERR_INVALID
    assert b"null config" in hxlib.hx_last_error()
    bad = _lib.hx_kv_config(num_layers=1, num_kv_heads=1, head_dim=127, max_seqs=1,
                            max_tokens_per_seq=8, num_blocks=0)
    assert hxlib.hx_kv_create(C.byref(bad), C.byref(out)) == _lib.HX_ERR_INVALID
    assert hxlib.hx_decode_workspace_bytes(None, 1, 1) == 0
    assert hxlib.hx_snapshot_bytes(None, 4) == 0


def test_gather_endpoint_arguments_are_checked_without_a_device(hxlib):
    """The multi-GPU endpoint validates rank/world/sizes before any CUDA call,
    and the gathering decode refuses an unconnected endpoint."""
    import ctypes as C
    from hxinfer_b200 import _lib
    assert 0 < hxlib.hx_dist_handle_bytes() <= 128
    out = C.c_void_p()
    for rank, world, nbytes in ((0, 0, 64), (0, 9, 64), (2, 2, 64), (-1, 2, 64), (0, 2, 0)):
        assert hxlib.hx_dist_create(rank, world, nbytes, C.byref(out)) == _lib.HX_ERR_INVALID
        assert not out.value
    assert hxlib.hx_dist_create(0, 2, 64, None) == _lib.HX_ERR_INVALID
    assert hxlib.hx_dist_export(None, None) == _lib.HX_ERR_INVALID
    assert hxlib.hx_dist_connect(None, None) == _lib.HX_ERR_INVALID
    assert hxlib.hx_dist_wait(None, 1, None) == _lib.HX_ERR_INVALID
    assert hxlib.hx_dist_destroy(None) == _lib.HX_OK
    assert hxlib.hx_dist_buffer(None) is None
    assert hxlib.hx_decode_attention_gather(None, 0, None, _lib.HX_FP16, None, None, 0, 1, 1.0,
                                            None, 0, None, 1, 0, _lib.HX_FP16, None, 0,
                                            None) == _lib.HX_ERR_INVALID


def test_convert_arguments_are_checked_without_a_device(hxlib):
    """hx_convert refuses bad dtype pairs, null, overlapping and misaligned
    pointers before any CUDA call (the addresses below are never touched)."""
    from hxinfer_b200 import _lib
    FP16, FP32, BF16, BAD = _lib.HX_FP16, _lib.HX_FP32, _lib.HX_BF16, _lib.HX_ERR_INVALID
    a, b = 0x10000, 0x80000
    assert hxlib.hx_convert(None, FP16, None, BF16, 0, None) == _lib.HX_OK  # n = 0: nothing to do
    assert hxlib.hx_convert(a, BF16, b, FP16, 8, None) == BAD            # BF16 is a source format only
    assert hxlib.hx_convert(a, FP16, b, 2, 8, None) == BAD               # Int8 is not converted
    assert hxlib.hx_convert(None, FP16, b, BF16, 8, None) == BAD
    assert hxlib.hx_convert(a, FP16, None, BF16, 8, None) == BAD
    assert hxlib.hx_convert(a, FP16, a + 4, FP16, 8, None) == BAD        # overlapping copy
    assert hxlib.hx_convert(a, FP16, a + 8, FP32, 8, None) == BAD        # overlapping narrowing
    assert hxlib.hx_convert(a, FP16, a, FP32, 8, None) == BAD            # in place needs equal sizes
    assert hxlib.hx_convert(a + 1, FP16, b, BF16, 8, None) == BAD        # dst not 2-byte aligned
    assert hxlib.hx_convert(a + 2, FP32, b, FP16, 8, None) == BAD        # FP32 dst not 4-byte aligned
    assert b"aligned" in hxlib.hx_last_error()


def test_header_is_c99_and_links_from_c(tmp_path):
    """The boundary is a C ABI: include/hx_kv.h compiles as strict C99, and a
    C program that takes the address of every declared function links
    against libhxkv.so (unmangled names, matching declarations)."""
    import shutil
    import subprocess
    gcc = shutil.which("gcc")
    if not gcc:
        import pytest
        pytest.skip("gcc not present")
    inc, pkg = os.path.join(ROOT, "include"), os.path.join(ROOT, "hxinfer_b200")
    names = sorted(declared_functions())
    src = tmp_path / "uses_every_entry_point.c"
    src.write_text("#include <stddef.h>\n#include <stdint.h>\n#include \"hx_kv.h\"\n"
                   "void* const entry_points[] = {\n" +
                   "".join(f"    (void*){n},\n" for n in names) + "};\n"
                   "int main(void) { return entry_points[0] == NULL; }\n")
    r = subprocess.run([gcc, "-std=c99", "-Wall", "-Wextra", "-Werror", f"-I{inc}", str(src),
                        "-o", str(tmp_path / "a.out"),
                        f"-L{pkg}", "-lhxkv", f"-Wl,-rpath,{pkg}"], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr[-3000:]


def test_every_entry_point_refuses_null_arguments(hxlib):
    """Each function of the ABI called with null pointers and zero sizes and
    ids returns a status (or a benign value) instead of crashing, and none
    needs a device to do so."""
    import ctypes as C
    from hxinfer_b200 import _lib
    statuses = {}
    for name, (restype, argtypes) in sorted(_lib.SIGNATURES.items()):
        args = []
        for a in argtypes:
            if a in (C.c_float, C.c_double):
                args.append(1.0)
            elif a in (C.c_uint32,):
                args.append(1)
            elif a in (C.c_int, C.c_int32, C.c_int64, C.c_size_t, C.c_uint64):
                args.append(0)
            else:
                args.append(None)
        statuses[name] = getattr(hxlib, name)(*args)
    int_status = {n: v for n, v in statuses.items() if _lib.SIGNATURES[n][0] is C.c_int}
    # hx_device_status reads the device: HX_ERR_CUDA without one, HX_OK with one
    assert int_status.pop("hx_device_status") in (_lib.HX_OK, _lib.HX_ERR_CUDA)
    # destroying nothing succeeds; everything else refuses the null arguments
    for n in ("hx_kv_destroy", "hx_dist_destroy", "hx_rope_table_destroy"):
        assert int_status.pop(n) == _lib.HX_OK, n
    bad = {n: v for n, v in int_status.items() if v != _lib.HX_ERR_INVALID}
    assert not bad, bad
    assert statuses["hx_decode_workspace_bytes"] == 0 and statuses["hx_snapshot_bytes"] == 0
