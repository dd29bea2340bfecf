"""ctypes binding of libhxkv.so (the C ABI declared in include/hx_kv.h).

The library is the only compute path: if it is missing or fails to load this
module raises; there is no CPU or eager fallback.
"""
from __future__ import annotations

import ctypes as C
import os

PKG = os.path.dirname(os.path.abspath(__file__))
# HXINFER_B200_LIB selects another build of the library (e.g. to compare two
# builds in one process run); default: the in-tree libhxkv.so.
LIB_PATH = os.environ.get("HXINFER_B200_LIB") or os.path.join(PKG, "libhxkv.so")

HX_OK, HX_ERR_INVALID, HX_ERR_CAPACITY, HX_ERR_OOM, HX_ERR_CUDA = 0, 1, 2, 3, 4
HX_ERR_NCCL, HX_ERR_TIMEOUT, HX_ERR_NOT_FOUND, HX_ERR_UNSUPPORTED = 5, 6, 7, 8
HX_FP32, HX_FP16, HX_BF16 = 1, 3, 16
HX_KV_OVERLAP_LAUNCH = 1


class hx_kv_config(C.Structure):
    _fields_ = [("num_layers", C.c_int32), ("num_kv_heads", C.c_int32), ("head_dim", C.c_int32),
                ("max_seqs", C.c_int32), ("max_tokens_per_seq", C.c_int32),
                ("num_blocks", C.c_int64), ("flags", C.c_int32)]


class hx_kv_info(C.Structure):
    _fields_ = [("num_layers", C.c_int32), ("num_kv_heads", C.c_int32), ("head_dim", C.c_int32),
                ("max_seqs", C.c_int32), ("max_blocks_per_seq", C.c_int32),
                ("num_blocks", C.c_int64), ("free_blocks", C.c_int64), ("pool", C.c_void_p),
                ("pool_bytes", C.c_size_t), ("layer_stride_bytes", C.c_int64),
                ("kv_stride_bytes", C.c_int64), ("block_stride_bytes", C.c_int64),
                ("head_stride_bytes", C.c_int64), ("block_table", C.c_void_p)]


class hx_rope_config(C.Structure):
    _fields_ = [("head_dim", C.c_int32), ("max_pos", C.c_int32), ("theta", C.c_float),
                ("use_yarn", C.c_int32), ("yarn_factor", C.c_float), ("yarn_beta_fast", C.c_float),
                ("yarn_beta_slow", C.c_float), ("yarn_orig_max_pos", C.c_int32)]


class hx_append_spec(C.Structure):
    _fields_ = [("k", C.c_void_p), ("v", C.c_void_p), ("bq", C.c_void_p), ("bk", C.c_void_p),
                ("bv", C.c_void_p), ("dtype", C.c_int32), ("table", C.c_void_p)]


_P = C.c_void_p
_I = C.c_int
# name -> (restype, argtypes); this table is the Python view of include/hx_kv.h
SIGNATURES = {
    "hx_status_string": (C.c_char_p, [_I]),
    "hx_last_error": (C.c_char_p, []),
    "hx_device_status": (_I, [_I]),
    "hx_kv_create": (_I, [C.POINTER(hx_kv_config), C.POINTER(_P)]),
    "hx_kv_wrap": (_I, [_P, _P, _I, _I, _I, C.POINTER(_P)]),
    "hx_kv_destroy": (_I, [_P]),
    "hx_kv_get_info": (_I, [_P, C.POINTER(hx_kv_info)]),
    "hx_kv_reserve": (_I, [_P, _I, _I, _P]),
    "hx_kv_release": (_I, [_P, _I, _P]),
    "hx_kv_write": (_I, [_P, _I, _I, _I, _I, _P, _P, _I, _P]),
    "hx_kv_read": (_I, [_P, _I, _I, _I, _I, _P, _P, _P]),
    "hx_kv_fill_normal": (_I, [_P, C.c_uint64, _P]),
    "hx_rope_table_create": (_I, [C.POINTER(hx_rope_config), C.POINTER(_P)]),
    "hx_rope_table_destroy": (_I, [_P]),
    "hx_rope_qk": (_I, [_P, _P, _I, _I, _I, _I, _I, _I, _P, _P]),
    "hx_rope_append": (_I, [_P, _I, _P, _P, _P, _I, _P, _P, _P, _P, _P, _I, _I, _P, _P, _I, _P]),
    "hx_qkv_rope_append": (_I, [_P, _I, _P, _I, _I, _P, _P, _P, _I, _P, _P, _P, _P, _P, _I, _I,
                                _P, _P, _I, _P]),
    "hx_decode_workspace_bytes": (C.c_size_t, [_P, _I, _I]),
    "hx_decode_attention": (_I, [_P, _I, _P, _I, _P, _P, _I, _I, C.c_float, _P, _I, _P,
                                 C.c_size_t, _P]),
    "hx_decode_attention_noalloc": (_I, [_P, _I, _P, _I, _P, _P, _I, _I, C.c_float, _P, _I,
                                         _P]),
    "hx_append_decode_attention": (_I, [_P, _I, _P, C.POINTER(hx_append_spec), _P, _P, _I, _I,
                                        C.c_float, _P, _I, _P, C.c_size_t, _P]),
    "hx_prefill_attention": (_I, [_P, _I, _P, _I, _I, _I, _I, C.c_float, _P, _I, _P]),
    "hx_snapshot_bytes": (C.c_size_t, [_P, _I]),
    "hx_kv_snapshot": (_I, [_P, _I, _I, _P, C.c_size_t, _P]),
    "hx_kv_restore": (_I, [_P, _I, _I, _P, C.c_size_t, _P]),
    "hx_kv_snapshot_layers": (_I, [C.POINTER(_P), _I, _I, _P, C.c_size_t, _P]),
    "hx_kv_restore_layers": (_I, [C.POINTER(_P), _I, _I, _P, C.c_size_t, _P]),
    "hx_prefix_hash": (C.c_uint64, [C.POINTER(C.c_int32), C.c_size_t]),
    "hx_convert": (_I, [_P, _I, _P, _I, C.c_size_t, _P]),
    "hx_dist_handle_bytes": (C.c_size_t, []),
    "hx_dist_create": (_I, [_I, _I, C.c_size_t, C.POINTER(_P)]),
    "hx_dist_export": (_I, [_P, _P]),
    "hx_dist_connect": (_I, [_P, _P]),
    "hx_dist_destroy": (_I, [_P]),
    "hx_dist_buffer": (_P, [_P]),
    "hx_decode_attention_gather": (_I, [_P, _I, _P, _I, _P, _P, _I, _I, C.c_float, _P,
                                        C.c_size_t, _P, _I, _I, _I, _P, C.c_size_t, _P]),
    "hx_append_decode_attention_gather": (_I, [_P, _I, _P, C.POINTER(hx_append_spec), _P, _P,
                                               _I, _I, C.c_float, _P, C.c_size_t, _P, _I, _I,
                                               _I, _P, C.c_size_t, _P]),
    "hx_dist_wait": (_I, [_P, C.c_uint32, _P]),
}

_lib = None


class HXError(RuntimeError):
    def __init__(self, status: int, msg: str):
        super().__init__(f"hx status {status}: {msg}")
        self.status = status


def load():
    """Loads libhxkv.so (building it first if it is absent and nvcc exists)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        from . import build as _build
        _build.build()
    lib = C.CDLL(LIB_PATH)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def check(rc: int, what: str = ""):
    if rc != HX_OK:
        msg = load().hx_last_error().decode(errors="replace")
        raise HXError(rc, f"{what}: {msg}" if what else msg)
    return rc
