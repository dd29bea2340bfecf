"""ctypes front end of the CPU oracle — TEST INFRASTRUCTURE ONLY.

Only tests/, ``__graft_entry__.smoke()`` and the CPU-baseline leg of
``bench.py`` import this module, and only as the checker.  It wraps

* ``oracle/liboracle.so`` — the C restatement in ``hx_oracle.c`` of the
  reference's CPU algorithms (RoPE rope_cpu.cpp:5-39, the CPU attention loop
  attention.cpp:49-85 with the GQA mapping of attention_score_cuda.cu:20-21,
  softmax_cpu.cpp:6-46, the prefix-cache FNV-1a hash prefix_cache.h:42-49);
* ``oracle/_ref/libhxref.so`` (optional) — the reference engine's own CPU ops
  compiled from its sources by ``oracle/Makefile``;

and restates in numpy the checkpoint dtype conversions of the reference's
SafetensorsReader::get_tensor_gpu (model_loaders/src/safetensors_loader.cpp:
12-27, 124-205), pinned by tests/golden/convert_golden.npz to CUDA's host
__float2half / __half2float, the functions the reference's loops call.

All inputs are fp32 numpy arrays; fp16 data is rounded with numpy (RNE) and
upcast before it reaches the oracle, because the reference CPU ops are
fp32-only (hxinfer-engine/include/base/dispatch.h:10-19).
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
_F = C.POINTER(C.c_float)
_I = C.POINTER(C.c_int)

_lib = None
_ref = None


def _fp(a: np.ndarray):
    assert a.dtype == np.float32 and a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(_F)


def _ip(a: np.ndarray):
    assert a.dtype == np.int32 and a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(_I)


def lib():
    """The C restatement (built by ``make -C oracle``)."""
    global _lib
    if _lib is None:
        path = os.path.join(HERE, "liboracle.so")
        if not os.path.exists(path):
            raise RuntimeError(f"oracle library missing: {path} (run make -C oracle)")
        L = C.CDLL(path)
        L.orc_rope_neox.argtypes = [_F, C.c_long, C.c_int, C.c_int, C.c_int, C.c_int, C.c_float]
        L.orc_rope_neox_rows.argtypes = [_F, C.c_long, C.c_int, C.c_int, C.c_int, _I, C.c_float]
        L.orc_yarn_scale.argtypes = [_F, C.c_int, C.c_int, C.c_float, C.c_float, C.c_float,
                                     C.c_float, C.c_int]
        L.orc_yarn_attn_factor.argtypes = [C.c_float]
        L.orc_yarn_attn_factor.restype = C.c_float
        L.orc_rope_neox_yarn.argtypes = [_F, C.c_long, C.c_int, C.c_int, C.c_int, C.c_int,
                                         C.c_float, _F, C.c_float]
        L.orc_rope_table.argtypes = [_F, C.c_int, C.c_int, C.c_float, _F, C.c_float]
        L.orc_softmax.argtypes = [_F, _F, C.c_long]
        L.orc_decode_attention.argtypes = [_F, _F, _F, C.c_int, C.c_int, C.c_int, C.c_int, _F]
        L.orc_prefill_attention.argtypes = [_F, _F, _F, C.c_int, C.c_int, C.c_int, C.c_int,
                                            C.c_int, _F]
        L.orc_decode_attention_batch.argtypes = [_F, C.POINTER(_F), C.POINTER(_F), _I, C.c_int,
                                                 C.c_int, C.c_int, C.c_int, _F, C.c_int]
        L.orc_fnv1a64.argtypes = [_I, C.c_long]
        L.orc_fnv1a64.restype = C.c_uint64
        _lib = L
    return _lib


def ref_available() -> bool:
    return os.path.exists(os.path.join(HERE, "_ref", "libhxref.so"))


def ref():
    """The reference engine's own CPU ops (built by ``make -C oracle ref``)."""
    global _ref
    if _ref is None:
        path = os.path.join(HERE, "_ref", "libhxref.so")
        if not os.path.exists(path):
            raise RuntimeError(f"reference library missing: {path} (run make -C oracle ref)")
        R = C.CDLL(path)
        R.ref_rope_cpu.argtypes = [_F, _F, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_float]
        R.ref_rope_cuda.argtypes = [_F, _F, C.c_int, C.c_int, C.c_int, C.c_int, C.c_float,
                                    C.c_int, C.c_float, C.c_float, C.c_float, C.c_int]
        R.ref_softmax_cpu.argtypes = [_F, _F, C.c_int]
        R.ref_attention_layer_cpu.argtypes = [C.c_int, C.c_int, C.c_int, C.c_float, _F, _F, _F,
                                              _F, _F, C.c_int, _F]
        R.ref_prefix_hash.argtypes = [_I, C.c_int]
        R.ref_prefix_hash.restype = C.c_ulonglong
        R.ref_prefix_cache_roundtrip.argtypes = [C.c_int, C.c_int, C.c_int, C.c_int, _F, _F, _I,
                                                 C.c_int, _I, C.c_int, _F, _F,
                                                 C.POINTER(C.c_longlong)]
        _ref = R
    return _ref


# ---------------------------------------------------------------- restatement

def rope(x: np.ndarray, num_heads: int, head_dim: int, step, base: float) -> np.ndarray:
    """NeoX RoPE of x [rows, num_heads*head_dim]; ``step`` is an int or one int per row."""
    y = np.ascontiguousarray(x, dtype=np.float32).copy()
    rows = y.shape[0] if y.ndim > 1 else 1
    row_dim = y.shape[-1]
    if np.isscalar(step):
        lib().orc_rope_neox(_fp(y), rows, row_dim, num_heads, head_dim, int(step), base)
    else:
        st = np.ascontiguousarray(step, dtype=np.int32)
        assert st.shape[0] == rows
        lib().orc_rope_neox_rows(_fp(y), rows, row_dim, num_heads, head_dim, _ip(st), base)
    return y


def yarn_scale(head_dim: int, factor: float, base: float, beta_fast: float, beta_slow: float,
               orig_max_pos: int) -> np.ndarray:
    out = np.zeros(head_dim // 2, np.float32)
    lib().orc_yarn_scale(_fp(out), head_dim // 2, head_dim, factor, base, beta_fast, beta_slow,
                         orig_max_pos)
    return out


def yarn_attn_factor(factor: float) -> float:
    return float(lib().orc_yarn_attn_factor(factor))


def rope_yarn(x: np.ndarray, num_heads: int, head_dim: int, step: int, base: float,
              scale: np.ndarray, attn_factor: float) -> np.ndarray:
    y = np.ascontiguousarray(x, dtype=np.float32).copy()
    rows = y.shape[0] if y.ndim > 1 else 1
    s = np.ascontiguousarray(scale, dtype=np.float32)
    lib().orc_rope_neox_yarn(_fp(y), rows, y.shape[-1], num_heads, head_dim, step, base, _fp(s),
                             attn_factor)
    return y


def rope_table(max_pos: int, head_dim: int, base: float, yarn=None, attn_factor=1.0):
    out = np.zeros((max_pos, head_dim // 2, 2), np.float32)
    ys = None if yarn is None else np.ascontiguousarray(yarn, dtype=np.float32)
    lib().orc_rope_table(_fp(out), max_pos, head_dim, base, None if ys is None else _fp(ys),
                         attn_factor)
    return out


def softmax(x: np.ndarray) -> np.ndarray:
    a = np.ascontiguousarray(x, dtype=np.float32)
    out = np.zeros_like(a)
    lib().orc_softmax(_fp(a), _fp(out), a.size)
    return out


def decode_attention(q: np.ndarray, k_cache: np.ndarray, v_cache: np.ndarray, Hq: int,
                     Hkv: int, head_dim: int) -> np.ndarray:
    """q [Hq*hd]; k_cache/v_cache token-major [L, Hkv*hd] -> out [Hq*hd]."""
    q = np.ascontiguousarray(q, dtype=np.float32).reshape(-1)
    k = np.ascontiguousarray(k_cache, dtype=np.float32)
    v = np.ascontiguousarray(v_cache, dtype=np.float32)
    L = k.shape[0]
    out = np.zeros(Hq * head_dim, np.float32)
    lib().orc_decode_attention(_fp(q), _fp(k), _fp(v), L, Hq, Hkv, head_dim, _fp(out))
    return out


def prefill_attention(q: np.ndarray, k_cache: np.ndarray, v_cache: np.ndarray, start: int,
                      Hq: int, Hkv: int, head_dim: int) -> np.ndarray:
    """q [n, Hq*hd] (rotated) at positions start..start+n-1; causal over the cache."""
    q = np.ascontiguousarray(q, dtype=np.float32)
    k = np.ascontiguousarray(k_cache, dtype=np.float32)
    v = np.ascontiguousarray(v_cache, dtype=np.float32)
    n = q.shape[0]
    assert k.shape[0] >= start + n
    out = np.zeros_like(q)
    lib().orc_prefill_attention(_fp(q), _fp(k), _fp(v), start, n, Hq, Hkv, head_dim, _fp(out))
    return out


def decode_attention_batch(q: np.ndarray, k_caches, v_caches, Hq: int, Hkv: int, head_dim: int,
                           nthreads: int = 1) -> np.ndarray:
    """q [n_seqs, Hq*hd]; k_caches[s]/v_caches[s] token-major [L_s, Hkv*hd]."""
    q = np.ascontiguousarray(q, dtype=np.float32)
    n = q.shape[0]
    ks = [np.ascontiguousarray(k, dtype=np.float32) for k in k_caches]
    vs = [np.ascontiguousarray(v, dtype=np.float32) for v in v_caches]
    kp = (_F * n)(*[_fp(k) for k in ks])
    vp = (_F * n)(*[_fp(v) for v in vs])
    lens = np.array([k.shape[0] for k in ks], np.int32)
    out = np.zeros_like(q)
    lib().orc_decode_attention_batch(_fp(q), kp, vp, _ip(lens), n, Hq, Hkv, head_dim, _fp(out),
                                     nthreads)
    return out


def fnv1a64(tokens) -> int:
    t = np.ascontiguousarray(tokens, dtype=np.int32)
    return int(lib().orc_fnv1a64(_ip(t), t.size))


def f16(x: np.ndarray) -> np.ndarray:
    """Round to fp16 (RNE) and upcast: the fp16 storage seen by an fp32 CPU op."""
    return np.asarray(x, dtype=np.float32).astype(np.float16).astype(np.float32)


# ---------------------------------------------------------------- reference

def ref_rope(q: np.ndarray, k: np.ndarray, Hq: int, Hkv: int, head_dim: int, step: int,
             base: float):
    qq = np.ascontiguousarray(q, dtype=np.float32).copy()
    kk = np.ascontiguousarray(k, dtype=np.float32).copy()
    rows = qq.shape[0] if qq.ndim > 1 else 1
    rc = ref().ref_rope_cpu(_fp(qq), _fp(kk), rows, Hq, Hkv, head_dim, step, base)
    assert rc == 0
    return qq, kk


def ref_rope_cuda(q: np.ndarray, k: np.ndarray, Hq: int, Hkv: int, head_dim: int, step: int,
                  base: float, yarn: dict | None = None):
    """The reference's own rope_cuda (rope_cuda.cu:98-152) on one token row,
    run on the current CUDA device; ``yarn`` = dict(factor, beta_fast,
    beta_slow, orig_max_pos) turns its YaRN path on.  Needs a GPU."""
    qq = np.ascontiguousarray(q, dtype=np.float32).reshape(-1).copy()
    kk = np.ascontiguousarray(k, dtype=np.float32).reshape(-1).copy()
    y = yarn or {}
    rc = ref().ref_rope_cuda(_fp(qq), _fp(kk), Hq, Hkv, head_dim, step, base, 1 if yarn else 0,
                             y.get("factor", 1.0), y.get("beta_fast", 32.0),
                             y.get("beta_slow", 1.0), y.get("orig_max_pos", 4096))
    assert rc == 0, f"ref_rope_cuda returned {rc}"
    return qq, kk


def ref_softmax(x: np.ndarray) -> np.ndarray:
    a = np.ascontiguousarray(x, dtype=np.float32)
    out = np.zeros_like(a)
    assert ref().ref_softmax_cpu(_fp(a), _fp(out), a.size) == 0
    return out


def ref_attention_layer(dim: int, head: int, theta: float, wq, wk, wv, wo, x) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    ws = [np.ascontiguousarray(w, dtype=np.float32) for w in (wq, wk, wv, wo)]
    n = x.shape[0]
    out = np.zeros_like(x)
    rc = ref().ref_attention_layer_cpu(dim, head, n, theta, *[_fp(w) for w in ws], _fp(x), n,
                                       _fp(out))
    assert rc == 0
    return out


def ref_hash(tokens) -> int:
    t = np.ascontiguousarray(tokens, dtype=np.int32)
    return int(ref().ref_prefix_hash(_ip(t), t.size))


def ref_prefix_roundtrip(layers, dim, head, seq_len, init_kv, overwrite_kv, prefix, probe):
    init_kv = np.ascontiguousarray(init_kv, dtype=np.float32)
    overwrite_kv = np.ascontiguousarray(overwrite_kv, dtype=np.float32)
    pre = np.ascontiguousarray(prefix, dtype=np.int32)
    prb = np.ascontiguousarray(probe, dtype=np.int32)
    after_miss = np.zeros_like(init_kv)
    after_restore = np.zeros_like(init_kv)
    hits = (C.c_longlong * 3)()
    rc = ref().ref_prefix_cache_roundtrip(layers, dim, head, seq_len, _fp(init_kv),
                                          _fp(overwrite_kv), _ip(pre), pre.size, _ip(prb),
                                          prb.size, _fp(after_miss), _fp(after_restore), hits)
    assert rc == 0
    return after_miss, after_restore, list(hits)


# ---------------------------------------------------------------- checkpoint dtype conversion
# SafetensorsReader::get_tensor_gpu converts on the CPU before uploading
# (model_loaders/src/safetensors_loader.cpp:124-205).  numpy's float32 ->
# float16 cast is the IEEE 754 narrowing (round to nearest even, overflow to
# infinity) that CUDA's __float2half performs; BF16 -> FP32 is a 16-bit shift.

def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    """BF16 bit patterns (uint16) -> fp32, exact: the 16 bits become the top
    half of the fp32 word (safetensors_loader.cpp:20-24, 135-146)."""
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_f16(x: np.ndarray) -> np.ndarray:
    """fp32 -> fp16 as __float2half (safetensors_loader.cpp:25, 158-168)."""
    with np.errstate(over="ignore", invalid="ignore"):
        return np.asarray(x, dtype=np.float32).astype(np.float16)


def convert(raw: np.ndarray, src: str, dst: str) -> np.ndarray:
    """One tensor as SafetensorsReader::get_tensor_gpu returns it.

    raw: the tensor's bytes (uint8); src: its safetensors dtype ("F32", "F16",
    "BF16" or "I8"); dst: the target DataType ("FP16", "FP32" or "Int8").
    Pairs follow safetensors_loader.cpp (BF16->FP16 :125-132, BF16->FP32
    :135-146, F16->FP16 :149-155, F32->FP16 :158-168, F32->FP32 :171-177,
    F16->FP32 :180-197) and I8->Int8 (the byte copy of its fallback,
    :200-205).  Other pairs raise ValueError.
    """
    raw = np.ascontiguousarray(raw, dtype=np.uint8)
    if src == "BF16" and dst == "FP16":
        return f32_to_f16(bf16_bits_to_f32(raw.view(np.uint16)))
    if src == "BF16" and dst == "FP32":
        return bf16_bits_to_f32(raw.view(np.uint16))
    if src == "F16" and dst == "FP16":
        return raw.view(np.float16).copy()
    if src == "F32" and dst == "FP16":
        return f32_to_f16(raw.view(np.float32))
    if src == "F32" and dst == "FP32":
        return raw.view(np.float32).copy()
    if src == "F16" and dst == "FP32":
        return raw.view(np.float16).astype(np.float32)
    if src == "I8" and dst == "Int8":
        return raw.view(np.int8).copy()
    raise ValueError(f"no conversion {src} -> {dst}")


def canonical_nan_bits(a: np.ndarray) -> np.ndarray:
    """Bit patterns of a float16 / float32 array with every NaN replaced by
    one quiet NaN (0x7FFF / 0x7FFFFFFF): NaN outputs are compared as NaN, not
    by payload."""
    a = np.asarray(a)
    if a.dtype == np.float16:
        bits = a.view(np.uint16).copy()
        bits[np.isnan(a)] = 0x7FFF
        return bits
    assert a.dtype == np.float32
    bits = a.view(np.uint32).copy()
    bits[np.isnan(a)] = 0x7FFFFFFF
    return bits
