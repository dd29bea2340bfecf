"""Generate the golden vectors in tests/golden/reference_golden.npz.

Every output in the file comes from the reference engine's own CPU code,
compiled from its sources by ``make -C oracle ref`` into
``oracle/_ref/libhxref.so`` and called through ``oracle/ref_driver.cpp``.
Inputs are seeded (numpy PCG64) N(0,1) values rounded to fp16 and upcast, the
fp16 storage the KV-cache path keeps.  Run from the repository root:

    make -C oracle all ref && python tests/golden/make_golden.py

Cases (reference file:line of the code that produced each output):
  rope_kat_*      the RoPE known-answer inputs of tests/unit/test_unit_ops.cpp:197-229
  rope_qwen_*     Qwen2.5-7B q/k (28/4 heads x 128) at step 1024, theta 1e6  (rope_cpu.cpp:5-39)
  rope_llama_*    LLaMA-2-7B q/k (32/32 heads x 128) at step 7, theta 1e4
  softmax_*       1025 scores                                               (softmax_cpu.cpp:6-46)
  attn_*          AttentionLayer CPU branch, MHA 2 heads x 128, 20 positions,
                  signed-permutation projections so q/k/v/o are exact       (attention.cpp:37-88)
  hash_*          PrefixCacheManager::compute_hash of token vectors         (prefix_cache.h:42-49)
  prefix_*        PrefixCacheManager store / lookup / restore on a 2-layer
                  CPU LlamaModel (dim 16, seq_len 8, prefix 5)               (prefix_cache.h:58-151)
"""
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)
from oracle import oracle as O  # noqa: E402

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "reference_golden.npz")


def signed_perm(dim: int, seed: int) -> np.ndarray:
    r = np.random.default_rng(seed)
    w = np.zeros((dim, dim), np.float32)
    w[np.arange(dim), r.permutation(dim)] = r.choice([-2.0, -1.0, 0.5, 1.0], dim)
    return w


def main():
    if not O.ref_available():
        sys.exit("oracle/_ref/libhxref.so missing: run make -C oracle ref first")
    g = {}
    rng = np.random.default_rng(20261201)

    kat = np.array([[1.0, 2.0, 3.0, 4.0]], np.float32)
    for step in (0, 1):
        q, k = O.ref_rope(kat, kat, 1, 1, 4, step, 10000.0)
        g[f"rope_kat_in"] = kat
        g[f"rope_kat_q_step{step}"] = q
        g[f"rope_kat_k_step{step}"] = k

    for name, hq, hkv, step, theta in (("qwen", 28, 4, 1024, 1e6), ("llama", 32, 32, 7, 1e4)):
        q = O.f16(rng.standard_normal((3, hq * 128)))
        k = O.f16(rng.standard_normal((3, hkv * 128)))
        rq, rk = O.ref_rope(q, k, hq, hkv, 128, step, theta)
        g[f"rope_{name}_q_in"], g[f"rope_{name}_k_in"] = q, k
        g[f"rope_{name}_q_out"], g[f"rope_{name}_k_out"] = rq, rk
        g[f"rope_{name}_meta"] = np.array([hq, hkv, step, theta], np.float64)

    s = (rng.standard_normal(1025) * 3).astype(np.float32)
    g["softmax_in"], g["softmax_out"] = s, O.ref_softmax(s)

    head, hd, npos, theta = 2, 128, 20, 1e4
    dim = head * hd
    ws = [signed_perm(dim, 100 + i) for i in range(4)]
    x = O.f16(rng.standard_normal((npos, dim)))
    g["attn_w"] = np.stack(ws)
    g["attn_x"] = x
    g["attn_out"] = O.ref_attention_layer(dim, head, theta, *ws, x)
    g["attn_meta"] = np.array([head, hd, npos, theta], np.float64)

    toks = [np.array(t, np.int32) for t in ([1, 2, 3], [151643, 0, 7, 99999], [-1], [], list(range(2048)))]
    g["hash_tokens"] = np.concatenate([t for t in toks]).astype(np.int32)
    g["hash_lens"] = np.array([t.size for t in toks], np.int32)
    g["hash_out"] = np.array([O.ref_hash(t) for t in toks], np.uint64)

    layers, pdim, phead, seq_len, plen = 2, 16, 2, 8, 5
    init_kv = rng.standard_normal((layers, 2, seq_len, pdim)).astype(np.float32)
    over_kv = rng.standard_normal((layers, 2, seq_len, pdim)).astype(np.float32)
    prefix = rng.integers(0, 152064, plen).astype(np.int32)
    probe = prefix.copy()
    probe[-1] += 1
    after_miss, after_restore, hits = O.ref_prefix_roundtrip(layers, pdim, phead, seq_len, init_kv,
                                                              over_kv, prefix, probe)
    g["prefix_meta"] = np.array([layers, pdim, phead, seq_len, plen], np.int32)
    g["prefix_init_kv"], g["prefix_over_kv"] = init_kv, over_kv
    g["prefix_tokens"], g["prefix_probe"] = prefix, probe
    g["prefix_after_miss"], g["prefix_after_restore"] = after_miss, after_restore
    g["prefix_hits"] = np.array(hits, np.int64)

    np.savez_compressed(OUT, **g)
    print(f"wrote {OUT} ({os.path.getsize(OUT)} bytes, {len(g)} arrays)")


if __name__ == "__main__":
    main()
