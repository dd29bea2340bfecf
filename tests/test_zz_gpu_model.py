"""The reference's CausalLMModel on the GPU with the drop-in attention layer.

oracle/model_driver.cpp, built twice by `make -C oracle models` (where the
reference sources are present; the binaries travel with the repository):
model_ref is the reference engine as it is, model_b200 the same engine with
the hot-path headers replaced by this build's and libhxinfer.so / libhxkv.so
linked in.  Both load one toy checkpoint (random weights, written here in
the safetensors layout the reference's DenseModelLoader reads) and run
CausalLMModel::forward one token per call (causal_lm_model.cpp:4-12,
transformer.cpp:4-17), writing every position's logits.

Bars: model_b200's logits against model_ref's within 1e-2 of the largest
logit magnitude, and the same argmax at every position (the reference keeps
its KV cache in fp32, this build in fp16: the 2e-3 / 1e-2 tolerance of the
attention layer, carried through the toy model); PrefixCacheManager at model
level (store, overwrite, restore, continue) bit-exact against the first run.
"""
import json
import os
import subprocess
import sys

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
sys.path.insert(0, HERE)
from safetensors_files import write_safetensors  # noqa: E402

pytestmark = pytest.mark.gpu

REF_BIN = os.path.join(ROOT, "oracle", "_ref", "model_ref")
B200_BIN = os.path.join(ROOT, "oracle", "_ref", "model_b200")
TOKENS, PREFIX = 100, 70

TOY = {
    # name: (model type, config.json fields)
    "llama": ("llama", {"hidden_size": 512, "intermediate_size": 1024, "num_hidden_layers": 2,
                        "num_attention_heads": 4, "num_key_value_heads": 4, "vocab_size": 1000}),
    "qwen2_gqa": ("qwen2", {"hidden_size": 1024, "intermediate_size": 2048, "num_hidden_layers": 2,
                            "num_attention_heads": 8, "num_key_value_heads": 2, "vocab_size": 1000,
                            "rope_theta": 1000000.0}),
    "yarn": ("llama", {"hidden_size": 512, "intermediate_size": 1024, "num_hidden_layers": 2,
                       "num_attention_heads": 4, "num_key_value_heads": 2, "vocab_size": 1000,
                       "rope_scaling": {"type": "yarn", "factor": 4.0,
                                        "original_max_position_embeddings": 32}}),
}


def write_toy(path, kind, cfg, seed):
    rng = np.random.default_rng(seed)
    d, f, nl, v = cfg["hidden_size"], cfg["intermediate_size"], cfg["num_hidden_layers"], cfg["vocab_size"]
    hd = d // cfg["num_attention_heads"]
    kvd = cfg["num_key_value_heads"] * hd

    def w(*shape, std=0.05):
        return ("F16", shape, (rng.standard_normal(shape) * std).astype(np.float16).tobytes())

    def norm(n):
        return ("F32", (n,), (1.0 + 0.1 * rng.standard_normal(n)).astype(np.float32).tobytes())

    t = [("model.embed_tokens.weight",) + w(v, d, std=1.0), ("model.norm.weight",) + norm(d),
         ("lm_head.weight",) + w(v, d)]
    for i in range(nl):
        p = f"model.layers.{i}."
        t += [(p + "input_layernorm.weight",) + norm(d), (p + "post_attention_layernorm.weight",) + norm(d),
              (p + "self_attn.q_proj.weight",) + w(d, d), (p + "self_attn.k_proj.weight",) + w(kvd, d),
              (p + "self_attn.v_proj.weight",) + w(kvd, d), (p + "self_attn.o_proj.weight",) + w(d, d),
              (p + "mlp.gate_proj.weight",) + w(f, d), (p + "mlp.up_proj.weight",) + w(f, d),
              (p + "mlp.down_proj.weight",) + w(d, f)]
        if kind == "qwen2":
            for n, size in (("q", d), ("k", kvd), ("v", kvd)):
                b = (0.1 * rng.standard_normal(size)).astype(np.float32)
                t.append((p + f"self_attn.{n}_proj.bias", "F32", (size,), b.tobytes()))
    os.makedirs(path, exist_ok=True)
    write_safetensors(os.path.join(path, "model.safetensors"), t)
    with open(os.path.join(path, "config.json"), "w") as fh:
        json.dump(cfg, fh)


def run(binary, model_dir, kind, out, prefix=None):
    cmd = [binary, model_dir, kind, str(TOKENS), out] + ([str(prefix)] if prefix else [])
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, (cmd, r.stdout[-2000:], r.stderr[-2000:])
    return np.fromfile(out, dtype=np.float32)


@pytest.mark.skipif(not (os.path.exists(REF_BIN) and os.path.exists(B200_BIN)),
                    reason="model drivers not built (make -C oracle models, needs the reference sources)")
@pytest.mark.parametrize("name", sorted(TOY))
def test_causal_lm_with_dropin_layer(tmp_path, name):
    kind, cfg = TOY[name]
    model_dir = str(tmp_path / name)
    write_toy(model_dir, kind, cfg, seed=len(name))
    v = cfg["vocab_size"]
    ref = run(REF_BIN, model_dir, kind, str(tmp_path / "ref.bin")).reshape(TOKENS, v)
    got = run(B200_BIN, model_dir, kind, str(tmp_path / "b200.bin"), PREFIX)
    assert got.size == (2 * TOKENS - PREFIX) * v
    got = got.reshape(-1, v)
    first, again = got[:TOKENS], got[TOKENS:]
    assert np.isfinite(ref).all() and np.isfinite(first).all()
    err = np.abs(first - ref).max()
    scale = np.abs(ref).max()
    assert err <= 1e-2 * scale, f"{name}: max |b200 - ref| {err:.3e}, max |ref| {scale:.3e}"
    assert (first.argmax(1) == ref.argmax(1)).all(), f"{name}: argmax differs at " \
        f"{np.nonzero(first.argmax(1) != ref.argmax(1))[0].tolist()}"
    # the continuation after a model-level restore reproduces the first run bit for bit
    assert np.array_equal(again.view(np.uint32), first[PREFIX:].view(np.uint32))
