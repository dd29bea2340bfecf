// attention_loader.cpp — config.json and attention weights of a dense
// checkpoint (the KV-cache path's part of model_loaders/src/
// dense_model_loader.cpp:20-156).
#include "model_loaders/attention_loader.h"

#include <fstream>
#include <iostream>
#include <iterator>
#include <stdexcept>

#include "json_lite.h"
#include "model_loaders/safetensors_loader.h"

namespace hxinfer {

namespace {

using json_lite::Value;

std::string weight_name(int layer, const std::string& suffix)
{
    return "model.layers." + std::to_string(layer) + "." + suffix;
}

int required_int(const Value& cfg, const char* key)
{
    const Value* v = cfg.find(key);
    if (!v || v->kind != Value::Number)
        throw std::runtime_error(std::string("config.json: missing or non-numeric '") + key + "'");
    return v->is_int ? (int)v->integer : (int)v->number;
}

int int_or(const Value& obj, const char* key, int fallback)
{
    const Value* v = obj.find(key);
    if (!v || v->kind != Value::Number) return fallback;
    return v->is_int ? (int)v->integer : (int)v->number;
}

float float_or(const Value& obj, const char* key, float fallback)
{
    const Value* v = obj.find(key);
    if (!v || v->kind != Value::Number) return fallback;
    return v->is_int ? (float)v->integer : (float)v->number;
}

std::string string_or(const Value& obj, const char* key, const std::string& fallback)
{
    const Value* v = obj.find(key);
    return v && v->kind == Value::String ? v->str : fallback;
}

}  // namespace

void AttentionLoader::load_config(const std::string& model_dir, ModelConfig& out_config)
{
    const std::string config_path = model_dir + "/config.json";
    std::ifstream cf(config_path, std::ios::binary);
    if (!cf) throw std::runtime_error("config.json not found: " + config_path);
    const std::string text((std::istreambuf_iterator<char>(cf)), std::istreambuf_iterator<char>());
    Value cfg;
    std::string err;
    if (!json_lite::parse(text.data(), text.data() + text.size(), cfg, &err) || cfg.kind != Value::Object)
        throw std::runtime_error("config.json is not a JSON object: " + config_path + " " + err);

    out_config.dim = required_int(cfg, "hidden_size");
    out_config.hidden_dim = required_int(cfg, "intermediate_size");
    out_config.layer = required_int(cfg, "num_hidden_layers");
    out_config.head = required_int(cfg, "num_attention_heads");
    out_config.kv_head = int_or(cfg, "num_key_value_heads", out_config.head);
    out_config.vocab_size = required_int(cfg, "vocab_size");
    out_config.seq_len = 4096;
    out_config.rope_theta = float_or(cfg, "rope_theta", 10000.0f);

    const Value* rs = cfg.find("rope_scaling");
    if (rs && rs->kind == Value::Object) {
        const std::string rs_type = string_or(*rs, "type", string_or(*rs, "rope_type", ""));
        if (rs_type == "yarn") {
            out_config.rope_use_yarn = true;
            out_config.rope_factor = float_or(*rs, "factor", 1.0f);
            out_config.rope_orig_max_pos = int_or(*rs, "original_max_position_embeddings", 4096);
            out_config.rope_beta_fast = float_or(*rs, "beta_fast", 32.0f);
            out_config.rope_beta_slow = float_or(*rs, "beta_slow", 1.0f);
        }
    }
}

std::vector<std::shared_ptr<AttentionLayer>> AttentionLoader::load_layers(
    const std::string& model_dir, ModelConfig& out_config,
    const std::shared_ptr<CUDAAllocator>& cuda_alloc)
{
    load_config(model_dir, out_config);
    ModelConfig& c = out_config;
    std::cout << ">>> [Loader] attention layers: dim=" << c.dim << " layers=" << c.layer << " heads=" << c.head
              << " kv_heads=" << c.kv_head << " rope_theta=" << c.rope_theta
              << (c.rope_use_yarn ? " (YaRN)" : "") << "\n";

    SafetensorsMultiReader reader;
    if (!reader.load_directory(model_dir))
        throw std::runtime_error("No .safetensors files found in: " + model_dir);

    std::vector<std::shared_ptr<AttentionLayer>> layers;
    layers.reserve(c.layer);
    for (int i = 0; i < c.layer; ++i) {
        auto get = [&](const char* suffix, DataType dt) {
            auto t = reader.get_tensor_gpu(weight_name(i, suffix), cuda_alloc, dt);
            if (!t) throw std::runtime_error("cannot load " + weight_name(i, suffix));
            return t;
        };
        auto wq = get("self_attn.q_proj.weight", c.weight_dtype);
        auto wk = get("self_attn.k_proj.weight", c.weight_dtype);
        auto wv = get("self_attn.v_proj.weight", c.weight_dtype);
        auto wo = get("self_attn.o_proj.weight", c.weight_dtype);
        if (reader.has_tensor(weight_name(i, "self_attn.q_proj.bias"))) {
            auto bq = get("self_attn.q_proj.bias", c.bias_dtype);
            auto bk = get("self_attn.k_proj.bias", c.bias_dtype);
            auto bv = get("self_attn.v_proj.bias", c.bias_dtype);
            layers.push_back(std::make_shared<AttentionLayer>(cuda_alloc, c, wq, wk, wv, wo, bq, bk, bv));
        } else {
            layers.push_back(std::make_shared<AttentionLayer>(cuda_alloc, c, wq, wk, wv, wo));
        }
    }
    return layers;
}

}  // namespace hxinfer
