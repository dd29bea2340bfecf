// model_loaders/dense_model_loader.h — the KV-cache path's part of the
// reference's DenseModelLoader (model_loaders/include/dense_model_loader.h:
// 9-25, model_loaders/src/dense_model_loader.cpp:20-156).
//
// The reference's load() reads config.json, opens the shards and builds a
// whole CausalLMModel (embedding, TransformerLayers, final norm, lm_head).
// This build keeps the two steps that feed the attention layers:
//   load_config            config.json -> ModelConfig (dense_model_loader.cpp:27-52,
//                          same keys, defaults and seq_len of 4096)
//   load_attention_layers  q/k/v/o projections (and the q/k/v biases when the
//                          checkpoint has them, as Qwen2 does) of every layer,
//                          named model.layers.<i>.self_attn.* as in
//                          dense_model_loader.cpp:16-18, 92-120, into
//                          AttentionLayer objects over this build's KV cache.
// Embedding, norms, MLP and lm_head belong to the reference's other layers and
// are not loaded here.
#ifndef HXINFER_B200_DENSE_MODEL_LOADER_H
#define HXINFER_B200_DENSE_MODEL_LOADER_H
#include <memory>
#include <string>
#include <vector>

#include "base/allocator.h"
#include "base/config.h"
#include "layer/attention.h"
#include "model_loaders/safetensors_loader.h"

namespace hxinfer {

enum class ModelType {
    LLaMA,  // LLaMA-2/3, Mistral, InternLM2/3 (no QKV bias)
    Qwen2,  // Qwen2/2.5 (QKV bias)
};

class DenseModelLoader {
public:
    // Throws std::runtime_error when config.json is missing, is not valid JSON
    // or lacks a required key (hidden_size, intermediate_size,
    // num_hidden_layers, num_attention_heads, vocab_size).
    static void load_config(const std::string& model_dir, ModelConfig& out_config);

    // load_config, then every layer's attention weights (weights as
    // out_config.weight_dtype, biases as out_config.bias_dtype, converted on
    // the device).  Throws std::runtime_error when no shard loads or a weight
    // is missing or unreadable (the reference passes nullptr on instead).
    // `type` only names the model in the log line; the bias is detected from
    // the checkpoint, as in the reference.
    static std::vector<std::shared_ptr<AttentionLayer>> load_attention_layers(
        const std::string& model_dir, ModelConfig& out_config,
        const std::shared_ptr<CUDAAllocator>& cuda_alloc, ModelType type = ModelType::LLaMA);
};

}  // namespace hxinfer
#endif
