// model_loaders/attention_loader.h — the KV-cache path's part of the
// reference's DenseModelLoader::load (model_loaders/src/
// dense_model_loader.cpp:20-156), as a helper of its own.
//
// The reference's DenseModelLoader::load reads config.json, opens the shards
// through SafetensorsMultiReader and builds a whole CausalLMModel.  The reader
// calls it makes (load_directory, num_tensors, has_tensor, get_tensor_gpu)
// have the same signatures in this build's SafetensorsMultiReader
// (model_loaders/safetensors_loader.h), which is the drop-in.  AttentionLoader
// does the two steps that feed the attention layers, for callers that hold no
// CausalLMModel (tests, attention-only benchmarks on real checkpoints):
//   load_config  config.json -> ModelConfig (dense_model_loader.cpp:27-52:
//                same keys, defaults and seq_len of 4096)
//   load_layers  q/k/v/o projections of every layer, and the q/k/v biases when
//                the checkpoint has them (Qwen2), named
//                model.layers.<i>.self_attn.* (dense_model_loader.cpp:16-18,
//                92-120), into AttentionLayer objects over this build's cache.
#ifndef HXINFER_B200_ATTENTION_LOADER_H
#define HXINFER_B200_ATTENTION_LOADER_H
#include <memory>
#include <string>
#include <vector>

#include "base/allocator.h"
#include "base/config.h"
#include "layer/attention.h"

namespace hxinfer {

class AttentionLoader {
public:
    // Throws std::runtime_error when config.json is missing, is not valid JSON
    // or lacks a required key (hidden_size, intermediate_size,
    // num_hidden_layers, num_attention_heads, vocab_size).
    static void load_config(const std::string& model_dir, ModelConfig& out_config);

    // load_config, then every layer's attention weights (weights as
    // out_config.weight_dtype, biases as out_config.bias_dtype, converted on
    // the device).  Throws std::runtime_error when no shard loads or a weight
    // is missing or unreadable (the reference passes nullptr on instead).  The
    // bias is detected from the checkpoint, as in the reference.
    static std::vector<std::shared_ptr<AttentionLayer>> load_layers(
        const std::string& model_dir, ModelConfig& out_config,
        const std::shared_ptr<CUDAAllocator>& cuda_alloc);
};

}  // namespace hxinfer
#endif
