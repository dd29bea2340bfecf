// base/config.h — model configuration and element/device types.
//
// Same names, fields and enum values as the reference engine's
// hxinfer-engine/include/base/config.h:5-51, so code written against the
// reference (ModelConfig from its loader, DataType codes) compiles unchanged.
// The KV cache of this build always stores fp16 whatever activation_dtype is.
#ifndef HXINFER_B200_CONFIG_H
#define HXINFER_B200_CONFIG_H
#include <cstdint>

namespace hxinfer {

enum class DataType { kDataTypeUnknown = 0, kDataTypeFP32 = 1, kDataTypeInt8 = 2, kDataTypeFP16 = 3 };
enum class DeviceType { kDeviceCPU = 0, kDeviceCUDA = 1 };

inline int DataTypeSize(DataType t)
{
    switch (t) {
    case DataType::kDataTypeFP32: return 4;
    case DataType::kDataTypeInt8: return 1;
    case DataType::kDataTypeFP16: return 2;
    default: return 0;
    }
}

struct ModelConfig {
    int dim;
    int hidden_dim;
    int layer;
    int head;
    int kv_head;
    int vocab_size;
    int seq_len;

    float rope_factor = 1.0f;
    float rope_beta_fast = 32.0f;
    float rope_beta_slow = 1.0f;
    float rope_theta = 10000.0f;
    int rope_orig_max_pos = 4096;
    bool rope_use_yarn = false;

    DataType weight_dtype = DataType::kDataTypeFP16;
    DataType activation_dtype = DataType::kDataTypeFP32;
    DataType norm_weight_dtype = DataType::kDataTypeFP32;
    DataType bias_dtype = DataType::kDataTypeFP32;
    DataType logits_dtype = DataType::kDataTypeFP32;
};

}  // namespace hxinfer
#endif
