// ops.cpp — the kept hot-path operators over the C ABI.
//   rope_tensor / rope_cpu / rope_cuda      math_ops.h:28-30 (reference rope_tensor.cpp:4-12)
//   attention_score_cuda                    math_ops.h:67-73 (reference attention_score_cuda.cu:163-214)
#include <cuda_runtime.h>

#include <cmath>
#include <iostream>
#include <stdexcept>

#include "device_context.h"
#include "op/math_ops.h"

namespace hxinfer {

static int hx_dtype_of(DataType t)
{
    if (t == DataType::kDataTypeFP16) return HX_FP16;
    if (t == DataType::kDataTypeFP32) return HX_FP32;
    return -1;
}

void rope_tensor(std::shared_ptr<Tensor>& q, std::shared_ptr<Tensor>& k, ModelConfig& config,
                 int step, float base)
{
    if (q->tensor_device_type() == DeviceType::kDeviceCUDA) {
        rope_cuda(q, k, config, step, base);
    } else if (q->tensor_device_type() == DeviceType::kDeviceCPU) {
        rope_cpu(q, k, config, step, base);
    } else {
        std::cerr << "Unknown device type for rope_tensor!" << std::endl;
    }
}

void rope_cpu(std::shared_ptr<Tensor>&, std::shared_ptr<Tensor>&, ModelConfig&, int, float)
{
    throw std::runtime_error("rope_cpu: CPU tensors are not supported by the B200 build");
}

void rope_cuda(std::shared_ptr<Tensor>& q, std::shared_ptr<Tensor>& k, ModelConfig& config,
               int step, float base)
{
    if (q->tensor_device_type() != DeviceType::kDeviceCUDA ||
        k->tensor_device_type() != DeviceType::kDeviceCUDA) {
        std::cerr << "[Fatal Error] rope_cuda expects CUDA Tensors!" << std::endl;
        return;
    }
    if (q->tensor_data_type() != k->tensor_data_type()) {
        std::cerr << "[hxinfer] rope_cuda: q and k must have the same dtype" << std::endl;
        return;
    }
    const int head_dim = config.dim / config.head;
    const int kv_head = config.kv_head > 0 ? config.kv_head : config.head;
    const int rows = static_cast<int>(q->tensor_total_elements() / (size_t)(config.head * head_dim));
    const hx_rope_table* t = detail::rope_table(config, base, head_dim, step + 1);
    if (!t) {
        std::cerr << "[hxinfer] rope_cuda: " << hx_last_error() << std::endl;
        return;
    }
    int rc = hx_rope_qk(q->raw_data_ptr(), k->raw_data_ptr(), hx_dtype_of(q->tensor_data_type()),
                        rows, config.head, kv_head, head_dim, step, t, nullptr);
    if (rc != HX_OK) std::cerr << "[hxinfer] rope_cuda: " << hx_last_error() << std::endl;
}

void attention_score_cuda(const std::shared_ptr<Tensor>& q, const std::shared_ptr<Tensor>& curr_k,
                          const std::shared_ptr<Tensor>& curr_v, std::shared_ptr<Tensor>& k_cache,
                          std::shared_ptr<Tensor>& v_cache, std::shared_ptr<Tensor>& output,
                          ModelConfig& config, int pos)
{
    for (const Tensor* t : {q.get(), curr_k.get(), curr_v.get(), k_cache.get(), v_cache.get(),
                            output.get()}) {
        if (t->tensor_device_type() != DeviceType::kDeviceCUDA) {
            std::cerr << "[hxinfer] attention_score_cuda expects CUDA Tensors!" << std::endl;
            return;
        }
    }
    const int dim = config.dim, head = config.head;
    const int head_dim = dim / head;
    const int kv_head = config.kv_head > 0 ? config.kv_head : head;
    const int kv_dim = kv_head * head_dim;
    const auto& shp = k_cache->tensor_shapes();
    const int rows = shp.size() >= 2 ? shp[0] : static_cast<int>(k_cache->tensor_total_elements() / kv_dim);
    if ((size_t)rows * kv_dim * 2 > k_cache->tensor_total_byte_size() ||
        (size_t)rows * kv_dim * 2 > v_cache->tensor_total_byte_size()) {
        std::cerr << "[hxinfer] attention_score_cuda: cache tensors too small" << std::endl;
        return;
    }
    hx_kv_cache* kv = detail::wrapped_cache(k_cache->raw_data_ptr(), v_cache->raw_data_ptr(),
                                            kv_head, head_dim, rows);
    const int32_t* r = detail::ramp(pos + 2);
    if (!kv || !r) {
        std::cerr << "[hxinfer] attention_score_cuda: " << hx_last_error() << std::endl;
        return;
    }
    const size_t ws_bytes = hx_decode_workspace_bytes(kv, 1, head);
    const float scale = 1.0f / sqrtf(static_cast<float>(head_dim));
    const int q_dt = hx_dtype_of(q->tensor_data_type()), k_dt = hx_dtype_of(curr_k->tensor_data_type());
    if (head_dim == 128 && q_dt == k_dt && head / kv_head <= 16) {
        // the append and the attention in one launch (q and k already
        // rotated by rope_tensor: no table, no bias)
        const hx_append_spec a{curr_k->raw_data_ptr(), curr_v->raw_data_ptr(), nullptr, nullptr,
                               nullptr, k_dt, nullptr};
        const int rc = hx_append_decode_attention(kv, 0, q->raw_data_ptr(), &a, r, r + pos + 1, 1,
                                                  head, scale, output->raw_data_ptr(),
                                                  hx_dtype_of(output->tensor_data_type()),
                                                  detail::workspace(ws_bytes), ws_bytes, nullptr);
        if (rc != HX_OK) std::cerr << "[hxinfer] attention_score_cuda: " << hx_last_error() << std::endl;
        return;
    }
    // append (the caller already rotated q and k with rope_tensor)
    int rc = hx_rope_append(kv, 0, nullptr, curr_k->raw_data_ptr(), curr_v->raw_data_ptr(),
                            hx_dtype_of(curr_k->tensor_data_type()), nullptr, nullptr, nullptr, r,
                            r + pos, 1, head, nullptr, nullptr, HX_FP16, nullptr);
    if (rc == HX_OK) {
        void* ws = detail::workspace(ws_bytes);
        rc = hx_decode_attention(kv, 0, q->raw_data_ptr(), hx_dtype_of(q->tensor_data_type()), r,
                                 r + pos + 1, 1, head, scale, output->raw_data_ptr(),
                                 hx_dtype_of(output->tensor_data_type()), ws, ws_bytes, nullptr);
    }
    if (rc != HX_OK) std::cerr << "[hxinfer] attention_score_cuda: " << hx_last_error() << std::endl;
}

}  // namespace hxinfer
