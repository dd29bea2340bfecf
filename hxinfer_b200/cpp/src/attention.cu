// attention.cu — AttentionLayer over the C ABI
// (reference: hxinfer-engine/src/layer/attention.cpp:13-88, include/layer/attention.h:35-102).
#include <cublas_v2.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cmath>
#include <iostream>
#include <stdexcept>

#include "device_context.h"
#include "layer/attention.h"

namespace hxinfer {

namespace {

__global__ void f32_to_f16_kernel(const float* __restrict__ x, __half* __restrict__ y, int n)
{
    int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) y[i] = __float2half_rn(x[i]);
}

int hx_dtype_of(DataType t)
{
    return t == DataType::kDataTypeFP16 ? HX_FP16 : (t == DataType::kDataTypeFP32 ? HX_FP32 : -1);
}

std::shared_ptr<Tensor> make(std::shared_ptr<Allocator>& a, std::vector<int> s, DataType t)
{
    auto x = std::make_shared<Tensor>(a, s, t);
    x->tensor_set_device_type(a->device_type());
    return x;
}

}  // namespace

AttentionLayer::AttentionLayer(std::shared_ptr<Allocator> allocator, ModelConfig& config,
                               std::shared_ptr<Tensor>& wq, std::shared_ptr<Tensor>& wk,
                               std::shared_ptr<Tensor>& wv, std::shared_ptr<Tensor>& wo)
    : Layer("Attention"), config_(config), wq_(wq), wk_(wk), wv_(wv), wo_(wo), has_bias_(false)
{
    init(allocator);
}

AttentionLayer::AttentionLayer(std::shared_ptr<Allocator> allocator, ModelConfig& config,
                               std::shared_ptr<Tensor>& wq, std::shared_ptr<Tensor>& wk,
                               std::shared_ptr<Tensor>& wv, std::shared_ptr<Tensor>& wo,
                               std::shared_ptr<Tensor>& bq, std::shared_ptr<Tensor>& bk,
                               std::shared_ptr<Tensor>& bv)
    : Layer("Attention"), config_(config), wq_(wq), wk_(wk), wv_(wv), wo_(wo), has_bias_(true),
      bq_(bq), bk_(bk), bv_(bv)
{
    init(allocator);
}

void AttentionLayer::init(std::shared_ptr<Allocator> allocator)
{
    const int dim = config_.dim;
    if (config_.kv_head <= 0) config_.kv_head = config_.head;
    const int kv_dim = config_.kv_head * (dim / config_.head);
    activation_dtype_ = config_.activation_dtype;
    curr_q_ = make(allocator, {1, dim}, activation_dtype_);
    curr_k_ = make(allocator, {1, kv_dim}, activation_dtype_);
    curr_v_ = make(allocator, {1, kv_dim}, activation_dtype_);
    q_rot_ = make(allocator, {1, dim}, activation_dtype_);
    after_qktv_ = make(allocator, {1, dim}, activation_dtype_);
    x16_ = make(allocator, {1, std::max(dim, kv_dim)}, DataType::kDataTypeFP16);
    // fp16 storage whatever the activation dtype
    k_cache_ = make(allocator, {config_.seq_len, kv_dim}, DataType::kDataTypeFP16);
    v_cache_ = make(allocator, {config_.seq_len, kv_dim}, DataType::kDataTypeFP16);
    if (allocator->device_type() == DeviceType::kDeviceCUDA) {
        int rc = hx_kv_wrap(k_cache_->raw_data_ptr(), v_cache_->raw_data_ptr(), config_.kv_head,
                            dim / config_.head, config_.seq_len, &kv_);
        if (rc != HX_OK) throw std::runtime_error(std::string("AttentionLayer: ") + hx_last_error());
    }
}

AttentionLayer::~AttentionLayer()
{
    if (kv_) hx_kv_destroy(kv_);
}

// y[N] = W[N][K] x[K] with cuBLAS (fp32 accumulation), the layout of the
// reference's Linear weights (out x in, row-major).
void AttentionLayer::project(const std::shared_ptr<Tensor>& w, const std::shared_ptr<Tensor>& x,
                             std::shared_ptr<Tensor>& y)
{
    const int K = static_cast<int>(x->tensor_total_elements());
    const int N = static_cast<int>(y->tensor_total_elements());
    if (w->tensor_total_elements() != (size_t)N * K)
        throw std::runtime_error("AttentionLayer: weight shape does not match");
    cublasHandle_t h = detail::cublas();
    if (!h) throw std::runtime_error("AttentionLayer: cuBLAS handle");
    const float one = 1.0f, zero = 0.0f;
    const DataType wt = w->tensor_data_type(), xt = x->tensor_data_type(), yt = y->tensor_data_type();
    const void* xp = x->raw_data_ptr();
    cudaDataType_t xct;
    if (wt == DataType::kDataTypeFP16) {
        if (xt == DataType::kDataTypeFP32) {  // weights fp16, activations fp32
            f32_to_f16_kernel<<<(K + 255) / 256, 256>>>(x->tensor_data_ptr<float>(),
                                                       x16_->tensor_data_ptr<__half>(), K);
            xp = x16_->raw_data_ptr();
        }
        xct = CUDA_R_16F;
    } else if (wt == DataType::kDataTypeFP32 && xt == DataType::kDataTypeFP32) {
        xct = CUDA_R_32F;
    } else {
        throw std::runtime_error("AttentionLayer: unsupported weight/activation dtypes");
    }
    const cudaDataType_t wct = wt == DataType::kDataTypeFP16 ? CUDA_R_16F : CUDA_R_32F;
    const cudaDataType_t yct = yt == DataType::kDataTypeFP16 ? CUDA_R_16F : CUDA_R_32F;
    cublasStatus_t st = cublasGemmEx(h, CUBLAS_OP_T, CUBLAS_OP_N, N, 1, K, &one, w->raw_data_ptr(),
                                     wct, K, xp, xct, K, &zero, y->raw_data_ptr(), yct, N,
                                     CUBLAS_COMPUTE_32F, CUBLAS_GEMM_DEFAULT);
    if (st != CUBLAS_STATUS_SUCCESS) throw std::runtime_error("AttentionLayer: cublasGemmEx failed");
}

void AttentionLayer::forward(std::shared_ptr<Tensor>& input, std::shared_ptr<Tensor>& output, int pos)
{
    if (input->tensor_device_type() != DeviceType::kDeviceCUDA || !kv_)
        throw std::runtime_error("AttentionLayer: the B200 build runs on CUDA tensors only");
    if (pos < 0 || pos >= config_.seq_len)
        throw std::runtime_error("AttentionLayer: pos outside the cache");
    const int head_dim = config_.dim / config_.head;
    const int32_t* r = detail::ramp(pos + 2);
    const hx_rope_table* table = detail::rope_table(config_, config_.rope_theta, head_dim, pos + 1);
    if (!r || !table) throw std::runtime_error(std::string("AttentionLayer: ") + hx_last_error());
    const int at = hx_dtype_of(activation_dtype_);
    const DataType in_t = input->tensor_data_type();
    const bool fp16_weights = wq_->tensor_data_type() == DataType::kDataTypeFP16 &&
                              wk_->tensor_data_type() == DataType::kDataTypeFP16 &&
                              wv_->tensor_data_type() == DataType::kDataTypeFP16;
    int rc;
    if (fp16_weights && head_dim == 128 && config_.dim % 8 == 0 && config_.dim <= 8192 &&
        (in_t == DataType::kDataTypeFP16 || in_t == DataType::kDataTypeFP32)) {
        // the reference's fp16-weight projection (matmul_qkv_cuda) fused with
        // bias + RoPE + append in one launch
        rc = hx_qkv_rope_append(kv_, 0, input->raw_data_ptr(), hx_dtype_of(in_t), config_.dim,
                                wq_->raw_data_ptr(), wk_->raw_data_ptr(), wv_->raw_data_ptr(), at,
                                has_bias_ ? bq_->raw_data_ptr() : nullptr,
                                has_bias_ ? bk_->raw_data_ptr() : nullptr,
                                has_bias_ ? bv_->raw_data_ptr() : nullptr, r, r + pos, 1,
                                config_.head, table, q_rot_->raw_data_ptr(), at, nullptr);
    } else {
        project(wq_, input, curr_q_);
        project(wk_, input, curr_k_);
        project(wv_, input, curr_v_);
        rc = hx_rope_append(kv_, 0, curr_q_->raw_data_ptr(), curr_k_->raw_data_ptr(),
                            curr_v_->raw_data_ptr(), at,
                            has_bias_ ? bq_->raw_data_ptr() : nullptr,
                            has_bias_ ? bk_->raw_data_ptr() : nullptr,
                            has_bias_ ? bv_->raw_data_ptr() : nullptr, r, r + pos, 1, config_.head,
                            table, q_rot_->raw_data_ptr(), at, nullptr);
    }
    if (rc == HX_OK) {
        const size_t ws_bytes = hx_decode_workspace_bytes(kv_, 1, config_.head);
        void* ws = detail::workspace(ws_bytes);
        rc = hx_decode_attention(kv_, 0, q_rot_->raw_data_ptr(), at, r, r + pos + 1, 1,
                                 config_.head, 1.0f / sqrtf(static_cast<float>(head_dim)),
                                 after_qktv_->raw_data_ptr(), at, ws, ws_bytes, nullptr);
    }
    if (rc != HX_OK) throw std::runtime_error(std::string("AttentionLayer: ") + hx_last_error());
    project(wo_, after_qktv_, output);
}

}  // namespace hxinfer
