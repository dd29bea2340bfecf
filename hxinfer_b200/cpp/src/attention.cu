// attention.cu — AttentionLayer over the C ABI
// (reference: hxinfer-engine/src/layer/attention.cpp:13-88, include/layer/attention.h:35-102).
#include <cublas_v2.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <iostream>
#include <stdexcept>

#include "device_context.h"
#include "layer/attention.h"

namespace hxinfer {

namespace {

__global__ void f32_to_f16_kernel(const float* __restrict__ x, __half* __restrict__ y, int64_t n)
{
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
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
    allocator_ = allocator;
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
    project_rows(w, x->raw_data_ptr(), x->tensor_data_type(), y->raw_data_ptr(), y->tensor_data_type(),
                 1, K, N, x16_);
}

// rows x K activations times the [n_out][K] weight: one cublasGemmEx,
// column-major view y^T[n_out][rows] = W[n_out][K] . x^T[K][rows].
void AttentionLayer::project_rows(const std::shared_ptr<Tensor>& w, const void* x, DataType xt,
                                  void* y, DataType yt, int rows, int K, int n_out,
                                  const std::shared_ptr<Tensor>& x16)
{
    if (w->tensor_total_elements() != (size_t)n_out * K)
        throw std::runtime_error("AttentionLayer: weight shape does not match");
    cublasHandle_t h = detail::cublas();
    if (!h) throw std::runtime_error("AttentionLayer: cuBLAS handle");
    const float one = 1.0f, zero = 0.0f;
    const DataType wt = w->tensor_data_type();
    const void* xp = x;
    cudaDataType_t xct;
    if (wt == DataType::kDataTypeFP16) {
        if (xt == DataType::kDataTypeFP32) {  // weights fp16, activations fp32
            const int64_t n = (int64_t)rows * K;
            if (x16->tensor_total_elements() < (size_t)n)
                throw std::runtime_error("AttentionLayer: fp16 staging too small");
            f32_to_f16_kernel<<<(unsigned)((n + 255) / 256), 256>>>(static_cast<const float*>(x),
                                                                   x16->tensor_data_ptr<__half>(), n);
            xp = x16->raw_data_ptr();
        }
        xct = CUDA_R_16F;
    } else if (wt == DataType::kDataTypeFP32 && xt == DataType::kDataTypeFP32) {
        xct = CUDA_R_32F;
    } else {
        throw std::runtime_error("AttentionLayer: unsupported weight/activation dtypes");
    }
    const cudaDataType_t wct = wt == DataType::kDataTypeFP16 ? CUDA_R_16F : CUDA_R_32F;
    const cudaDataType_t yct = yt == DataType::kDataTypeFP16 ? CUDA_R_16F : CUDA_R_32F;
    cublasStatus_t st = cublasGemmEx(h, CUBLAS_OP_T, CUBLAS_OP_N, n_out, rows, K, &one, w->raw_data_ptr(),
                                     wct, K, xp, xct, K, &zero, y, yct, n_out, CUBLAS_COMPUTE_32F,
                                     CUBLAS_GEMM_DEFAULT);
    if (st != CUBLAS_STATUS_SUCCESS) throw std::runtime_error("AttentionLayer: cublasGemmEx failed");
}

void AttentionLayer::reserve_rows(int n)
{
    if (n <= rows_cap_) return;
    int cap = 64;
    while (cap < n) cap *= 2;
    cap = std::min(cap, config_.seq_len);
    const int dim = config_.dim;
    const int kv_dim = config_.kv_head * (dim / config_.head);
    q_n_ = make(allocator_, {cap, dim}, activation_dtype_);
    k_n_ = make(allocator_, {cap, kv_dim}, activation_dtype_);
    v_n_ = make(allocator_, {cap, kv_dim}, activation_dtype_);
    q16_n_ = make(allocator_, {cap, dim}, DataType::kDataTypeFP16);
    attn_n_ = make(allocator_, {cap, dim}, activation_dtype_);
    x16_n_ = make(allocator_, {cap, std::max(dim, kv_dim)}, DataType::kDataTypeFP16);
    for (auto* t : {&q_n_, &k_n_, &v_n_, &q16_n_, &attn_n_, &x16_n_})
        if (!(*t)->raw_data_ptr()) throw std::runtime_error("AttentionLayer: scratch allocation failed");
    rows_cap_ = cap;
}

void AttentionLayer::forward(std::shared_ptr<Tensor>& input, std::shared_ptr<Tensor>& output, int pos)
{
    if (input->tensor_device_type() != DeviceType::kDeviceCUDA || !kv_)
        throw std::runtime_error("AttentionLayer: the B200 build runs on CUDA tensors only");
    const size_t elems = input->tensor_total_elements();
    if (config_.dim <= 0 || elems == 0 || elems % (size_t)config_.dim)
        throw std::runtime_error("AttentionLayer: input is not [n, dim]");
    if (output->tensor_total_elements() != elems)
        throw std::runtime_error("AttentionLayer: output must hold as many elements as the input");
    const size_t n = elems / (size_t)config_.dim;
    if (pos < 0 || (size_t)pos + n > (size_t)config_.seq_len)
        throw std::runtime_error("AttentionLayer: pos outside the cache");
    if (n > 1) {
        forward_tokens(input, output, pos, static_cast<int>(n));
        return;
    }
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
    } else if (head_dim == 128 && config_.kv_head > 0 && config_.head / config_.kv_head <= 16) {
        // other weight dtypes: cuBLAS projections as the reference, then bias
        // + RoPE + append + attention in one launch
        project(wq_, input, curr_q_);
        project(wk_, input, curr_k_);
        project(wv_, input, curr_v_);
        const hx_append_spec a{curr_k_->raw_data_ptr(), curr_v_->raw_data_ptr(),
                               has_bias_ ? bq_->raw_data_ptr() : nullptr,
                               has_bias_ ? bk_->raw_data_ptr() : nullptr,
                               has_bias_ ? bv_->raw_data_ptr() : nullptr, at, table};
        const size_t ws_bytes = hx_decode_workspace_bytes(kv_, 1, config_.head);
        void* ws = detail::workspace(ws_bytes);
        rc = hx_append_decode_attention(kv_, 0, curr_q_->raw_data_ptr(), &a, r, r + pos + 1, 1,
                                        config_.head, 1.0f / sqrtf(static_cast<float>(head_dim)),
                                        after_qktv_->raw_data_ptr(), at, ws, ws_bytes, nullptr);
        if (rc != HX_OK) throw std::runtime_error(std::string("AttentionLayer: ") + hx_last_error());
        project(wo_, after_qktv_, output);
        return;
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

// n > 1 tokens of sequence 0 at positions pos .. pos+n-1 (the caller checked
// pos + n <= seq_len).
void AttentionLayer::forward_tokens(std::shared_ptr<Tensor>& input, std::shared_ptr<Tensor>& output,
                                    int pos, int n)
{
    const int dim = config_.dim, hq = config_.head, head_dim = dim / hq;
    const int kv_dim = config_.kv_head * head_dim;
    const int32_t* r = detail::ramp(pos + n + 1);  // positions r + pos, lengths r + pos + 1
    const int32_t* seq0 = detail::zeros(n);
    const hx_rope_table* table = detail::rope_table(config_, config_.rope_theta, head_dim, pos + n);
    if (!r || !seq0 || !table) throw std::runtime_error(std::string("AttentionLayer: ") + hx_last_error());
    reserve_rows(n);
    const int at = hx_dtype_of(activation_dtype_);
    const DataType in_t = input->tensor_data_type();
    const bool fp16_weights = wq_->tensor_data_type() == DataType::kDataTypeFP16 &&
                              wk_->tensor_data_type() == DataType::kDataTypeFP16 &&
                              wv_->tensor_data_type() == DataType::kDataTypeFP16;
    const void* bq = has_bias_ ? bq_->raw_data_ptr() : nullptr;
    const void* bk = has_bias_ ? bk_->raw_data_ptr() : nullptr;
    const void* bv = has_bias_ ? bv_->raw_data_ptr() : nullptr;
    int rc;
    if (fp16_weights && head_dim == 128 && dim % 8 == 0 && dim <= 8192 && n <= 8 &&
        (in_t == DataType::kDataTypeFP16 || in_t == DataType::kDataTypeFP32)) {
        // up to one token group: the fused projection reads each weight once
        rc = hx_qkv_rope_append(kv_, 0, input->raw_data_ptr(), hx_dtype_of(in_t), dim,
                                wq_->raw_data_ptr(), wk_->raw_data_ptr(), wv_->raw_data_ptr(), at, bq, bk,
                                bv, seq0, r + pos, n, hq, table, q16_n_->raw_data_ptr(), HX_FP16, nullptr);
    } else {
        const void* x = input->raw_data_ptr();
        DataType xt = in_t;
        if (fp16_weights && in_t == DataType::kDataTypeFP32) {  // one fp16 copy for the three GEMMs
            const int64_t m = (int64_t)n * dim;
            f32_to_f16_kernel<<<(unsigned)((m + 255) / 256), 256>>>(input->tensor_data_ptr<float>(),
                                                                   x16_n_->tensor_data_ptr<__half>(), m);
            x = x16_n_->raw_data_ptr();
            xt = DataType::kDataTypeFP16;
        }
        project_rows(wq_, x, xt, q_n_->raw_data_ptr(), activation_dtype_, n, dim, dim, x16_n_);
        project_rows(wk_, x, xt, k_n_->raw_data_ptr(), activation_dtype_, n, dim, kv_dim, x16_n_);
        project_rows(wv_, x, xt, v_n_->raw_data_ptr(), activation_dtype_, n, dim, kv_dim, x16_n_);
        rc = hx_rope_append(kv_, 0, q_n_->raw_data_ptr(), k_n_->raw_data_ptr(), v_n_->raw_data_ptr(), at, bq,
                            bk, bv, seq0, r + pos, n, hq, table, q16_n_->raw_data_ptr(), HX_FP16, nullptr);
    }
    const float scale = 1.0f / sqrtf(static_cast<float>(head_dim));
    if (rc == HX_OK && head_dim == 128) {
        rc = hx_prefill_attention(kv_, 0, q16_n_->raw_data_ptr(), 0, pos, n, hq, scale,
                                  attn_n_->raw_data_ptr(), at, nullptr);
    } else if (rc == HX_OK) {
        // no tcgen05 prefill for this head size: one decode call per token
        // over positions [0, pos + i] (the layer's cache holds one sequence,
        // so the rows cannot go into one call as separate sequences)
        const size_t ws_bytes = hx_decode_workspace_bytes(kv_, 1, hq);
        void* ws = detail::workspace(ws_bytes);
        const size_t out_row = (size_t)dim * DataTypeSize(activation_dtype_);
        const char* q16 = static_cast<const char*>(q16_n_->raw_data_ptr());
        char* attn = static_cast<char*>(attn_n_->raw_data_ptr());
        for (int i = 0; i < n && rc == HX_OK; ++i)
            rc = hx_decode_attention(kv_, 0, q16 + (size_t)i * dim * 2, HX_FP16, seq0, r + pos + 1 + i, 1, hq,
                                     scale, attn + i * out_row, at, ws, ws_bytes, nullptr);
    }
    if (rc != HX_OK) throw std::runtime_error(std::string("AttentionLayer: ") + hx_last_error());
    project_rows(wo_, attn_n_->raw_data_ptr(), activation_dtype_, output->raw_data_ptr(),
                 output->tensor_data_type(), n, dim, dim, x16_n_);
}

}  // namespace hxinfer
