// layer/attention.h — AttentionLayer with the reference's constructors,
// forward(input, output, pos) and cache getters
// (hxinfer-engine/include/layer/attention.h:35-102).
//
// forward on CUDA tensors: with fp16 weights (head_dim 128, dim a multiple of
// 8 up to 8192) ONE launch does the q/k/v projections + optional bias + RoPE
// at `pos` + K/V append (hx_qkv_rope_append); otherwise cuBLAS GEMVs (as the
// reference) followed by one fused bias + RoPE + append launch
// (hx_rope_append).  Then split-K decode attention over pos+1 positions
// (hx_decode_attention), then the o projection.
//
// forward also takes n > 1 tokens at once (input and output [n, dim], tokens at
// positions pos .. pos+n-1; the reference takes one token per call): the
// projections become GEMMs (the fused launch for n <= 8), one bias + RoPE +
// append launch covers the n tokens, and causal prefill attention
// (hx_prefill_attention, tcgen05; head_dim 128) or, for other head sizes, one
// decode call per token replaces the per-token decode.  Row i equals what the
// i-th of n single-token calls returns, up to fp32 summation order and the
// rotated q being held in fp16 for the prefill kernel.
//
// The per-layer cache lives in k_cache_ / v_cache_ ([seq_len, kv_dim] fp16
// tensors, head-major inside) and is reached by PrefixCacheManager through
// get_k_cache()/get_v_cache() and kv_cache().
#ifndef HXINFER_B200_ATTENTION_H
#define HXINFER_B200_ATTENTION_H
#include <memory>
#include <stdexcept>

#include "base/allocator.h"
#include "base/config.h"
#include "hx_kv.h"
#include "layer/layer.h"
#include "tensor/tensor.h"

namespace hxinfer {

class AttentionLayer : public Layer {
public:
    AttentionLayer(std::shared_ptr<Allocator> allocator, ModelConfig& config,
                   std::shared_ptr<Tensor>& wq, std::shared_ptr<Tensor>& wk,
                   std::shared_ptr<Tensor>& wv, std::shared_ptr<Tensor>& wo);
    AttentionLayer(std::shared_ptr<Allocator> allocator, ModelConfig& config,
                   std::shared_ptr<Tensor>& wq, std::shared_ptr<Tensor>& wk,
                   std::shared_ptr<Tensor>& wv, std::shared_ptr<Tensor>& wo,
                   std::shared_ptr<Tensor>& bq, std::shared_ptr<Tensor>& bk,
                   std::shared_ptr<Tensor>& bv);
    ~AttentionLayer() override;

    void forward(std::shared_ptr<Tensor>& input, std::shared_ptr<Tensor>& output, int pos);
    void forward(std::shared_ptr<Tensor>&, std::shared_ptr<Tensor>&) override
    {
        throw std::runtime_error("AttentionLayer requires 'pos' parameter!\n");
    }

    std::shared_ptr<Tensor>& get_k_cache() { return k_cache_; }
    std::shared_ptr<Tensor>& get_v_cache() { return v_cache_; }
    // The cache handle over k_cache_/v_cache_ (for snapshots).
    hx_kv_cache* kv_cache() const { return kv_; }

private:
    void init(std::shared_ptr<Allocator> allocator);
    void project(const std::shared_ptr<Tensor>& w, const std::shared_ptr<Tensor>& x,
                 std::shared_ptr<Tensor>& y);
    // y[rows][n_out] = x[rows][k] W^T, W = w ([n_out][k] row-major); x16 holds
    // the fp16 copy of x when the weights are fp16 and x is fp32.
    void project_rows(const std::shared_ptr<Tensor>& w, const void* x, DataType x_dtype, void* y,
                      DataType y_dtype, int rows, int k, int n_out, const std::shared_ptr<Tensor>& x16);
    void forward_tokens(std::shared_ptr<Tensor>& input, std::shared_ptr<Tensor>& output, int pos,
                        int n);
    void reserve_rows(int n);

    ModelConfig config_;
    std::shared_ptr<Tensor> wq_, wk_, wv_, wo_;
    bool has_bias_ = false;
    std::shared_ptr<Tensor> bq_, bk_, bv_;
    std::shared_ptr<Tensor> curr_q_, curr_k_, curr_v_, q_rot_, x16_;
    std::shared_ptr<Tensor> k_cache_, v_cache_;
    std::shared_ptr<Tensor> after_qktv_;
    DataType activation_dtype_;
    hx_kv_cache* kv_ = nullptr;
    // scratch of multi-token calls, grown on demand
    std::shared_ptr<Allocator> allocator_;
    int rows_cap_ = 0;
    std::shared_ptr<Tensor> q_n_, k_n_, v_n_, q16_n_, attn_n_, x16_n_;
};

}  // namespace hxinfer
#endif
