// TransformerLayer for n rows (declared in layer/transformer.h): the
// reference's step order (transformer.cpp:4-17) over [n, dim] buffers.
#include "layer/transformer.h"

#include "../rows.h"
#include "op/math_ops.h"

namespace hxinfer {

TransformerLayer::TransformerLayer(std::shared_ptr<Allocator> allocator, ModelConfig& modelConfig,
                                   std::shared_ptr<Tensor>& attn_norm_w, std::shared_ptr<Tensor>& wq,
                                   std::shared_ptr<Tensor>& wk, std::shared_ptr<Tensor>& wv,
                                   std::shared_ptr<Tensor>& wo, std::shared_ptr<Tensor>& ffn_norm_w,
                                   std::shared_ptr<Tensor>& w_gate, std::shared_ptr<Tensor>& w_up,
                                   std::shared_ptr<Tensor>& w_down, bool enable_fused)
    : Layer("Transformer"), config_(modelConfig)
{
    attentionLayer_ = std::make_shared<AttentionLayer>(allocator, config_, wq, wk, wv, wo);
    init(allocator, attn_norm_w, ffn_norm_w, w_gate, w_up, w_down);
    if (enable_fused) swigluLayer_->enable_fused();
}

TransformerLayer::TransformerLayer(std::shared_ptr<Allocator> allocator, ModelConfig& modelConfig,
                                   std::shared_ptr<Tensor>& attn_norm_w, std::shared_ptr<Tensor>& wq,
                                   std::shared_ptr<Tensor>& wk, std::shared_ptr<Tensor>& wv,
                                   std::shared_ptr<Tensor>& wo, std::shared_ptr<Tensor>& ffn_norm_w,
                                   std::shared_ptr<Tensor>& w_gate, std::shared_ptr<Tensor>& w_up,
                                   std::shared_ptr<Tensor>& w_down, bool enable_fused,
                                   std::shared_ptr<Tensor>& bq, std::shared_ptr<Tensor>& bk,
                                   std::shared_ptr<Tensor>& bv)
    : Layer("Transformer"), config_(modelConfig)
{
    attentionLayer_ = std::make_shared<AttentionLayer>(allocator, config_, wq, wk, wv, wo, bq, bk, bv);
    init(allocator, attn_norm_w, ffn_norm_w, w_gate, w_up, w_down);
    if (enable_fused) swigluLayer_->enable_fused();
}

TransformerLayer::TransformerLayer(std::shared_ptr<Allocator> allocator, ModelConfig& modelConfig,
                                   std::shared_ptr<Tensor>& attn_norm_w, std::shared_ptr<Tensor>& wq,
                                   std::shared_ptr<Tensor>& wk, std::shared_ptr<Tensor>& wv,
                                   std::shared_ptr<Tensor>& wo, std::shared_ptr<Tensor>& ffn_norm_w,
                                   std::shared_ptr<Tensor>& w_gate, std::shared_ptr<Tensor>& w_up,
                                   std::shared_ptr<Tensor>& w_down)
    : Layer("Transformer"), config_(modelConfig)
{
    attentionLayer_ = std::make_shared<AttentionLayer>(allocator, config_, wq, wk, wv, wo);
    init(allocator, attn_norm_w, ffn_norm_w, w_gate, w_up, w_down);
}

void TransformerLayer::init(std::shared_ptr<Allocator> allocator, std::shared_ptr<Tensor>& attn_norm_w,
                            std::shared_ptr<Tensor>& ffn_norm_w, std::shared_ptr<Tensor>& w_gate,
                            std::shared_ptr<Tensor>& w_up, std::shared_ptr<Tensor>& w_down)
{
    allocator_ = allocator;
    attn_norm_ = std::make_shared<RMSNormLayer>(attn_norm_w);
    ffn_norm_ = std::make_shared<RMSNormLayer>(ffn_norm_w);
    swigluLayer_ = std::make_shared<SwigluLayer>(allocator, config_, w_gate, w_up, w_down);
    rows(1);
}

void TransformerLayer::rows(int n)
{
    const int dim = config_.dim;
    if (n > cap_rows_) {
        cap_rows_ = grown_rows(n, config_.seq_len);
        for (auto* t : {&norm_out_, &attn_out_, &ffn_out_, &residual_})
            alloc_rows(allocator_, *t, cap_rows_, dim, config_.activation_dtype);
    }
    for (auto* t : {&norm_out_, &attn_out_, &ffn_out_, &residual_}) (*t)->tensor_reshape({n, dim});
}

void TransformerLayer::forward(std::shared_ptr<Tensor>& input, std::shared_ptr<Tensor>& output, int pos)
{
    rows(static_cast<int>(input->tensor_total_elements() / config_.dim));
    attn_norm_->forward(input, norm_out_);
    attentionLayer_->forward(norm_out_, attn_out_, pos);
    fused_add_rmsnorm_tensor(attn_out_, input, norm_out_, residual_, ffn_norm_->get_weight());
    swigluLayer_->forward(norm_out_, ffn_out_);
    add_tensor(residual_, ffn_out_, output);
}

}  // namespace hxinfer
