// CausalLMModel for n tokens per call (declared in model/causal_lm_model.h):
// embedding, the layers over [n, dim] rows (ping-pong buffers, as
// causal_lm_model.cpp:4-12), the final RMSNorm and lm_head on the last row,
// or on every row when the output holds n * vocab logits.
#include "model/causal_lm_model.h"

#include "../rows.h"
#include "op/math_ops.h"

namespace hxinfer {

CausalLMModel::CausalLMModel(std::shared_ptr<Allocator> allocator,
                             std::shared_ptr<EmbeddingLayer>& embeddingLayer,
                             std::vector<std::shared_ptr<TransformerLayer>>& block,
                             std::shared_ptr<RMSNormLayer>& final_norm, std::shared_ptr<LinearLayer>& lm_head,
                             ModelConfig& config)
    : Layer("CausalLMModel"),
      embeddingLayer_(embeddingLayer),
      blocks_(block),
      final_norm_(final_norm),
      lm_head_(lm_head),
      config_(config),
      activation_dtype_(config.activation_dtype),
      allocator_(allocator)
{
    rows(1);
}

void CausalLMModel::rows(int n)
{
    if (n > cap_rows_) {
        cap_rows_ = grown_rows(n, config_.seq_len);
        alloc_rows(allocator_, ping_, cap_rows_, config_.dim, activation_dtype_);
        alloc_rows(allocator_, pang_, cap_rows_, config_.dim, activation_dtype_);
    }
    ping_->tensor_reshape({n, config_.dim});
    pang_->tensor_reshape({n, config_.dim});
}

void CausalLMModel::forward(std::shared_ptr<Tensor>& input, std::shared_ptr<Tensor>& output, int pos)
{
    const int n = static_cast<int>(input->tensor_total_elements());
    if (n < 1) throw std::runtime_error("CausalLMModel::forward: no tokens");
    rows(n);
    embeddingLayer_->forward(input, ping_);
    for (auto& b : blocks_) {
        b->forward(ping_, pang_, pos);
        std::swap(ping_, pang_);
    }
    const size_t vocab = static_cast<size_t>(config_.vocab_size);
    if (n == 1 || output->tensor_total_elements() == n * vocab) {
        final_norm_->forward(ping_, ping_);
        lm_head_->forward(ping_, output);
        return;
    }
    // last row only: a view of ping_'s row n-1
    const size_t row_bytes = static_cast<size_t>(config_.dim) * DataTypeSize(activation_dtype_);
    auto last = std::make_shared<Tensor>(static_cast<char*>(ping_->raw_data_ptr()) + (n - 1) * row_bytes,
                                         std::vector<int>{1, config_.dim}, activation_dtype_,
                                         ping_->tensor_device_type());
    final_norm_->forward(last, last);
    lm_head_->forward(last, output);
}

}  // namespace hxinfer
