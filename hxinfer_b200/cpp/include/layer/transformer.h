// layer/transformer.h — TransformerLayer with the reference's three
// constructors, get_attention and forward(input, output, pos)
// (hxinfer-engine/include/layer/transformer.h:8-99), for n rows.
//
// forward takes input/output [n, dim]: the tokens at positions
// pos .. pos+n-1 (the reference's buffers are [1, dim], one token per call).
// The step order is the reference's (transformer.cpp:4-17): RMSNorm,
// attention, fused residual add + RMSNorm, SwiGLU, residual add; each of the
// reference's operators already runs over all rows of its input, and the
// attention layer of this build prefills n rows with its tcgen05 kernel.
// The four [rows, dim] buffers grow on demand (powers of two, capped at
// seq_len rows).
#ifndef HXINFER_B200_TRANSFORMER_H
#define HXINFER_B200_TRANSFORMER_H
#include <stdexcept>

#include "attention.h"
#include "layer.h"
#include "rmsnorm.h"
#include "swiglu.h"

namespace hxinfer {

class TransformerLayer : public Layer {
public:
    TransformerLayer(std::shared_ptr<Allocator> allocator, ModelConfig& modelConfig,
                     std::shared_ptr<Tensor>& attn_norm_w, std::shared_ptr<Tensor>& wq,
                     std::shared_ptr<Tensor>& wk, std::shared_ptr<Tensor>& wv, std::shared_ptr<Tensor>& wo,
                     std::shared_ptr<Tensor>& ffn_norm_w, std::shared_ptr<Tensor>& w_gate,
                     std::shared_ptr<Tensor>& w_up, std::shared_ptr<Tensor>& w_down, bool enable_fused);
    TransformerLayer(std::shared_ptr<Allocator> allocator, ModelConfig& modelConfig,
                     std::shared_ptr<Tensor>& attn_norm_w, std::shared_ptr<Tensor>& wq,
                     std::shared_ptr<Tensor>& wk, std::shared_ptr<Tensor>& wv, std::shared_ptr<Tensor>& wo,
                     std::shared_ptr<Tensor>& ffn_norm_w, std::shared_ptr<Tensor>& w_gate,
                     std::shared_ptr<Tensor>& w_up, std::shared_ptr<Tensor>& w_down, bool enable_fused,
                     std::shared_ptr<Tensor>& bq, std::shared_ptr<Tensor>& bk, std::shared_ptr<Tensor>& bv);
    TransformerLayer(std::shared_ptr<Allocator> allocator, ModelConfig& modelConfig,
                     std::shared_ptr<Tensor>& attn_norm_w, std::shared_ptr<Tensor>& wq,
                     std::shared_ptr<Tensor>& wk, std::shared_ptr<Tensor>& wv, std::shared_ptr<Tensor>& wo,
                     std::shared_ptr<Tensor>& ffn_norm_w, std::shared_ptr<Tensor>& w_gate,
                     std::shared_ptr<Tensor>& w_up, std::shared_ptr<Tensor>& w_down);

    std::shared_ptr<AttentionLayer>& get_attention() { return attentionLayer_; }

    void forward(std::shared_ptr<Tensor>& input, std::shared_ptr<Tensor>& output, int pos);
    void forward(std::shared_ptr<Tensor>&, std::shared_ptr<Tensor>&) override
    {
        throw std::runtime_error("TransformerLayer requires 'pos' parameter!\n");
    }

private:
    void init(std::shared_ptr<Allocator> allocator, std::shared_ptr<Tensor>& attn_norm_w,
              std::shared_ptr<Tensor>& ffn_norm_w, std::shared_ptr<Tensor>& w_gate,
              std::shared_ptr<Tensor>& w_up, std::shared_ptr<Tensor>& w_down);
    void rows(int n);

    std::shared_ptr<RMSNormLayer> attn_norm_;
    std::shared_ptr<AttentionLayer> attentionLayer_;
    std::shared_ptr<RMSNormLayer> ffn_norm_;
    std::shared_ptr<SwigluLayer> swigluLayer_;
    std::shared_ptr<Allocator> allocator_;
    std::shared_ptr<Tensor> norm_out_, attn_out_, ffn_out_, residual_;
    int cap_rows_ = 0;
    ModelConfig config_;
};

}  // namespace hxinfer
#endif
