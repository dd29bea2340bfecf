// model/causal_lm_model.h — CausalLMModel with the reference's constructor,
// forward(input, output, pos) and get_blocks
// (hxinfer-engine/include/model/causal_lm_model.h:11-51), for n tokens.
//
// forward(input, output, pos): input holds n token ids (the reference holds
// one), for positions pos .. pos+n-1; the layers run on [n, dim] rows, so a
// prompt is prefilled in one call.  output takes the logits of the last
// token ([1, vocab], as the reference) or, when it has n * vocab elements,
// of every token.  The reference's LlamaModel and Qwen2Model derive from this
// class unchanged.
#ifndef HXINFER_B200_CAUSAL_LM_MODEL_H
#define HXINFER_B200_CAUSAL_LM_MODEL_H
#include <stdexcept>
#include <vector>

#include "layer/embedding.h"
#include "layer/layer.h"
#include "layer/linear.h"
#include "layer/transformer.h"

namespace hxinfer {

class CausalLMModel : public Layer {
protected:
    std::shared_ptr<EmbeddingLayer> embeddingLayer_;
    std::vector<std::shared_ptr<TransformerLayer>> blocks_;
    std::shared_ptr<RMSNormLayer> final_norm_;
    std::shared_ptr<LinearLayer> lm_head_;
    std::shared_ptr<Tensor> ping_;
    std::shared_ptr<Tensor> pang_;
    ModelConfig& config_;
    DataType activation_dtype_;

public:
    CausalLMModel(std::shared_ptr<Allocator> allocator, std::shared_ptr<EmbeddingLayer>& embeddingLayer,
                  std::vector<std::shared_ptr<TransformerLayer>>& block,
                  std::shared_ptr<RMSNormLayer>& final_norm, std::shared_ptr<LinearLayer>& lm_head,
                  ModelConfig& config);

    void forward(std::shared_ptr<Tensor>& input, std::shared_ptr<Tensor>& output, int pos);

    std::vector<std::shared_ptr<TransformerLayer>>& get_blocks() { return blocks_; }

    void forward(std::shared_ptr<Tensor>&, std::shared_ptr<Tensor>&) override
    {
        throw std::runtime_error("CausalLMModel requires 'pos' parameter!");
    }

private:
    void rows(int n);

    std::shared_ptr<Allocator> allocator_;
    int cap_rows_ = 0;
};

}  // namespace hxinfer
#endif
