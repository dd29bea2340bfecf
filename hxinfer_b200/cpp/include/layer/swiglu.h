// layer/swiglu.h — SwigluLayer with the reference's constructor, enable_fused
// and forward (hxinfer-engine/include/layer/swiglu.h:6-31), for n rows.
//
// The reference sizes its two [seq_len, hidden_dim] activation buffers up
// front (swiglu.cpp:9-14: 2 x 180 MB per layer for LLaMA-2-7B in fp32) and
// its fused gate/up path, matmul_gate_up_cuda, is written for one row.  Here
// the buffers grow on demand (powers of two, capped at seq_len rows), one row
// keeps the reference's fused path when enabled, and n > 1 rows take the
// reference's unfused path (two GEMMs over the rows, SiLU, multiply).
#ifndef HXINFER_B200_SWIGLU_H
#define HXINFER_B200_SWIGLU_H
#include "layer.h"
#include "linear.h"

namespace hxinfer {

class SwigluLayer : public Layer {
public:
    SwigluLayer(std::shared_ptr<Allocator> allocator, ModelConfig& config, std::shared_ptr<Tensor>& w_gate,
                std::shared_ptr<Tensor>& w_up, std::shared_ptr<Tensor>& w_down);
    void enable_fused() { use_fused_ = true; }
    // input [n, dim] -> output [n, dim]
    void forward(std::shared_ptr<Tensor>& input, std::shared_ptr<Tensor>& output) override;

private:
    void rows(int n);

    std::shared_ptr<Allocator> allocator_;
    std::shared_ptr<Tensor> w_gate_, w_up_, w_down_;
    bool use_fused_ = false;
    std::shared_ptr<LinearLayer> gate_proj_, up_proj_, down_proj_;
    std::shared_ptr<Tensor> after_gate_, after_up_;
    int cap_rows_ = 0;
    ModelConfig config_;
};

}  // namespace hxinfer
#endif
