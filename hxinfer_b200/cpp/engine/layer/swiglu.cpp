// SwigluLayer for n rows (declared in layer/swiglu.h).  The operator calls
// are the reference's (swiglu.cpp:20-42): fused gate/up for one row when
// enabled, else gate GEMM, SiLU, up GEMM, multiply; then the down GEMM.
#include "layer/swiglu.h"

#include "../rows.h"

namespace hxinfer {

SwigluLayer::SwigluLayer(std::shared_ptr<Allocator> allocator, ModelConfig& config,
                         std::shared_ptr<Tensor>& w_gate, std::shared_ptr<Tensor>& w_up,
                         std::shared_ptr<Tensor>& w_down)
    : Layer("Swiglu"), allocator_(allocator), w_gate_(w_gate), w_up_(w_up), w_down_(w_down), config_(config)
{
    gate_proj_ = std::make_shared<LinearLayer>(w_gate_);
    up_proj_ = std::make_shared<LinearLayer>(w_up_);
    down_proj_ = std::make_shared<LinearLayer>(w_down_);
    rows(1);
}

void SwigluLayer::rows(int n)
{
    if (n > cap_rows_) {
        cap_rows_ = grown_rows(n, config_.seq_len);
        alloc_rows(allocator_, after_gate_, cap_rows_, config_.hidden_dim, config_.activation_dtype);
        alloc_rows(allocator_, after_up_, cap_rows_, config_.hidden_dim, config_.activation_dtype);
    }
    after_gate_->tensor_reshape({n, config_.hidden_dim});
    after_up_->tensor_reshape({n, config_.hidden_dim});
}

void SwigluLayer::forward(std::shared_ptr<Tensor>& input, std::shared_ptr<Tensor>& output)
{
    const int n = static_cast<int>(input->tensor_total_elements() / config_.dim);
    rows(n);
    if (n == 1 && use_fused_ && input->tensor_device_type() == DeviceType::kDeviceCUDA) {
        matmul_gate_up_cuda(input, w_gate_, w_up_, after_gate_, after_up_);
        silu_tensor(after_gate_, after_gate_);
        mul_tensor(after_gate_, after_up_, after_gate_);
    } else {
        gate_proj_->forward(input, after_gate_);
        silu_tensor(after_gate_, after_gate_);
        up_proj_->forward(input, after_up_);
        mul_tensor(after_gate_, after_up_, after_gate_);
    }
    down_proj_->forward(after_gate_, output);
}

}  // namespace hxinfer
