// layer/layer.h — the reference's Layer base (hxinfer-engine/include/layer/layer.h:6-11).
#ifndef HXINFER_B200_LAYER_H
#define HXINFER_B200_LAYER_H
#include <memory>
#include <string>

#include "tensor/tensor.h"

namespace hxinfer {

class Layer {
public:
    std::string layer_name_;
    explicit Layer(std::string layer_name) : layer_name_(std::move(layer_name)) {}
    virtual void forward(std::shared_ptr<Tensor>& input, std::shared_ptr<Tensor>& output) = 0;
    virtual ~Layer() = default;
};

}  // namespace hxinfer
#endif
