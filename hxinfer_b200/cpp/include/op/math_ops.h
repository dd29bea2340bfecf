// op/math_ops.h — the hot-path operators of the reference's operator API,
// declared exactly as in hxinfer-engine/include/op/math_ops.h:28-30,67-73.
//
//  * rope_tensor dispatches on the tensor's device: CUDA tensors go to
//    rope_cuda; CPU tensors are outside this build (rope_cpu throws).
//  * rope_cuda rotates q and k in place (NeoX, YaRN when config.rope_use_yarn);
//    the result equals the reference rope_cpu bit for bit.
//  * attention_score_cuda appends curr_k / curr_v at position `pos` of the
//    caller's k_cache / v_cache tensors and writes softmax(q K^T/sqrt(d)) V over
//    pos+1 positions to `output`.  The cache tensors are opaque storage: this
//    build keeps them head-major fp16 ([kv_head][rows][head_dim]) inside the
//    caller's allocation, `rows` being the tensor's first dimension.
//
// Errors follow the reference's CUDA ops: a message on std::cerr and return.
// Everything runs on the legacy default stream, as in the reference.
#ifndef HXINFER_B200_MATH_OPS_H
#define HXINFER_B200_MATH_OPS_H
#include <memory>

#include "tensor/tensor.h"

namespace hxinfer {

void rope_tensor(std::shared_ptr<Tensor>& q, std::shared_ptr<Tensor>& k, ModelConfig& config,
                 int step, float base = 10000);
void rope_cpu(std::shared_ptr<Tensor>& q, std::shared_ptr<Tensor>& k, ModelConfig& config,
              int step, float base = 10000);
void rope_cuda(std::shared_ptr<Tensor>& q, std::shared_ptr<Tensor>& k, ModelConfig& config,
               int step, float base = 10000);

void attention_score_cuda(const std::shared_ptr<Tensor>& q, const std::shared_ptr<Tensor>& curr_k,
                          const std::shared_ptr<Tensor>& curr_v, std::shared_ptr<Tensor>& k_cache,
                          std::shared_ptr<Tensor>& v_cache, std::shared_ptr<Tensor>& output,
                          ModelConfig& config, int pos);

}  // namespace hxinfer
#endif
