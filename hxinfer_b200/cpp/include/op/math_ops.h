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
//
// The rest of the reference's operator API is declared below as well, with
// the reference's signatures, because this header replaces the reference's
// at the same path: the engine's other sources (op/*_tensor.cpp, op/cpu,
// op/cuda, the layers) keep defining and calling those operators.
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

// ---- implemented by the reference engine's own sources (not by this build)
using TensorPtr = std::shared_ptr<Tensor>;
void add_tensor(const TensorPtr& input_a, const TensorPtr& input_b, TensorPtr& output);
void add_cpu(const TensorPtr& input_a, const TensorPtr& input_b, TensorPtr& output);
void add_cuda(const TensorPtr& input_a, const TensorPtr& input_b, TensorPtr& output);
void mul_tensor(const TensorPtr& input_a, const TensorPtr& input_b, TensorPtr& output);
void mul_cpu(const TensorPtr& input_a, const TensorPtr& input_b, TensorPtr& output);
void mul_cuda(const TensorPtr& input_a, const TensorPtr& input_b, TensorPtr& output);
void softmax_tensor(const TensorPtr& input, TensorPtr& output);
void softmax_cpu(const TensorPtr& input, TensorPtr& output);
void softmax_cuda(const TensorPtr& input, TensorPtr& output);
void matmul_tensor(const TensorPtr& input, const TensorPtr& weight, TensorPtr& output);
void matmul_cpu(const TensorPtr& input, const TensorPtr& weight, TensorPtr& output);
void matmul_cuda(const TensorPtr& input, const TensorPtr& weight, TensorPtr& output);
void rmsnorm_tensor(const TensorPtr& input, const TensorPtr& weight, TensorPtr& output, float eps = 1e-5);
void rmsnorm_cpu(const TensorPtr& input, const TensorPtr& weight, TensorPtr& output, float eps = 1e-5);
void rmsnorm_cuda(const TensorPtr& input, const TensorPtr& weight, TensorPtr& output, float eps = 1e-5);
void embedding_tensor(const TensorPtr& token_ids, const TensorPtr& weight, TensorPtr& output);
void embedding_cpu(const TensorPtr& token_ids, const TensorPtr& weight, TensorPtr& output);
void embedding_cuda(const TensorPtr& token_ids, const TensorPtr& weight, TensorPtr& output);
void silu_tensor(const TensorPtr& input, TensorPtr& output);
void silu_cpu(const TensorPtr& input, TensorPtr& output);
void silu_cuda(const TensorPtr& input, TensorPtr& output);
int argmax_tensor(const TensorPtr& input);
int argmax_cpu(const TensorPtr& input);
int argmax_cuda(const TensorPtr& input);
int sample_tensor(const TensorPtr& logits, float temperature, float top_p);
void matmul_qkv_cuda(const TensorPtr& input, const TensorPtr& wq, const TensorPtr& wk,
                     const TensorPtr& wv, TensorPtr& q_out, TensorPtr& k_out, TensorPtr& v_out);
void matmul_gate_up_cuda(const TensorPtr& input, const TensorPtr& w_gate, const TensorPtr& w_up,
                         TensorPtr& gate_out, TensorPtr& up_out);
void fused_add_rmsnorm_cuda(TensorPtr& hidden_states, TensorPtr& residual, TensorPtr& hidden_out,
                            TensorPtr& residual_out, const TensorPtr& weight, float eps = 1e-5);
void fused_add_rmsnorm_tensor(TensorPtr& hidden_states, TensorPtr& residual, TensorPtr& hidden_out,
                              TensorPtr& residual_out, const TensorPtr& weight, float eps = 1e-5);

}  // namespace hxinfer
#endif
