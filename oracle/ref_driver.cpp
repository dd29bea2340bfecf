// ref_driver.cpp — C entry points over the reference engine's own CPU code.
//
// TEST INFRASTRUCTURE ONLY.  Compiled by oracle/Makefile together with the
// reference sources where they lie (never copied) into oracle/_ref/libhxref.so.
// The tests use it to pin the C oracle (hx_oracle.c) and to produce the golden
// vectors under tests/golden/; the CPU benchmark arm times it.  Nothing in the
// product links it.
//
// Every wrapper builds reference Tensors on the reference CPUAllocator and
// calls the reference function unmodified:
//   rope_cpu            hxinfer-engine/src/op/cpu/rope_cpu.cpp:5-39
//   rope_cuda (YaRN)    hxinfer-engine/src/op/cuda/rope_cuda.cu:98-152, on a GPU
//   softmax_cpu         hxinfer-engine/src/op/cpu/softmax_cpu.cpp:6-46
//   AttentionLayer CPU  hxinfer-engine/src/layer/attention.cpp:37-88 (MHA only)
//   PrefixCacheManager  hxinfer-engine/include/cache/prefix_cache.h:16-155
#include <cuda_runtime.h>

#include <cstring>
#include <iostream>
#include <memory>
#include <unordered_map>
#include <vector>

#include "base/allocator.h"
#include "base/config.h"
#include "layer/attention.h"
#include "model/llama_model.h"
#include "op/math_ops.h"
#include "tensor/tensor.h"

// compute_hash is private in the reference class; expose it to this driver
// only, so the tests can pin the FNV-1a restatement against it.
#define private public
#include "cache/prefix_cache.h"
#undef private

using namespace hxinfer;

namespace {

std::shared_ptr<Allocator> cpu_alloc()
{
    static std::shared_ptr<Allocator> a = std::make_shared<CPUAllocator>();
    return a;
}

std::shared_ptr<Tensor> make_tensor(std::vector<int> shape, const float* src)
{
    auto t = std::make_shared<Tensor>(cpu_alloc(), shape, DataType::kDataTypeFP32);
    if (src) std::memcpy(t->raw_data_ptr(), src, t->tensor_total_byte_size());
    return t;
}

}  // namespace

extern "C" {

// RoPE over q [rows][head*head_dim] and k [rows][kv_head*head_dim] at `step`.
int ref_rope_cpu(float* q, float* k, int rows, int head, int kv_head, int head_dim,
                 int step, float base)
{
    try {
        ModelConfig cfg{};
        cfg.dim = head * head_dim;
        cfg.head = head;
        cfg.kv_head = kv_head;
        auto tq = make_tensor({rows, head * head_dim}, q);
        auto tk = make_tensor({rows, kv_head * head_dim}, k);
        rope_cpu(tq, tk, cfg, step, base);
        std::memcpy(q, tq->raw_data_ptr(), tq->tensor_total_byte_size());
        std::memcpy(k, tk->raw_data_ptr(), tk->tensor_total_byte_size());
        return 0;
    } catch (const std::exception& e) {
        std::cerr << "ref_rope_cpu: " << e.what() << std::endl;
        return 1;
    }
}

// The reference's rope_cuda (rope_cuda.cu:98-152) on one token row, on the
// current CUDA device: q [head*head_dim], k [kv_head*head_dim] fp32, rotated
// in place by the reference's own kernels, with its YaRN settings when
// use_yarn != 0 (multipliers rope_cuda.cu:13-30, attention factor :32-35).
// Returns 0, 1 on a C++ exception, 2 on a CUDA error.
int ref_rope_cuda(float* q, float* k, int head, int kv_head, int head_dim, int step, float base,
                  int use_yarn, float factor, float beta_fast, float beta_slow, int orig_max_pos)
{
    try {
        ModelConfig cfg{};
        cfg.dim = head * head_dim;
        cfg.head = head;
        cfg.kv_head = kv_head;
        cfg.rope_theta = base;
        cfg.rope_use_yarn = use_yarn != 0;
        cfg.rope_factor = factor;
        cfg.rope_beta_fast = beta_fast;
        cfg.rope_beta_slow = beta_slow;
        cfg.rope_orig_max_pos = orig_max_pos;
        auto cuda = std::make_shared<CUDAAllocator>();
        auto tq = std::make_shared<Tensor>(cuda, std::vector<int>{1, head * head_dim},
                                           DataType::kDataTypeFP32);
        auto tk = std::make_shared<Tensor>(cuda, std::vector<int>{1, kv_head * head_dim},
                                           DataType::kDataTypeFP32);
        const size_t qb = tq->tensor_total_byte_size(), kb = tk->tensor_total_byte_size();
        if (cudaMemcpy(tq->raw_data_ptr(), q, qb, cudaMemcpyHostToDevice) != cudaSuccess ||
            cudaMemcpy(tk->raw_data_ptr(), k, kb, cudaMemcpyHostToDevice) != cudaSuccess)
            return 2;
        rope_cuda(tq, tk, cfg, step, base);
        if (cudaDeviceSynchronize() != cudaSuccess) return 2;
        if (cudaMemcpy(q, tq->raw_data_ptr(), qb, cudaMemcpyDeviceToHost) != cudaSuccess ||
            cudaMemcpy(k, tk->raw_data_ptr(), kb, cudaMemcpyDeviceToHost) != cudaSuccess)
            return 2;
        return 0;
    } catch (const std::exception& e) {
        std::cerr << "ref_rope_cuda: " << e.what() << std::endl;
        return 1;
    }
}

int ref_softmax_cpu(const float* in, float* out, int n)
{
    try {
        auto ti = make_tensor({n}, in);
        auto to = make_tensor({n}, nullptr);
        softmax_cpu(ti, to);
        std::memcpy(out, to->raw_data_ptr(), sizeof(float) * (size_t)n);
        return 0;
    } catch (const std::exception& e) {
        std::cerr << "ref_softmax_cpu: " << e.what() << std::endl;
        return 1;
    }
}

// Runs the reference AttentionLayer on the CPU (its MHA-only branch) for
// positions 0..n_pos-1.  x: [n_pos][dim] inputs, weights [dim][dim] row-major
// (out = W x), out: [n_pos][dim].
int ref_attention_layer_cpu(int dim, int head, int seq_len, float theta, const float* wq,
                            const float* wk, const float* wv, const float* wo, const float* x,
                            int n_pos, float* out)
{
    try {
        ModelConfig cfg{};
        cfg.dim = dim;
        cfg.head = head;
        cfg.kv_head = head;
        cfg.seq_len = seq_len;
        cfg.rope_theta = theta;
        auto twq = make_tensor({dim, dim}, wq);
        auto twk = make_tensor({dim, dim}, wk);
        auto twv = make_tensor({dim, dim}, wv);
        auto two = make_tensor({dim, dim}, wo);
        AttentionLayer layer(cpu_alloc(), cfg, twq, twk, twv, two);
        auto tin = make_tensor({1, dim}, nullptr);
        auto tout = make_tensor({1, dim}, nullptr);
        for (int p = 0; p < n_pos; p++) {
            std::memcpy(tin->raw_data_ptr(), x + (size_t)p * dim, sizeof(float) * (size_t)dim);
            layer.forward(tin, tout, p);
            std::memcpy(out + (size_t)p * dim, tout->raw_data_ptr(), sizeof(float) * (size_t)dim);
        }
        return 0;
    } catch (const std::exception& e) {
        std::cerr << "ref_attention_layer_cpu: " << e.what() << std::endl;
        return 1;
    }
}

unsigned long long ref_prefix_hash(const int* tokens, int n)
{
    ModelConfig cfg{};
    PrefixCacheManager mgr(cpu_alloc(), cfg);
    return (unsigned long long)mgr.compute_hash(std::vector<int>(tokens, tokens + n));
}

// Builds a CPU LlamaModel of `layers` MHA layers and drives the reference
// PrefixCacheManager through store / lookup / restore.
//   init_kv, overwrite_kv, after_miss, after_restore: [layers][2][seq_len][dim]
//   hits[0] = lookup(prefix) after store, hits[1] = lookup(probe),
//   hits[2] = cache_size() after store.
int ref_prefix_cache_roundtrip(int layers, int dim, int head, int seq_len,
                               const float* init_kv, const float* overwrite_kv,
                               const int* prefix, int prefix_len, const int* probe,
                               int probe_len, float* after_miss, float* after_restore,
                               long long* hits)
{
    try {
        static ModelConfig cfg{};  // CausalLMModel keeps a reference to it
        cfg = ModelConfig{};
        cfg.dim = dim;
        cfg.hidden_dim = dim;
        cfg.layer = layers;
        cfg.head = head;
        cfg.kv_head = head;
        cfg.vocab_size = 4;
        cfg.seq_len = seq_len;
        auto a = cpu_alloc();
        std::vector<std::shared_ptr<TransformerLayer>> blocks;
        for (int l = 0; l < layers; l++) {
            auto n1 = make_tensor({dim}, nullptr), n2 = make_tensor({dim}, nullptr);
            auto wq = make_tensor({dim, dim}, nullptr), wk = make_tensor({dim, dim}, nullptr);
            auto wv = make_tensor({dim, dim}, nullptr), wo = make_tensor({dim, dim}, nullptr);
            auto wg = make_tensor({dim, dim}, nullptr), wu = make_tensor({dim, dim}, nullptr);
            auto wd = make_tensor({dim, dim}, nullptr);
            blocks.push_back(std::make_shared<TransformerLayer>(a, cfg, n1, wq, wk, wv, wo, n2, wg,
                                                                wu, wd));
        }
        auto emb = std::make_shared<EmbeddingLayer>(make_tensor({4, dim}, nullptr));
        auto fnorm = std::make_shared<RMSNormLayer>(make_tensor({dim}, nullptr));
        auto head_w = std::make_shared<LinearLayer>(make_tensor({4, dim}, nullptr));
        LlamaModel model(a, emb, blocks, fnorm, head_w, cfg);

        size_t plane = (size_t)seq_len * dim;
        auto load = [&](const float* src) {
            for (int l = 0; l < layers; l++) {
                auto& attn = model.get_blocks()[l]->get_attention();
                std::memcpy(attn->get_k_cache()->raw_data_ptr(), src + (2 * l + 0) * plane, plane * 4);
                std::memcpy(attn->get_v_cache()->raw_data_ptr(), src + (2 * l + 1) * plane, plane * 4);
            }
        };
        auto save = [&](float* dst) {
            for (int l = 0; l < layers; l++) {
                auto& attn = model.get_blocks()[l]->get_attention();
                std::memcpy(dst + (2 * l + 0) * plane, attn->get_k_cache()->raw_data_ptr(), plane * 4);
                std::memcpy(dst + (2 * l + 1) * plane, attn->get_v_cache()->raw_data_ptr(), plane * 4);
            }
        };

        PrefixCacheManager mgr(a, cfg);
        std::vector<int> pre(prefix, prefix + prefix_len), prb(probe, probe + probe_len);
        load(init_kv);
        mgr.store(pre, model);
        load(overwrite_kv);
        hits[0] = mgr.lookup(pre);
        hits[1] = mgr.lookup(prb);
        hits[2] = (long long)mgr.cache_size();
        mgr.restore(prb, model);  // a miss: the reference prints and leaves the caches alone
        save(after_miss);
        mgr.restore(pre, model);
        save(after_restore);
        return 0;
    } catch (const std::exception& e) {
        std::cerr << "ref_prefix_cache_roundtrip: " << e.what() << std::endl;
        return 1;
    }
}

}  // extern "C"
