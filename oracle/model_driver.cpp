// model_driver.cpp — runs the reference engine's CausalLMModel end to end
// (test infrastructure only).
//
// Loads a model directory with the reference's DenseModelLoader
// (model_loaders/src/dense_model_loader.cpp:20-158) and feeds it one token
// per CausalLMModel::forward call (causal_lm_model.cpp:4-12), as the
// reference's drivers do (demos/bench_1024.cpp:60-70): the input is a
// one-element tensor holding the token id, the output the fp32 logits.
// oracle/Makefile compiles this file twice:
//   model_ref    the reference engine as it is (its own AttentionLayer,
//                rope and attention kernels, CPU tensors and allocators);
//   model_b200   the same engine sources with the hot-path headers replaced
//                by this build's (HX_DROPIN defined), linked against
//                libhxinfer.so / libhxkv.so: the drop-in a maintainer makes.
// Both write the logits of every position, so the two runs compare row by
// row.  model_b200 then checks PrefixCacheManager at model level: it stores
// the first `prefix` positions, overwrites them by running other tokens at
// those positions, restores, and runs the remaining tokens again; those
// logits are appended to the output and must equal the first run's.
//
// usage: model_driver <model_dir> <llama|qwen2> <tokens> <out.bin> [prefix]
#include <cuda_runtime.h>

#include <cstdio>
#include <cstdlib>
#include <memory>
#include <string>
#include <vector>

#include "base/allocator.h"
#include "base/config.h"
#include "dense_model_loader.h"
#include "tensor/tensor.h"
#ifdef HX_DROPIN
#include "cache/prefix_cache.h"
#endif

using namespace hxinfer;

static int token_at(int i, int vocab, int salt) { return (int)((i * 7919L + 13 + salt * 104729L) % vocab); }

int main(int argc, char** argv)
{
    if (argc < 5) {
        std::fprintf(stderr, "usage: %s <model_dir> <llama|qwen2> <tokens> <out.bin> [prefix]\n", argv[0]);
        return 2;
    }
    const std::string dir = argv[1];
    const ModelType type = std::string(argv[2]) == "qwen2" ? ModelType::Qwen2 : ModelType::LLaMA;
    const int n = std::atoi(argv[3]);
    const int prefix = argc > 5 ? std::atoi(argv[5]) : 0;

    auto cpu_alloc = std::make_shared<CPUAllocator>();
    auto cuda_alloc = std::make_shared<CUDAAllocator>();
    ModelConfig config;
    auto model = DenseModelLoader::load(dir, config, cpu_alloc, cuda_alloc, type);
    const int vocab = config.vocab_size;

    auto in_cpu = std::make_shared<Tensor>(cpu_alloc, std::vector<int>{1}, DataType::kDataTypeFP32);
    auto in_gpu = std::make_shared<Tensor>(cuda_alloc, std::vector<int>{1}, DataType::kDataTypeFP32);
    auto logits = std::make_shared<Tensor>(cuda_alloc, std::vector<int>{1, vocab}, DataType::kDataTypeFP32);
    in_gpu->tensor_set_device_type(DeviceType::kDeviceCUDA);
    logits->tensor_set_device_type(DeviceType::kDeviceCUDA);

    FILE* out = std::fopen(argv[4], "wb");
    if (!out) {
        std::perror(argv[4]);
        return 1;
    }
    std::vector<float> row(vocab);
    auto step = [&](int token, int pos, bool keep) -> bool {
        in_cpu->tensor_data_ptr<int>()[0] = token;
        cudaMemcpy(in_gpu->raw_data_ptr(), in_cpu->raw_data_ptr(), sizeof(int), cudaMemcpyHostToDevice);
        model->forward(in_gpu, logits, pos);
        if (!keep) return true;
        if (cudaMemcpy(row.data(), logits->raw_data_ptr(), vocab * sizeof(float), cudaMemcpyDeviceToHost) !=
            cudaSuccess)
            return false;
        return std::fwrite(row.data(), sizeof(float), vocab, out) == (size_t)vocab;
    };

    for (int i = 0; i < n; ++i)
        if (!step(token_at(i, vocab, 0), i, true)) {
            std::fprintf(stderr, "forward %d failed: %s\n", i, cudaGetErrorString(cudaGetLastError()));
            return 1;
        }
#ifdef HX_DROPIN
    if (prefix > 0 && prefix < n) {
        std::vector<int> toks(prefix);
        for (int i = 0; i < prefix; ++i) toks[i] = token_at(i, vocab, 0);
        PrefixCacheManager mgr(cpu_alloc, config);
        mgr.store(toks, *model);
        if (mgr.lookup(toks) != prefix) {
            std::fprintf(stderr, "prefix lookup missed\n");
            return 1;
        }
        for (int i = 0; i < prefix; ++i) step(token_at(i, vocab, 1), i, false);  // other tokens
        mgr.restore(toks, *model);
        for (int i = prefix; i < n; ++i)
            if (!step(token_at(i, vocab, 0), i, true)) return 1;
    }
#else
    (void)prefix;
#endif
    std::fclose(out);
    const cudaError_t e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
        std::fprintf(stderr, "device error: %s\n", cudaGetErrorString(e));
        return 1;
    }
    std::printf("model_driver: %d positions of %d logits written\n", n, vocab);
    return 0;
}
