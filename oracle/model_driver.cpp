// model_driver.cpp — runs the reference engine's CausalLMModel end to end
// (test infrastructure only).
//
// Loads a model directory with the reference's DenseModelLoader
// (model_loaders/src/dense_model_loader.cpp:20-158) and runs
// CausalLMModel::forward (causal_lm_model.cpp:4-12) over a fixed token
// sequence, the way the reference's drivers do (demos/bench_1024.cpp:60-70):
// the input tensor holds token ids, the output the fp32 logits.
// oracle/Makefile compiles this file twice:
//   model_ref    the reference engine as it is (its own AttentionLayer,
//                TransformerLayer, SwigluLayer and CausalLMModel, its rope
//                and attention kernels), one token per call;
//   model_b200   the same engine sources with the hot-path headers and the
//                n-row model classes replaced by this build's (HX_DROPIN),
//                linked against libhxinfer.so / libhxkv.so: the drop-in a
//                maintainer makes.  --chunk C feeds the prompt C tokens per
//                call (the layers then prefill with the tcgen05 kernel).
//
// usage: model_driver <model_dir> <llama|qwen2> <prompt> <out.bin | -> [options]
//   --chunk C    prompt tokens per forward call (default 1; model_b200 only)
//   --prefix P   model_b200: after the prompt, store the first P positions
//                with PrefixCacheManager, overwrite them by running other
//                tokens there, restore, and run positions P.. again one token
//                per call; those logits are appended to the output
//   --decode D   after the prompt, D single-token calls (timed; the per-token
//                figure excludes the first, which pays first-use set-up)
//   --warmup W   W untimed passes of the prompt (and two decode calls) first
// The logits of every position go to out.bin (fp32 [rows][vocab]) unless it
// is "-".  One JSON line on stdout gives the device time of the prompt pass
// and of the decode calls (CUDA events on the legacy default stream around
// the forward calls, host launch gaps included, as a caller sees them).
#include <cuda_runtime.h>

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
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
        std::fprintf(stderr, "usage: %s <model_dir> <llama|qwen2> <prompt> <out.bin|-> "
                             "[--chunk C] [--prefix P] [--decode D] [--warmup W]\n", argv[0]);
        return 2;
    }
    const std::string dir = argv[1];
    const ModelType type = std::string(argv[2]) == "qwen2" ? ModelType::Qwen2 : ModelType::LLaMA;
    const int prompt = std::atoi(argv[3]);
    const bool keep = std::strcmp(argv[4], "-") != 0;
    int chunk = 1, prefix = 0, decode = 0, warmup = 0;
    for (int a = 5; a + 1 < argc; a += 2) {
        if (!std::strcmp(argv[a], "--chunk")) chunk = std::atoi(argv[a + 1]);
        else if (!std::strcmp(argv[a], "--warmup")) warmup = std::atoi(argv[a + 1]);
        else if (!std::strcmp(argv[a], "--prefix")) prefix = std::atoi(argv[a + 1]);
        else if (!std::strcmp(argv[a], "--decode")) decode = std::atoi(argv[a + 1]);
        else {
            std::fprintf(stderr, "unknown option %s\n", argv[a]);
            return 2;
        }
    }
#ifndef HX_DROPIN
    if (chunk != 1 || prefix) {
        std::fprintf(stderr, "the reference engine takes one token per call and has no device prefix cache\n");
        return 2;
    }
#endif
    if (chunk < 1) chunk = 1;

    auto cpu_alloc = std::make_shared<CPUAllocator>();
    auto cuda_alloc = std::make_shared<CUDAAllocator>();
    ModelConfig config;
    auto model = DenseModelLoader::load(dir, config, cpu_alloc, cuda_alloc, type);
    const int vocab = config.vocab_size;

    FILE* out = keep ? std::fopen(argv[4], "wb") : nullptr;
    if (keep && !out) {
        std::perror(argv[4]);
        return 1;
    }
    std::vector<float> rows;
    // One forward call over tokens [pos, pos+n) of sequence `salt`; with `all`
    // the output holds every row's logits (n * vocab), else the last row's.
    struct Io {
        std::shared_ptr<Tensor> in_cpu, in_gpu, logits;
    };
    std::map<int, Io> io;  // by tokens per call, allocated once
    auto step = [&](int pos, int n, int salt, bool write) -> bool {
        const bool all = n > 1;
        Io& b = io[n];
        if (!b.in_cpu) {
            b.in_cpu = std::make_shared<Tensor>(cpu_alloc, std::vector<int>{n}, DataType::kDataTypeFP32);
            b.in_gpu = std::make_shared<Tensor>(cuda_alloc, std::vector<int>{n}, DataType::kDataTypeFP32);
            b.logits = std::make_shared<Tensor>(cuda_alloc, std::vector<int>{all ? n : 1, vocab},
                                                DataType::kDataTypeFP32);
            b.in_gpu->tensor_set_device_type(DeviceType::kDeviceCUDA);
            b.logits->tensor_set_device_type(DeviceType::kDeviceCUDA);
        }
        auto& in_cpu = b.in_cpu;
        auto& in_gpu = b.in_gpu;
        auto& logits = b.logits;
        for (int i = 0; i < n; ++i) in_cpu->tensor_data_ptr<int>()[i] = token_at(pos + i, vocab, salt);
        cudaMemcpy(in_gpu->raw_data_ptr(), in_cpu->raw_data_ptr(), n * sizeof(int), cudaMemcpyHostToDevice);
        model->forward(in_gpu, logits, pos);
        if (!write || !out) return true;
        rows.resize((size_t)n * vocab);
        if (cudaMemcpy(rows.data(), logits->raw_data_ptr(), rows.size() * sizeof(float),
                       cudaMemcpyDeviceToHost) != cudaSuccess)
            return false;
        return std::fwrite(rows.data(), sizeof(float), rows.size(), out) == rows.size();
    };
    // With one token per call every position's logits are written; with
    // chunks, each call writes all of its rows.
    // Untimed passes of the same calls (prompt, then two one-token calls):
    // first-use set-up (library handles, workspaces, kernel attributes) and
    // cold caches stay out of the timed pass, which rewrites the same
    // positions.
    for (int w = 0; w < warmup; ++w) {
        for (int pos = 0; pos < prompt; pos += chunk)
            if (!step(pos, std::min(chunk, prompt - pos), 0, false)) return 1;
        for (int t = 0; t < 2 && t < decode; ++t)
            if (!step(prompt + t, 1, 0, false)) return 1;
    }
    cudaEvent_t e0, e1, e2;
    cudaEventCreate(&e0);
    cudaEventCreate(&e1);
    cudaEventCreate(&e2);
    cudaEventRecord(e0, 0);
    for (int pos = 0; pos < prompt; pos += chunk) {
        const int n = std::min(chunk, prompt - pos);
        if (!step(pos, n, 0, true)) {
            std::fprintf(stderr, "forward at %d failed: %s\n", pos, cudaGetErrorString(cudaGetLastError()));
            return 1;
        }
    }
    cudaEventRecord(e1, 0);
    // The first decode call pays the one-token path's first-use set-up (after
    // a chunked prompt it is the first one-token call), so the per-token
    // figure is taken over the calls after it.
    cudaEvent_t e1b;
    cudaEventCreate(&e1b);
    for (int t = 0; t < decode; ++t) {
        if (!step(prompt + t, 1, 0, false)) return 1;
        if (t == 0) cudaEventRecord(e1b, 0);
    }
    if (decode == 0) cudaEventRecord(e1b, 0);
    cudaEventRecord(e2, 0);
    cudaEventSynchronize(e2);
    float prompt_ms = 0, first_decode_ms = 0, decode_ms = 0;
    cudaEventElapsedTime(&prompt_ms, e0, e1);
    cudaEventElapsedTime(&first_decode_ms, e1, e1b);
    cudaEventElapsedTime(&decode_ms, e1b, e2);
#ifdef HX_DROPIN
    if (prefix > 0 && prefix < prompt) {
        std::vector<int> toks(prefix);
        for (int i = 0; i < prefix; ++i) toks[i] = token_at(i, vocab, 0);
        PrefixCacheManager mgr(cpu_alloc, config);
        mgr.store(toks, *model);
        if (mgr.lookup(toks) != prefix) {
            std::fprintf(stderr, "prefix lookup missed\n");
            return 1;
        }
        for (int i = 0; i < prefix; ++i) step(i, 1, 1, false);  // other tokens at those positions
        mgr.restore(toks, *model);
        for (int i = prefix; i < prompt; ++i)
            if (!step(i, 1, 0, true)) return 1;
    }
    const char* build = "b200";
    const int status = hx_device_status(0);  // a kernel's recorded failure, HX_OK if none
#else
    const char* build = "ref";
    const int status = 0;
#endif
    if (out) std::fclose(out);
    const cudaError_t e = cudaDeviceSynchronize();
    if (status) std::fprintf(stderr, "device status %d: a kernel recorded a failure\n", status);
    if (e != cudaSuccess) {
        std::fprintf(stderr, "device error: %s\n", cudaGetErrorString(e));
        return 1;
    }
    std::printf("{\"build\": \"%s\", \"layers\": %d, \"dim\": %d, \"prompt\": %d, \"chunk\": %d, "
                "\"prompt_ms\": %.4f, \"decode_steps\": %d, \"first_decode_ms\": %.4f, "
                "\"decode_ms_per_token\": %.5f, \"device_status\": %d}\n",
                build, config.layer, config.dim, prompt, chunk, prompt_ms, decode, first_decode_ms,
                decode > 1 ? decode_ms / (decode - 1) : 0.0f, status);
    return status ? 1 : 0;
}
