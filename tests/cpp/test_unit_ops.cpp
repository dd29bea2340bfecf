// test_unit_ops.cpp — the reference's operator tests, run through this
// build's C++ interface (the kept rope_tensor / attention_score_cuda /
// AttentionLayer / PrefixCacheManager), plus parity against the CPU oracle.
//
// The first two tests restate hxinfer's tests/unit/test_unit_ops.cpp:197-229
// (RoPE) and :292-319 (attention) with the same inputs, constants and
// tolerances.  Exit status = number of failed checks.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <iostream>
#include <random>
#include <vector>

#include "base/allocator.h"
#include "base/config.h"
#include "cache/prefix_cache.h"
#include "hx_kv.h"
#include "hx_oracle.h"
#include "layer/attention.h"
#include "op/math_ops.h"
#include "tensor/tensor.h"
#include "test_common.h"

// ---- tests/unit/test_unit_ops.cpp:197-229
static void test_rope()
{
    std::cout << "=== test_rope ===" << std::endl;
    ModelConfig config{};
    config.dim = 4;
    config.head = 1;
    config.kv_head = 1;
    config.rope_theta = 10000.0f;
    std::vector<float> q_data = {1.0, 2.0, 3.0, 4.0};
    auto q = cuda_f32(q_data, {4});
    auto k = cuda_f32(q_data, {4});
    rope_tensor(q, k, config, 0, 10000.0f);
    auto q_out = read_f32(q);
    CHECK_NEAR(q_out[0], 1.0f, 1e-5, "rope pos=0 Q[0]=1.0 (identity)");
    CHECK_NEAR(q_out[1], 2.0f, 1e-5, "rope pos=0 Q[1]=2.0 (identity)");
    CHECK_NEAR(q_out[2], 3.0f, 1e-5, "rope pos=0 Q[2]=3.0 (identity)");
    CHECK_NEAR(q_out[3], 4.0f, 1e-5, "rope pos=0 Q[3]=4.0 (identity)");
    auto q2 = cuda_f32(q_data, {4});
    auto k2 = cuda_f32(q_data, {4});
    rope_tensor(q2, k2, config, 1, 10000.0f);
    auto q2_out = read_f32(q2);
    CHECK_NEAR(q2_out[0], -1.9841f, 1e-3, "rope pos=1 Q[0]=-1.9841");
    CHECK_NEAR(q2_out[2], 2.4624f, 1e-3, "rope pos=1 Q[2]=2.4624");
}

// ---- tests/unit/test_unit_ops.cpp:292-319
static void test_attention()
{
    std::cout << "=== test_attention_score ===" << std::endl;
    ModelConfig config{};
    config.dim = 2;
    config.head = 1;
    config.kv_head = 1;
    config.seq_len = 10;
    auto q = cuda_f32({1, 0}, {1, 2});
    auto curr_k = cuda_f32({1, 0}, {1, 2});
    auto curr_v = cuda_f32({5, 10}, {1, 2});
    auto k_cache = std::make_shared<Tensor>(cuda_alloc, std::vector<int>{10, 2}, DataType::kDataTypeFP32);
    auto v_cache = std::make_shared<Tensor>(cuda_alloc, std::vector<int>{10, 2}, DataType::kDataTypeFP32);
    auto out = std::make_shared<Tensor>(cuda_alloc, std::vector<int>{1, 2}, DataType::kDataTypeFP32);
    k_cache->tensor_set_device_type(DeviceType::kDeviceCUDA);
    v_cache->tensor_set_device_type(DeviceType::kDeviceCUDA);
    out->tensor_set_device_type(DeviceType::kDeviceCUDA);
    attention_score_cuda(q, curr_k, curr_v, k_cache, v_cache, out, config, 0);
    auto r = read_f32(out);
    CHECK_NEAR(r[0], 5.0f, 1e-3, "attn pos=0 out[0]=5");
    CHECK_NEAR(r[1], 10.0f, 1e-3, "attn pos=0 out[1]=10");
}

// rope_tensor on the Qwen2.5-7B shape equals the oracle (rope_cpu) bit for bit.
static void test_rope_bit_exact()
{
    std::cout << "=== test_rope_bit_exact (28/4 heads, theta 1e6) ===" << std::endl;
    std::mt19937_64 g(3);
    ModelConfig config{};
    config.dim = 28 * 128;
    config.head = 28;
    config.kv_head = 4;
    for (int step : {0, 5, 1024, 32768}) {
        auto qh = normal_f16(g, 28 * 128), kh = normal_f16(g, 4 * 128);
        auto q = cuda_f32(qh, {1, 28 * 128});
        auto k = cuda_f32(kh, {1, 4 * 128});
        rope_tensor(q, k, config, step, 1e6f);
        auto qg = read_f32(q), kg = read_f32(k);
        orc_rope_neox(qh.data(), 1, 28 * 128, 28, 128, step, 1e6f);
        orc_rope_neox(kh.data(), 1, 4 * 128, 4, 128, step, 1e6f);
        CHECK_TRUE(std::memcmp(qg.data(), qh.data(), qh.size() * 4) == 0, "rope q bit-exact step " << step);
        CHECK_TRUE(std::memcmp(kg.data(), kh.data(), kh.size() * 4) == 0, "rope k bit-exact step " << step);
    }
}

// attention_score_cuda over a growing GQA cache (Qwen 28/4 heads) vs the oracle.
static void test_attention_score_gqa()
{
    std::cout << "=== test_attention_score_gqa (28/4 heads, 300 steps) ===" << std::endl;
    const int Hq = 28, Hkv = 4, hd = 128, steps = 300, dim = Hq * hd, kv_dim = Hkv * hd;
    ModelConfig config{};
    config.dim = dim;
    config.head = Hq;
    config.kv_head = Hkv;
    config.seq_len = 512;
    std::mt19937_64 g(4);
    auto k_cache = std::make_shared<Tensor>(cuda_alloc, std::vector<int>{512, kv_dim}, DataType::kDataTypeFP32);
    auto v_cache = std::make_shared<Tensor>(cuda_alloc, std::vector<int>{512, kv_dim}, DataType::kDataTypeFP32);
    k_cache->tensor_set_device_type(DeviceType::kDeviceCUDA);
    v_cache->tensor_set_device_type(DeviceType::kDeviceCUDA);
    auto out = std::make_shared<Tensor>(cuda_alloc, std::vector<int>{1, dim}, DataType::kDataTypeFP32);
    std::vector<float> K, V;
    int bad = 0;
    for (int pos = 0; pos < steps; pos++) {
        auto qh = normal_f16(g, dim), kh = normal_f16(g, kv_dim), vh = normal_f16(g, kv_dim);
        K.insert(K.end(), kh.begin(), kh.end());
        V.insert(V.end(), vh.begin(), vh.end());
        auto q = cuda_f32(qh, {1, dim});
        auto ck = cuda_f32(kh, {1, kv_dim});
        auto cv = cuda_f32(vh, {1, kv_dim});
        attention_score_cuda(q, ck, cv, k_cache, v_cache, out, config, pos);
        if (pos % 37 == 0 || pos == steps - 1) {
            auto got = read_f32(out);
            std::vector<float> want(dim);
            orc_decode_attention(qh.data(), K.data(), V.data(), pos + 1, Hq, Hkv, hd, want.data());
            for (int i = 0; i < dim; i++) bad += !close(got[i], want[i]);
        }
    }
    CHECK_TRUE(bad == 0, "attention_score_cuda GQA within 2e-3 + 1e-2*|ref| (" << bad << " bad)");
}

// AttentionLayer::forward (fused bias+RoPE+append, decode) vs the oracle, with
// exact signed-permutation projections so only the attention path is compared.
// fp16_weights: the q/k/v/o weights are fp16 tensors (the reference's model
// weights), which takes the fused projection (hx_qkv_rope_append); the
// signed-permutation values are exact in fp16, so the comparison is unchanged.
static void test_attention_layer(int Hq, int Hkv, bool bias, bool fp16_weights = false)
{
    std::cout << "=== test_attention_layer (" << Hq << "/" << Hkv << " heads, bias " << bias
              << ", fp16 weights " << fp16_weights << ") ===" << std::endl;
    const int hd = 128, dim = Hq * hd, kv_dim = Hkv * hd, npos = 70;
    std::mt19937_64 g(100 + Hq + Hkv + bias);
    ModelConfig config{};
    config.dim = dim;
    config.head = Hq;
    config.kv_head = Hkv;
    config.seq_len = 128;
    config.rope_theta = 1e6f;
    config.weight_dtype = DataType::kDataTypeFP32;
    config.activation_dtype = DataType::kDataTypeFP32;
    auto wq_h = signed_perm(dim, g), wo_h = signed_perm(dim, g);
    auto wk_full = signed_perm(dim, g), wv_full = signed_perm(dim, g);
    std::vector<float> wk_h(wk_full.begin(), wk_full.begin() + (size_t)kv_dim * dim);
    std::vector<float> wv_h(wv_full.begin(), wv_full.begin() + (size_t)kv_dim * dim);
    auto wmake = fp16_weights ? cuda_f16 : cuda_f32;
    auto wq = wmake(wq_h, {dim, dim}), wk = wmake(wk_h, {kv_dim, dim});
    auto wv = wmake(wv_h, {kv_dim, dim}), wo = wmake(wo_h, {dim, dim});
    std::vector<float> bq_h(dim, 0.0f), bk_h(kv_dim, 0.0f), bv_h(kv_dim, 0.0f);
    if (bias) {
        bq_h = normal_f16(g, dim, 0.02f);
        bk_h = normal_f16(g, kv_dim, 0.02f);
        bv_h = normal_f16(g, kv_dim, 0.02f);
    }
    auto bq = cuda_f32(bq_h, {dim}), bk = cuda_f32(bk_h, {kv_dim}), bv = cuda_f32(bv_h, {kv_dim});
    std::unique_ptr<AttentionLayer> layer =
        bias ? std::make_unique<AttentionLayer>(cuda_alloc, config, wq, wk, wv, wo, bq, bk, bv)
             : std::make_unique<AttentionLayer>(cuda_alloc, config, wq, wk, wv, wo);
    auto out = std::make_shared<Tensor>(cuda_alloc, std::vector<int>{1, dim}, DataType::kDataTypeFP32);
    out->tensor_set_device_type(DeviceType::kDeviceCUDA);
    std::vector<float> K, V;
    int bad = 0;
    for (int pos = 0; pos < npos; pos++) {
        auto x = normal_f16(g, dim);
        auto in = cuda_f32(x, {1, dim});
        layer->forward(in, out, pos);
        auto q = matvec(wq_h, x, dim), k = matvec(wk_h, x, kv_dim), v = matvec(wv_h, x, kv_dim);
        for (int i = 0; i < dim; i++) q[i] += bq_h[i];
        for (int i = 0; i < kv_dim; i++) {
            k[i] += bk_h[i];
            v[i] += bv_h[i];
        }
        orc_rope_neox(q.data(), 1, dim, Hq, hd, pos, 1e6f);
        orc_rope_neox(k.data(), 1, kv_dim, Hkv, hd, pos, 1e6f);
        for (int i = 0; i < kv_dim; i++) {
            K.push_back(r16(k[i]));
            V.push_back(r16(v[i]));
        }
        std::vector<float> a(dim);
        orc_decode_attention(q.data(), K.data(), V.data(), pos + 1, Hq, Hkv, hd, a.data());
        auto want = matvec(wo_h, a, dim);
        auto got = read_f32(out);
        for (int i = 0; i < dim; i++) bad += !close(got[i], want[i]);
    }
    CHECK_TRUE(bad == 0, "AttentionLayer::forward within 2e-3 + 1e-2*|ref| (" << bad << " bad)");
}

// A model-shaped holder: get_blocks()[i]->get_attention(), as LlamaModel has.
struct Block {
    std::shared_ptr<AttentionLayer> attn;
    std::shared_ptr<AttentionLayer>& get_attention() { return attn; }
};
struct MiniModel {
    std::vector<std::shared_ptr<Block>> blocks;
    std::vector<std::shared_ptr<Block>>& get_blocks() { return blocks; }
};

static std::vector<uint16_t> read_cache(const std::shared_ptr<Tensor>& t)
{
    std::vector<uint16_t> h(t->tensor_total_byte_size() / 2);
    cudaMemcpy(h.data(), t->raw_data_ptr(), t->tensor_total_byte_size(), cudaMemcpyDeviceToHost);
    return h;
}

// PrefixCacheManager semantics of prefix_cache.h:58-151 on device caches.
static void test_prefix_cache()
{
    std::cout << "=== test_prefix_cache (2 layers, 4/2 heads) ===" << std::endl;
    const int Hq = 4, Hkv = 2, hd = 128, dim = Hq * hd, kv_dim = Hkv * hd, seq_len = 96;
    const int n_fill = 80, plen = 67;
    std::mt19937_64 g(9);
    ModelConfig config{};
    config.dim = dim;
    config.head = Hq;
    config.kv_head = Hkv;
    config.layer = 2;
    config.seq_len = seq_len;
    config.rope_theta = 1e4f;
    config.weight_dtype = DataType::kDataTypeFP32;
    config.activation_dtype = DataType::kDataTypeFP32;
    MiniModel model;
    std::vector<std::shared_ptr<Tensor>> keep;
    for (int l = 0; l < 2; l++) {
        auto wq = cuda_f32(normal_f16(g, (size_t)dim * dim, 0.05f), {dim, dim});
        auto wk = cuda_f32(normal_f16(g, (size_t)kv_dim * dim, 0.05f), {kv_dim, dim});
        auto wv = cuda_f32(normal_f16(g, (size_t)kv_dim * dim, 0.05f), {kv_dim, dim});
        auto wo = cuda_f32(normal_f16(g, (size_t)dim * dim, 0.05f), {dim, dim});
        keep.insert(keep.end(), {wq, wk, wv, wo});
        auto b = std::make_shared<Block>();
        b->attn = std::make_shared<AttentionLayer>(cuda_alloc, config, wq, wk, wv, wo);
        model.blocks.push_back(b);
    }
    auto out = std::make_shared<Tensor>(cuda_alloc, std::vector<int>{1, dim}, DataType::kDataTypeFP32);
    out->tensor_set_device_type(DeviceType::kDeviceCUDA);
    auto run = [&](int from, int to) {
        for (int pos = from; pos < to; pos++) {
            auto in = cuda_f32(normal_f16(g, dim), {1, dim});
            for (auto& b : model.blocks) b->attn->forward(in, out, pos);
        }
    };
    run(0, n_fill);
    std::vector<std::vector<uint16_t>> snapK, snapV;
    for (auto& b : model.blocks) {
        snapK.push_back(read_cache(b->attn->get_k_cache()));
        snapV.push_back(read_cache(b->attn->get_v_cache()));
    }
    std::vector<int> prefix(plen), probe;
    for (int i = 0; i < plen; i++) prefix[i] = static_cast<int>(g() % 152064);
    probe = prefix;
    probe.back() += 1;
    PrefixCacheManager mgr(std::make_shared<DeviceAllocator>(), config);
    mgr.store(prefix, model);
    run(0, n_fill);  // overwrite every cached position with new values
    std::vector<std::vector<uint16_t>> overK, overV;
    for (auto& b : model.blocks) {
        overK.push_back(read_cache(b->attn->get_k_cache()));
        overV.push_back(read_cache(b->attn->get_v_cache()));
    }
    CHECK_TRUE(mgr.lookup(prefix) == plen, "lookup(prefix) == prefix_len");
    CHECK_TRUE(mgr.lookup(probe) == 0, "lookup(other tokens) == 0");
    CHECK_TRUE(mgr.cache_size() == 1, "cache_size() == 1");
    mgr.restore(probe, model);  // miss: prints, changes nothing
    for (int l = 0; l < 2; l++)
        CHECK_TRUE(read_cache(model.blocks[l]->attn->get_k_cache()) == overK[l], "miss leaves K alone");
    mgr.restore(prefix, model);
    // head-major [kv_head][seq_len][hd]: positions < plen come back, the rest stay
    for (int l = 0; l < 2; l++) {
        auto k = read_cache(model.blocks[l]->attn->get_k_cache());
        auto v = read_cache(model.blocks[l]->attn->get_v_cache());
        bool ok = true;
        for (int h = 0; h < Hkv; h++)
            for (int p = 0; p < seq_len; p++)
                for (int d = 0; d < hd; d++) {
                    size_t i = ((size_t)h * seq_len + p) * hd + d;
                    const auto& wk = p < plen ? snapK[l] : overK[l];
                    const auto& wv = p < plen ? snapV[l] : overV[l];
                    ok = ok && k[i] == wk[i] && v[i] == wv[i];
                }
        CHECK_TRUE(ok, "restore: first prefix_len positions restored, later untouched (layer " << l << ")");
    }
}

int main()
{
    test_rope();
    test_attention();
    test_rope_bit_exact();
    test_attention_score_gqa();
    test_attention_layer(4, 4, false);
    test_attention_layer(28, 4, true);
    test_attention_layer(28, 4, true, true);
    test_attention_layer(8, 8, false, true);
    test_prefix_cache();
    cudaError_t e = cudaDeviceSynchronize();
    int st = hx_device_status(1);
    CHECK_TRUE(e == cudaSuccess, "no CUDA error (" << cudaGetErrorString(e) << ")");
    CHECK_TRUE(st == HX_OK, "device status ok (" << hx_status_string(st) << ")");
    std::cout << "passed " << g_pass << ", failed " << g_fail << std::endl;
    return g_fail;
}
