// test_layer_tokens.cpp — AttentionLayer::forward on n > 1 tokens per call
// (input/output [n, dim] at positions pos .. pos+n-1) against the CPU oracle
// of the reference's one-token-per-call loop (attention.cpp:13-88: q/k/v
// projections + bias, RoPE, append, attention over pos+1 positions, o
// projection, once per token).
//
// The projections use exact signed-permutation weights (as test_unit_ops.cpp
// does), so q/k/v are exact in any precision and the appended cache rows
// must equal the oracle's fp16 rows bit for bit; outputs are compared within
// the attention tolerance (2e-3 + 1e-2 |ref|).  Calls mix chunk sizes so that
// each path runs: n <= 8 with fp16 weights (fused projection), larger n
// (cuBLAS GEMMs), head_dim 128 (tcgen05 prefill) and 64 (one decode call per
// token), chunks crossing 64-position blocks, and a cache filled to a
// capacity that is not a multiple of 64.  Also PrefixCacheManager with host
// snapshots over caches filled that way.  Exit status = number of failures.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstring>
#include <iostream>
#include <stdexcept>
#include <string>
#include <vector>

#include "cache/prefix_cache.h"
#include "hx_oracle.h"
#include "layer/attention.h"
#include "test_common.h"

static std::vector<uint16_t> read_cache_bits(const std::shared_ptr<Tensor>& t)
{
    std::vector<uint16_t> h(t->tensor_total_byte_size() / 2);
    cudaMemcpy(h.data(), t->raw_data_ptr(), t->tensor_total_byte_size(), cudaMemcpyDeviceToHost);
    return h;
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

static void test_tokens(int Hq, int Hkv, int hd, bool bias, bool fp16_weights, int seq_len,
                        const std::vector<int>& chunks)
{
    std::cout << "=== test_tokens (" << Hq << "/" << Hkv << " heads x " << hd << ", bias " << bias
              << ", fp16 weights " << fp16_weights << ", seq_len " << seq_len << ") ===" << std::endl;
    const int dim = Hq * hd, kv_dim = Hkv * hd;
    std::mt19937_64 g(1000 + Hq * 7 + Hkv * 3 + hd + bias + 2 * fp16_weights);
    ModelConfig config{};
    config.dim = dim;
    config.head = Hq;
    config.kv_head = Hkv;
    config.seq_len = seq_len;
    config.rope_theta = 1e6f;
    config.weight_dtype = fp16_weights ? DataType::kDataTypeFP16 : DataType::kDataTypeFP32;
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

    std::vector<float> K, V;  // oracle cache rows [pos][kv_dim], fp16 values
    int pos = 0, bad = 0, calls_bad = 0;
    for (int n : chunks) {
        std::vector<float> x = normal_f16(g, (size_t)n * dim);
        auto in = cuda_f32(x, {n, dim});
        auto out = cuda_f32(std::vector<float>((size_t)n * dim, 0.0f), {n, dim});
        try {
            layer->forward(in, out, pos);
        } catch (const std::exception& e) {
            std::cout << "  forward(n=" << n << ", pos=" << pos << ") threw: " << e.what() << std::endl;
            calls_bad++;
            break;
        }
        auto got = read_f32(out);
        for (int t = 0; t < n; ++t) {
            const std::vector<float> xt(x.begin() + (size_t)t * dim, x.begin() + (size_t)(t + 1) * dim);
            auto q = matvec(wq_h, xt, dim), k = matvec(wk_h, xt, kv_dim), v = matvec(wv_h, xt, kv_dim);
            for (int i = 0; i < dim; i++) q[i] += bq_h[i];
            for (int i = 0; i < kv_dim; i++) {
                k[i] += bk_h[i];
                v[i] += bv_h[i];
            }
            orc_rope_neox(q.data(), 1, dim, Hq, hd, pos + t, 1e6f);
            orc_rope_neox(k.data(), 1, kv_dim, Hkv, hd, pos + t, 1e6f);
            for (int i = 0; i < kv_dim; i++) {
                K.push_back(r16(k[i]));
                V.push_back(r16(v[i]));
            }
            std::vector<float> a(dim);
            orc_decode_attention(q.data(), K.data(), V.data(), pos + t + 1, Hq, Hkv, hd, a.data());
            auto want = matvec(wo_h, a, dim);
            for (int i = 0; i < dim; i++) bad += !close(got[(size_t)t * dim + i], want[i]);
        }
        pos += n;
    }
    CHECK_TRUE(calls_bad == 0, "every multi-token forward returned");
    CHECK_TRUE(bad == 0, "rows within 2e-3 + 1e-2*|ref| of the one-token-per-call oracle (" << bad << " bad)");

    // the appended rows, head-major [kv_head][seq_len][hd] fp16 inside the cache tensors
    auto read_cache = [&](const std::shared_ptr<Tensor>& t) {
        std::vector<uint16_t> h(t->tensor_total_byte_size() / 2);
        cudaMemcpy(h.data(), t->raw_data_ptr(), t->tensor_total_byte_size(), cudaMemcpyDeviceToHost);
        return h;
    };
    auto kc = read_cache(layer->get_k_cache()), vc = read_cache(layer->get_v_cache());
    long cache_bad = 0;
    for (int p = 0; p < pos; ++p)
        for (int h = 0; h < Hkv; ++h)
            for (int d = 0; d < hd; ++d) {
                const size_t dev = ((size_t)h * seq_len + p) * hd + d, ref = (size_t)p * kv_dim + h * hd + d;
                const __half wk16 = __float2half_rn(K[ref]), wv16 = __float2half_rn(V[ref]);
                uint16_t bk16, bv16;
                std::memcpy(&bk16, &wk16, 2);
                std::memcpy(&bv16, &wv16, 2);
                cache_bad += (kc[dev] != bk16) + (vc[dev] != bv16);
            }
    CHECK_TRUE(cache_bad == 0, "appended K/V rows equal the oracle's fp16 rows (" << cache_bad << " differ)");
}

static void test_shape_errors()
{
    std::cout << "=== test_shape_errors ===" << std::endl;
    const int Hq = 2, hd = 128, dim = Hq * hd, seq_len = 100;
    std::mt19937_64 g(5);
    ModelConfig config{};
    config.dim = dim;
    config.head = Hq;
    config.kv_head = Hq;
    config.seq_len = seq_len;
    config.rope_theta = 1e4f;
    config.weight_dtype = DataType::kDataTypeFP32;
    config.activation_dtype = DataType::kDataTypeFP32;
    auto w = [&]() { return cuda_f32(signed_perm(dim, g), {dim, dim}); };
    auto wq = w(), wk = w(), wv = w(), wo = w();
    AttentionLayer layer(cuda_alloc, config, wq, wk, wv, wo);
    auto expect_throw = [&](int rows_in, int rows_out, int pos, const char* what) {
        auto in = cuda_f32(std::vector<float>((size_t)rows_in * dim, 0.5f), {rows_in, dim});
        auto out = cuda_f32(std::vector<float>((size_t)rows_out * dim, 0.0f), {rows_out, dim});
        bool threw = false;
        try {
            layer.forward(in, out, pos);
        } catch (const std::exception&) {
            threw = true;
        }
        CHECK_TRUE(threw, what);
    };
    expect_throw(3, 2, 0, "output with fewer rows than the input is refused");
    expect_throw(10, 10, 95, "pos + n past seq_len is refused");
    expect_throw(1, 1, seq_len, "pos == seq_len is refused");
    auto odd = cuda_f32(std::vector<float>(dim + 3, 0.5f), {dim + 3});
    auto odd_out = cuda_f32(std::vector<float>(dim + 3, 0.0f), {dim + 3});
    bool threw = false;
    try {
        layer.forward(odd, odd_out, 0);
    } catch (const std::exception&) {
        threw = true;
    }
    CHECK_TRUE(threw, "input that is not [n, dim] is refused");
}

// PrefixCacheManager given a CPUAllocator, as the reference's callers construct
// it (its snapshots are host tensors): snapshots stay in host memory and the
// restore semantics are the same as with device snapshots.  The caches are
// filled by multi-token forward calls.
static void test_prefix_cache_host_snapshots()
{
    std::cout << "=== test_prefix_cache_host_snapshots (2 layers, 4/2 heads) ===" << std::endl;
    const int Hq = 4, Hkv = 2, hd = 128, dim = Hq * hd, kv_dim = Hkv * hd, seq_len = 160;
    const int n_fill = 150, plen = 131;
    std::mt19937_64 g(17);
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
    auto fill = [&]() {  // positions 0 .. n_fill-1 in one call per layer
        auto in = cuda_f32(normal_f16(g, (size_t)n_fill * dim), {n_fill, dim});
        auto out = cuda_f32(std::vector<float>((size_t)n_fill * dim, 0.0f), {n_fill, dim});
        for (auto& b : model.blocks) b->attn->forward(in, out, 0);
    };
    fill();
    std::vector<std::vector<uint16_t>> snapK, snapV, overK, overV;
    for (auto& b : model.blocks) {
        snapK.push_back(read_cache_bits(b->attn->get_k_cache()));
        snapV.push_back(read_cache_bits(b->attn->get_v_cache()));
    }
    std::vector<int> prefix(plen);
    for (int i = 0; i < plen; i++) prefix[i] = static_cast<int>(g() % 152064);
    PrefixCacheManager mgr(std::make_shared<CPUAllocator>(), config);
    mgr.store(prefix, model);
    fill();  // overwrite every cached position
    for (auto& b : model.blocks) {
        overK.push_back(read_cache_bits(b->attn->get_k_cache()));
        overV.push_back(read_cache_bits(b->attn->get_v_cache()));
    }
    CHECK_TRUE(mgr.lookup(prefix) == plen && mgr.cache_size() == 1, "host snapshot stored and found");
    mgr.restore(prefix, model);
    for (int l = 0; l < 2; l++) {
        auto k = read_cache_bits(model.blocks[l]->attn->get_k_cache());
        auto v = read_cache_bits(model.blocks[l]->attn->get_v_cache());
        bool ok = true;
        for (int h = 0; h < Hkv; h++)
            for (int p = 0; p < seq_len; p++)
                for (int d = 0; d < hd; d++) {
                    const size_t i = ((size_t)h * seq_len + p) * hd + d;
                    const auto& wk = p < plen ? snapK[l] : overK[l];
                    const auto& wv = p < plen ? snapV[l] : overV[l];
                    ok = ok && k[i] == wk[i] && v[i] == wv[i];
                }
        CHECK_TRUE(ok, "host snapshot restore: first prefix_len positions back, later untouched (layer "
                           << l << ")");
    }
}

int main()
{
    // head_dim 128: fused projection for n <= 8 (fp16 weights), GEMMs above, tcgen05 prefill
    test_tokens(8, 2, 128, true, true, 4096, {1, 3, 8, 5, 64, 100, 1, 130, 2, 7});
    // MHA, fp32 weights: GEMMs for every n > 1
    test_tokens(4, 4, 128, false, false, 512, {2, 61, 1, 200, 9});
    // capacity 1000 (not a multiple of 64) filled to the last position
    test_tokens(4, 2, 128, true, true, 1000, {600, 399, 1});
    // head_dim 64: no tcgen05 prefill; one decode call per token
    test_tokens(4, 2, 64, true, true, 512, {1, 6, 70, 3, 150});
    test_shape_errors();
    test_prefix_cache_host_snapshots();
    cudaError_t e = cudaDeviceSynchronize();
    int st = hx_device_status(1);
    CHECK_TRUE(e == cudaSuccess, "no CUDA error (" << cudaGetErrorString(e) << ")");
    CHECK_TRUE(st == HX_OK, "device status ok (" << hx_status_string(st) << ")");
    std::cout << "passed " << g_pass << ", failed " << g_fail << std::endl;
    return g_fail;
}
