// test_common.h — helpers shared by the C++ GPU tests: check counters and
// macros, CUDA tensors from host vectors, fp16 rounding, seeded fp16-exact
// normals, the attention tolerance, and exact signed-permutation weights.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <iostream>
#include <memory>
#include <random>
#include <vector>

#include "base/allocator.h"
#include "base/config.h"
#include "tensor/tensor.h"

using namespace hxinfer;

static int g_pass = 0, g_fail = 0;

#define CHECK_NEAR(actual, expected, tol, name)                                                 \
    do {                                                                                        \
        double _a = (actual), _e = (expected);                                                  \
        if (std::fabs(_a - _e) < (tol)) {                                                       \
            g_pass++;                                                                           \
        } else {                                                                                \
            std::cout << "  FAIL: " << name << " (got=" << _a << ", exp=" << _e << ")" << std::endl; \
            g_fail++;                                                                           \
        }                                                                                       \
    } while (0)

#define CHECK_TRUE(cond, name)                                       \
    do {                                                             \
        if (cond) {                                                  \
            g_pass++;                                                \
        } else {                                                     \
            std::cout << "  FAIL: " << name << std::endl;            \
            g_fail++;                                                \
        }                                                            \
    } while (0)

static std::shared_ptr<Allocator> cuda_alloc = std::make_shared<CUDAAllocator>();

static std::shared_ptr<Tensor> cuda_f32(const std::vector<float>& data, std::vector<int> shape)
{
    auto t = std::make_shared<Tensor>(cuda_alloc, shape, DataType::kDataTypeFP32);
    t->tensor_set_device_type(DeviceType::kDeviceCUDA);
    cudaMemcpy(t->raw_data_ptr(), data.data(), data.size() * sizeof(float), cudaMemcpyHostToDevice);
    return t;
}

static std::shared_ptr<Tensor> cuda_f16(const std::vector<float>& data, std::vector<int> shape)
{
    auto t = std::make_shared<Tensor>(cuda_alloc, shape, DataType::kDataTypeFP16);
    t->tensor_set_device_type(DeviceType::kDeviceCUDA);
    std::vector<__half> h(data.size());
    for (size_t i = 0; i < data.size(); i++) h[i] = __float2half_rn(data[i]);
    cudaMemcpy(t->raw_data_ptr(), h.data(), h.size() * sizeof(__half), cudaMemcpyHostToDevice);
    return t;
}

static std::vector<float> read_f32(const std::shared_ptr<Tensor>& t)
{
    std::vector<float> h(t->tensor_total_elements());
    cudaMemcpy(h.data(), t->raw_data_ptr(), h.size() * sizeof(float), cudaMemcpyDeviceToHost);
    return h;
}

static float r16(float x) { return __half2float(__float2half_rn(x)); }

static std::vector<float> normal_f16(std::mt19937_64& g, size_t n, float scale = 1.0f)
{
    std::normal_distribution<float> d(0.0f, scale);
    std::vector<float> v(n);
    for (auto& x : v) x = r16(d(g));
    return v;
}

static bool close(float got, float want) { return std::fabs(got - want) <= 2e-3 + 1e-2 * std::fabs(want); }

static std::vector<float> signed_perm(int n, std::mt19937_64& g)
{
    std::vector<int> p(n);
    for (int i = 0; i < n; i++) p[i] = i;
    std::shuffle(p.begin(), p.end(), g);
    const float vals[4] = {-2.0f, -1.0f, 0.5f, 1.0f};
    std::vector<float> w((size_t)n * n, 0.0f);
    for (int i = 0; i < n; i++) w[(size_t)i * n + p[i]] = vals[g() % 4];
    return w;
}

static std::vector<float> matvec(const std::vector<float>& w, const std::vector<float>& x, int n_out)
{
    const int n_in = static_cast<int>(x.size());
    std::vector<float> y(n_out, 0.0f);
    for (int i = 0; i < n_out; i++)
        for (int k = 0; k < n_in; k++) y[i] += w[(size_t)i * n_in + k] * x[k];
    return y;
}
