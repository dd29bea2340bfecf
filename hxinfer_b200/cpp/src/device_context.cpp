// device_context.cpp — per-device shared state of the C++ operators.
#include "device_context.h"

#include <cuda_runtime.h>

#include <map>
#include <mutex>
#include <stdexcept>
#include <tuple>
#include <vector>

namespace hxinfer {
namespace detail {

namespace {

struct DeviceState {
    int32_t* ramp = nullptr;
    int ramp_n = 0;
    int32_t* zeros = nullptr;
    int zeros_n = 0;
    void* ws = nullptr;
    size_t ws_bytes = 0;
    cublasHandle_t cublas = nullptr;
    std::map<std::tuple<float, int, bool, float, float, float, int>, std::pair<hx_rope_table*, int>> tables;
    std::map<void*, std::tuple<void*, int, int, int, hx_kv_cache*>> wraps;
};

std::mutex g_mu;
DeviceState g_state[64];

DeviceState& state()
{
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) throw std::runtime_error("device ordinal out of range");
    return g_state[dev];
}

}  // namespace

const int32_t* ramp(int n)
{
    std::lock_guard<std::mutex> lk(g_mu);
    DeviceState& s = state();
    if (n > s.ramp_n) {
        int m = 4096;
        while (m < n) m *= 2;
        std::vector<int32_t> h(m);
        for (int i = 0; i < m; i++) h[i] = i;
        int32_t* d = nullptr;
        if (cudaMalloc(&d, sizeof(int32_t) * m) != cudaSuccess) return nullptr;
        cudaMemcpy(d, h.data(), sizeof(int32_t) * m, cudaMemcpyHostToDevice);
        if (s.ramp) cudaFree(s.ramp);
        s.ramp = d;
        s.ramp_n = m;
    }
    return s.ramp;
}

const int32_t* zeros(int n)
{
    std::lock_guard<std::mutex> lk(g_mu);
    DeviceState& s = state();
    if (n > s.zeros_n) {
        int m = 256;
        while (m < n) m *= 2;
        std::vector<int32_t> h(m, 0);
        int32_t* d = nullptr;
        if (cudaMalloc(&d, sizeof(int32_t) * m) != cudaSuccess) return nullptr;
        if (cudaMemcpy(d, h.data(), sizeof(int32_t) * m, cudaMemcpyHostToDevice) != cudaSuccess) {
            cudaFree(d);
            return nullptr;
        }
        if (s.zeros) cudaFree(s.zeros);
        s.zeros = d;
        s.zeros_n = m;
    }
    return s.zeros;
}

void* workspace(size_t bytes)
{
    std::lock_guard<std::mutex> lk(g_mu);
    DeviceState& s = state();
    if (bytes > s.ws_bytes) {
        if (s.ws) cudaFree(s.ws);
        s.ws = nullptr;
        s.ws_bytes = 0;
        if (cudaMalloc(&s.ws, bytes) != cudaSuccess) return nullptr;
        // zero-filled once, as hx_decode_attention requires; every call leaves
        // its counters zero again
        if (cudaMemset(s.ws, 0, bytes) != cudaSuccess) return nullptr;
        s.ws_bytes = bytes;
    }
    return s.ws;
}

cublasHandle_t cublas()
{
    std::lock_guard<std::mutex> lk(g_mu);
    DeviceState& s = state();
    if (!s.cublas && cublasCreate(&s.cublas) != CUBLAS_STATUS_SUCCESS) return nullptr;
    return s.cublas;
}

const hx_rope_table* rope_table(const ModelConfig& c, float base, int head_dim, int max_pos)
{
    std::lock_guard<std::mutex> lk(g_mu);
    DeviceState& s = state();
    auto key = std::make_tuple(base, head_dim, c.rope_use_yarn, c.rope_factor, c.rope_beta_fast,
                               c.rope_beta_slow, c.rope_orig_max_pos);
    auto it = s.tables.find(key);
    if (it != s.tables.end() && max_pos <= it->second.second) return it->second.first;
    int m = 4096;
    while (m < max_pos) m *= 2;
    hx_rope_config rc{};
    rc.head_dim = head_dim;
    rc.max_pos = m;
    rc.theta = base;
    rc.use_yarn = c.rope_use_yarn ? 1 : 0;
    rc.yarn_factor = c.rope_factor;
    rc.yarn_beta_fast = c.rope_beta_fast;
    rc.yarn_beta_slow = c.rope_beta_slow;
    rc.yarn_orig_max_pos = c.rope_orig_max_pos;
    hx_rope_table* t = nullptr;
    if (hx_rope_table_create(&rc, &t) != HX_OK) return nullptr;
    if (it != s.tables.end()) {
        cudaDeviceSynchronize();  // the old table may still be read by queued launches
        hx_rope_table_destroy(it->second.first);
    }
    s.tables[key] = std::make_pair(t, m);
    return t;
}

hx_kv_cache* wrapped_cache(void* k, void* v, int hkv, int hd, int capacity)
{
    std::lock_guard<std::mutex> lk(g_mu);
    DeviceState& s = state();
    auto it = s.wraps.find(k);
    if (it != s.wraps.end()) {
        auto& [vv, h, d, cap, handle] = it->second;
        if (vv == v && h == hkv && d == hd && cap == capacity) return handle;
        hx_kv_destroy(handle);
        s.wraps.erase(it);
    }
    hx_kv_cache* handle = nullptr;
    if (hx_kv_wrap(k, v, hkv, hd, capacity, &handle) != HX_OK) return nullptr;
    s.wraps[k] = std::make_tuple(v, hkv, hd, capacity, handle);
    return handle;
}

void forget_cache(void* k)
{
    std::lock_guard<std::mutex> lk(g_mu);
    DeviceState& s = state();
    auto it = s.wraps.find(k);
    if (it != s.wraps.end()) {
        hx_kv_destroy(std::get<4>(it->second));
        s.wraps.erase(it);
    }
}

}  // namespace detail
}  // namespace hxinfer
