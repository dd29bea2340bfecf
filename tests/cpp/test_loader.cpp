// test_loader.cpp — drives SafetensorsReader / SafetensorsMultiReader /
// AttentionLoader for tests/test_loader.py (CPU subcommands) and
// tests/test_zz_gpu_weights.py (GPU subcommands).  Prints one result per line;
// the Python tests hold the expectations.
//
//   info <file>                       header as parsed (no CUDA calls)
//   multi <dir> [probe ...]           directory of shards (no CUDA calls)
//   config <dir>                      AttentionLoader::load_config (no CUDA calls)
//   fetch <file|dir> <out_dir> <name>:<fp16|fp32|int8> ...
//                                     get_tensor_gpu, result bytes to <out_dir>/<i>.bin
//   json <file>                       each line parsed by json_lite: "ok <canonical JSON>"
//                                     or "error" (no CUDA calls)
//   time <file> <name> <fp16|fp32> <reps>
//                                     wall time of get_tensor_gpu (file bytes in the page
//                                     cache after the first call): "time <best ms> <file bytes>"
//   layers <model_dir> <ref_dir> <npos>
//                                     AttentionLoader::load_layers vs. AttentionLayers built from
//                                     the weights in <ref_dir>; forward outputs compared bitwise
#include <cuda_runtime.h>

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <iostream>
#include <memory>
#include <string>
#include <vector>

#include "json_lite.h"
#include "model_loaders/attention_loader.h"
#include "model_loaders/safetensors_loader.h"

using namespace hxinfer;

static uint64_t fnv1a(const void* p, size_t n)
{
    const unsigned char* b = static_cast<const unsigned char*>(p);
    uint64_t h = 1469598103934665603ull;
    for (size_t i = 0; i < n; ++i) {
        h ^= b[i];
        h *= 1099511628211ull;
    }
    return h;
}

static int cmd_info(const std::string& path)
{
    SafetensorsReader r;
    if (!r.load(path)) {
        std::cout << "load fail\n";
        return 0;
    }
    std::cout << "load ok\n";
    std::cout << "n " << r.num_tensors() << "\n";
    for (const auto& name : r.tensor_names()) {
        const SafetensorInfo* info = r.get_info(name);
        std::string shape;
        for (size_t i = 0; i < info->shape.size(); ++i) shape += (i ? "," : "") + std::to_string(info->shape[i]);
        if (shape.empty()) shape = "-";
        char h[32];
        std::snprintf(h, sizeof h, "%016llx",
                      (unsigned long long)fnv1a(r.get_raw_ptr(name), info->offset_end - info->offset_begin));
        std::cout << "t " << name << " " << info->dtype << " " << shape << " " << info->offset_begin << " "
                  << info->offset_end << " " << h << " " << (r.has_tensor(name) ? 1 : 0) << "\n";
    }
    const char* absent = "no.such.tensor";
    std::cout << "absent " << (!r.has_tensor(absent) && !r.get_info(absent) && !r.get_raw_ptr(absent)) << "\n";
    return 0;
}

static int cmd_multi(const std::string& dir, int argc, char** argv)
{
    SafetensorsMultiReader m;
    std::cout << "load " << (m.load_directory(dir) ? "ok" : "fail") << "\n";
    std::cout << "n " << m.num_tensors() << "\n";
    for (const auto& name : m.tensor_names()) std::cout << "m " << name << "\n";
    for (int i = 0; i < argc; ++i) std::cout << "has " << argv[i] << " " << (m.has_tensor(argv[i]) ? 1 : 0) << "\n";
    return 0;
}

// Canonical JSON text of a parsed value: members in document order, numbers
// as int64 or %.17g, strings with only the escapes JSON requires.
static void dump(const json_lite::Value& v, std::string& out)
{
    using json_lite::Value;
    switch (v.kind) {
    case Value::Null: out += "null"; break;
    case Value::Bool: out += v.boolean ? "true" : "false"; break;
    case Value::Number: {
        char buf[40];
        if (v.is_int)
            std::snprintf(buf, sizeof buf, "%lld", (long long)v.integer);
        else
            std::snprintf(buf, sizeof buf, "%.17g", v.number);
        out += buf;
        break;
    }
    case Value::String:
        out += '"';
        for (unsigned char c : v.str) {
            if (c == '"' || c == '\\') {
                out += '\\';
                out += (char)c;
            } else if (c < 0x20) {
                char buf[8];
                std::snprintf(buf, sizeof buf, "\\u%04x", c);
                out += buf;
            } else {
                out += (char)c;
            }
        }
        out += '"';
        break;
    case Value::Array:
        out += '[';
        for (size_t i = 0; i < v.items.size(); ++i) {
            if (i) out += ',';
            dump(v.items[i], out);
        }
        out += ']';
        break;
    case Value::Object:
        out += '{';
        for (size_t i = 0; i < v.members.size(); ++i) {
            if (i) out += ',';
            json_lite::Value key;
            key.kind = Value::String;
            key.str = v.members[i].first;
            dump(key, out);
            out += ':';
            dump(v.members[i].second, out);
        }
        out += '}';
        break;
    }
}

static int cmd_json(const std::string& path)
{
    std::ifstream f(path, std::ios::binary);
    std::string line;
    while (std::getline(f, line)) {
        json_lite::Value v;
        std::string err;
        if (json_lite::parse(line.data(), line.data() + line.size(), v, &err)) {
            std::string out;
            dump(v, out);
            std::cout << "ok " << out << "\n";
        } else {
            std::cout << "error\n";
        }
    }
    return 0;
}

static int cmd_config(const std::string& dir)
{
    ModelConfig c{};
    try {
        AttentionLoader::load_config(dir, c);
    } catch (const std::exception& e) {
        std::cout << "error " << e.what() << "\n";
        return 0;
    }
    char line[512];
    std::snprintf(line, sizeof line,
                  "config dim=%d hidden_dim=%d layer=%d head=%d kv_head=%d vocab=%d seq_len=%d "
                  "theta=%.9g yarn=%d factor=%.9g orig=%d beta_fast=%.9g beta_slow=%.9g",
                  c.dim, c.hidden_dim, c.layer, c.head, c.kv_head, c.vocab_size, c.seq_len, c.rope_theta,
                  c.rope_use_yarn ? 1 : 0, c.rope_factor, c.rope_orig_max_pos, c.rope_beta_fast,
                  c.rope_beta_slow);
    std::cout << line << "\n";
    return 0;
}

static int cmd_fetch(const std::string& path, const std::string& out_dir, int argc, char** argv)
{
    auto alloc = std::make_shared<CUDAAllocator>();
    SafetensorsReader one;
    SafetensorsMultiReader many;
    // a path not ending in .safetensors is a directory of shards
    const bool dir = path.size() <= 12 || path.compare(path.size() - 12, 12, ".safetensors") != 0;
    if (dir ? !many.load_directory(path) : !one.load(path)) {
        std::cout << "load fail\n";
        return 0;
    }
    for (int i = 0; i < argc; ++i) {
        const std::string spec = argv[i];
        const size_t colon = spec.rfind(':');
        const std::string name = spec.substr(0, colon), want = spec.substr(colon + 1);
        const DataType dt = want == "fp32" ? DataType::kDataTypeFP32
                            : want == "int8" ? DataType::kDataTypeInt8
                                             : DataType::kDataTypeFP16;
        auto t = dir ? many.get_tensor_gpu(name, alloc, dt) : one.get_tensor_gpu(name, alloc, dt);
        if (!t) {
            std::cout << "r " << i << " null\n";
            continue;
        }
        std::vector<char> host(t->tensor_total_byte_size());
        if (!host.empty() &&
            cudaMemcpy(host.data(), t->raw_data_ptr(), host.size(), cudaMemcpyDeviceToHost) != cudaSuccess) {
            std::cout << "r " << i << " copy-fail\n";
            continue;
        }
        std::ofstream f(out_dir + "/" + std::to_string(i) + ".bin", std::ios::binary);
        f.write(host.data(), (std::streamsize)host.size());
        std::cout << "r " << i << " ok " << host.size() << " " << (t->tensor_device_type() == DeviceType::kDeviceCUDA)
                  << "\n";
    }
    return 0;
}

static int cmd_time(const std::string& path, const std::string& name, const std::string& want, int reps)
{
    auto alloc = std::make_shared<CUDAAllocator>();
    SafetensorsReader r;
    if (!r.load(path) || !r.has_tensor(name)) {
        std::cout << "load fail\n";
        return 0;
    }
    const DataType dt = want == "fp32" ? DataType::kDataTypeFP32 : DataType::kDataTypeFP16;
    const SafetensorInfo* info = r.get_info(name);
    double best = 1e30;
    for (int i = 0; i < std::max(1, reps); ++i) {
        const auto t0 = std::chrono::steady_clock::now();
        auto t = r.get_tensor_gpu(name, alloc, dt);  // synchronous: data on the device at return
        const auto t1 = std::chrono::steady_clock::now();
        if (!t) {
            std::cout << "r null\n";
            return 0;
        }
        best = std::min(best, std::chrono::duration<double, std::milli>(t1 - t0).count());
    }
    std::cout << "time " << best << " " << (info->offset_end - info->offset_begin) << "\n";
    return 0;
}

static std::shared_ptr<Tensor> upload_file(const std::shared_ptr<CUDAAllocator>& alloc, const std::string& path,
                                           std::vector<int> shape, DataType dt)
{
    std::ifstream f(path, std::ios::binary);
    if (!f) return nullptr;
    std::vector<char> bytes((std::istreambuf_iterator<char>(f)), std::istreambuf_iterator<char>());
    auto t = std::make_shared<Tensor>(alloc, shape, dt);
    t->tensor_set_device_type(DeviceType::kDeviceCUDA);
    if (bytes.size() != t->tensor_total_byte_size()) return nullptr;
    cudaMemcpy(t->raw_data_ptr(), bytes.data(), bytes.size(), cudaMemcpyHostToDevice);
    return t;
}

static int cmd_layers(const std::string& model_dir, const std::string& ref_dir, int npos)
{
    auto alloc = std::make_shared<CUDAAllocator>();
    ModelConfig c{};
    std::vector<std::shared_ptr<AttentionLayer>> loaded;
    try {
        loaded = AttentionLoader::load_layers(model_dir, c, alloc);
    } catch (const std::exception& e) {
        std::cout << "error " << e.what() << "\n";
        return 0;
    }
    const int dim = c.dim, kv_dim = c.kv_head * (c.dim / c.head);
    std::cout << "loaded " << loaded.size() << "\n";
    for (int l = 0; l < (int)loaded.size(); ++l) {
        const std::string p = ref_dir + "/" + std::to_string(l) + ".";
        auto wq = upload_file(alloc, p + "wq.bin", {dim, dim}, c.weight_dtype);
        auto wk = upload_file(alloc, p + "wk.bin", {kv_dim, dim}, c.weight_dtype);
        auto wv = upload_file(alloc, p + "wv.bin", {kv_dim, dim}, c.weight_dtype);
        auto wo = upload_file(alloc, p + "wo.bin", {dim, dim}, c.weight_dtype);
        auto bq = upload_file(alloc, p + "bq.bin", {dim}, c.bias_dtype);
        auto bk = upload_file(alloc, p + "bk.bin", {kv_dim}, c.bias_dtype);
        auto bv = upload_file(alloc, p + "bv.bin", {kv_dim}, c.bias_dtype);
        if (!wq || !wk || !wv || !wo) {
            std::cout << "error reference weights of layer " << l << "\n";
            return 0;
        }
        const bool bias = bq && bk && bv;
        auto ref = bias ? std::make_shared<AttentionLayer>(alloc, c, wq, wk, wv, wo, bq, bk, bv)
                        : std::make_shared<AttentionLayer>(alloc, c, wq, wk, wv, wo);
        auto in = std::make_shared<Tensor>(alloc, std::vector<int>{1, dim}, DataType::kDataTypeFP32);
        auto out_a = std::make_shared<Tensor>(alloc, std::vector<int>{1, dim}, DataType::kDataTypeFP32);
        auto out_b = std::make_shared<Tensor>(alloc, std::vector<int>{1, dim}, DataType::kDataTypeFP32);
        for (auto& t : {in, out_a, out_b}) t->tensor_set_device_type(DeviceType::kDeviceCUDA);
        long mismatches = 0;
        double max_abs = 0.0;
        for (int pos = 0; pos < npos; ++pos) {
            std::vector<float> x(dim);
            for (int j = 0; j < dim; ++j) x[j] = std::sin(0.37f * j + 1.3f * pos + 0.5f * l);
            cudaMemcpy(in->raw_data_ptr(), x.data(), dim * 4, cudaMemcpyHostToDevice);
            loaded[l]->forward(in, out_a, pos);
            ref->forward(in, out_b, pos);
            std::vector<float> a(dim), b(dim);
            cudaMemcpy(a.data(), out_a->raw_data_ptr(), dim * 4, cudaMemcpyDeviceToHost);
            cudaMemcpy(b.data(), out_b->raw_data_ptr(), dim * 4, cudaMemcpyDeviceToHost);
            for (int j = 0; j < dim; ++j) {
                mismatches += std::memcmp(&a[j], &b[j], 4) != 0;
                max_abs = std::max(max_abs, (double)std::fabs(a[j]));
            }
        }
        const cudaError_t e = cudaDeviceSynchronize();
        std::cout << "layer " << l << " bias " << bias << " mismatches " << mismatches << " max_abs " << max_abs
                  << " cuda " << (e == cudaSuccess ? "ok" : cudaGetErrorString(e)) << "\n";
    }
    return 0;
}

int main(int argc, char** argv)
{
    if (argc < 3) {
        std::cerr << "usage: test_loader info|multi|config|fetch|layers ...\n";
        return 2;
    }
    const std::string cmd = argv[1];
    if (cmd == "info") return cmd_info(argv[2]);
    if (cmd == "multi") return cmd_multi(argv[2], argc - 3, argv + 3);
    if (cmd == "config") return cmd_config(argv[2]);
    if (cmd == "json") return cmd_json(argv[2]);
    if (cmd == "time" && argc == 6) return cmd_time(argv[2], argv[3], argv[4], std::atoi(argv[5]));
    if (cmd == "fetch" && argc >= 4) return cmd_fetch(argv[2], argv[3], argc - 4, argv + 4);
    if (cmd == "layers" && argc == 5) return cmd_layers(argv[2], argv[3], std::atoi(argv[4]));
    std::cerr << "bad arguments\n";
    return 2;
}
