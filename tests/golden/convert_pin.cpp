// convert_pin.cpp — runs the conversions of the reference's checkpoint loader
// (model_loaders/src/safetensors_loader.cpp:12-27, 124-197) on the host, with
// the functions those loops call: __float2half and __half2float from CUDA's
// cuda_fp16.h (host implementations).  Used only by make_convert_golden.py to
// pin the oracle's restatement.
//
//   convert_pin bf16_to_f16 <in.u16> <out.u16>   bits << 16 -> float -> __float2half
//   convert_pin f32_to_f16  <in.u32> <out.u16>   __float2half
//   convert_pin f16_to_f32  <in.u16> <out.u32>   __half2float
#include <cuda_fp16.h>

#include <cstdint>
#include <cstdio>
#include <cstring>
#include <vector>

template <typename T>
static std::vector<T> read_all(const char* path)
{
    std::vector<T> v;
    FILE* f = std::fopen(path, "rb");
    if (!f) return v;
    T x;
    while (std::fread(&x, sizeof(T), 1, f) == 1) v.push_back(x);
    std::fclose(f);
    return v;
}

template <typename T>
static bool write_all(const char* path, const std::vector<T>& v)
{
    FILE* f = std::fopen(path, "wb");
    if (!f) return false;
    const bool ok = std::fwrite(v.data(), sizeof(T), v.size(), f) == v.size();
    return std::fclose(f) == 0 && ok;
}

static uint16_t half_bits(__half h)
{
    uint16_t b;
    std::memcpy(&b, &h, 2);
    return b;
}

int main(int argc, char** argv)
{
    if (argc != 4) {
        std::fprintf(stderr, "usage: convert_pin bf16_to_f16|f32_to_f16|f16_to_f32 in out\n");
        return 2;
    }
    const char* mode = argv[1];
    if (!std::strcmp(mode, "bf16_to_f16")) {
        auto in = read_all<uint16_t>(argv[2]);
        std::vector<uint16_t> out(in.size());
        for (size_t i = 0; i < in.size(); ++i) {
            const uint32_t bits = (uint32_t)in[i] << 16;
            float f;
            std::memcpy(&f, &bits, 4);
            out[i] = half_bits(__float2half(f));
        }
        return write_all(argv[3], out) ? 0 : 1;
    }
    if (!std::strcmp(mode, "f32_to_f16")) {
        auto in = read_all<uint32_t>(argv[2]);
        std::vector<uint16_t> out(in.size());
        for (size_t i = 0; i < in.size(); ++i) {
            float f;
            std::memcpy(&f, &in[i], 4);
            out[i] = half_bits(__float2half(f));
        }
        return write_all(argv[3], out) ? 0 : 1;
    }
    if (!std::strcmp(mode, "f16_to_f32")) {
        auto in = read_all<uint16_t>(argv[2]);
        std::vector<uint32_t> out(in.size());
        for (size_t i = 0; i < in.size(); ++i) {
            __half h;
            std::memcpy(&h, &in[i], 2);
            const float f = __half2float(h);
            std::memcpy(&out[i], &f, 4);
        }
        return write_all(argv[3], out) ? 0 : 1;
    }
    std::fprintf(stderr, "unknown mode %s\n", mode);
    return 2;
}
