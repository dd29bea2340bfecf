// convert.cu — checkpoint dtype conversion on the device (weight loading).
//
// The reference converts BF16 / FP32 checkpoint tensors on the CPU, one
// element at a time, before a pageable cudaMemcpy
// (model_loaders/src/safetensors_loader.cpp:12-27 bf16_to_fp16, 124-197 the
// other pairs).  Here the raw checkpoint bytes go to the device unchanged and
// this kernel converts them at HBM speed, in place when the element sizes are
// equal (BF16 -> FP16, the common case for Qwen2 / LLaMA checkpoints).
//
// Arithmetic (same as the reference's loops):
//   BF16 -> FP32  the 16 bits become the top half of an FP32 word (exact)
//   FP32 -> FP16  round to nearest even, overflow to infinity (__float2half_rn)
//   BF16 -> FP16  BF16 -> FP32 -> FP16
//   FP16 -> FP32  exact
//
// Layout: one thread converts a group of eight elements with 16-byte accesses
// when both pointers are 16-byte aligned; the n % 8 tail, or everything when a
// pointer is not aligned, goes element by element.  Each element is read and
// written by the same thread, so dst == src is safe; plain coherent loads (no
// read-only cache path, no __restrict__) keep that true.  Bound: HBM.
#include "hx_common.cuh"

namespace hx {

constexpr int kConvThreads = 256;

template <int DT>
struct Elem;
template <>
struct Elem<HX_FP32> {
    using T = float;
    __device__ static float get(const T* p, int64_t i) { return __ldcs(p + i); }
    __device__ static void put(T* p, int64_t i, float v) { __stcs(p + i, v); }
    // eight elements at p[8g .. 8g+7]
    __device__ static void get8(const T* p, int64_t g, float (&f)[8])
    {
        const float4 a = __ldcs(reinterpret_cast<const float4*>(p) + 2 * g);
        const float4 b = __ldcs(reinterpret_cast<const float4*>(p) + 2 * g + 1);
        f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w;
        f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
    }
    __device__ static void put8(T* p, int64_t g, const float (&f)[8])
    {
        __stcs(reinterpret_cast<float4*>(p) + 2 * g, make_float4(f[0], f[1], f[2], f[3]));
        __stcs(reinterpret_cast<float4*>(p) + 2 * g + 1, make_float4(f[4], f[5], f[6], f[7]));
    }
};
template <>
struct Elem<HX_FP16> {
    using T = __half;
    __device__ static float get(const T* p, int64_t i) { return __half2float(p[i]); }
    __device__ static void put(T* p, int64_t i, float v) { p[i] = __float2half_rn(v); }
    __device__ static void get8(const T* p, int64_t g, float (&f)[8])
    {
        const uint4 v = __ldcs(reinterpret_cast<const uint4*>(p) + g);
        const __half2* h = reinterpret_cast<const __half2*>(&v);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const float2 x = __half22float2(h[e]);
            f[2 * e] = x.x;
            f[2 * e + 1] = x.y;
        }
    }
    __device__ static void put8(T* p, int64_t g, const float (&f)[8])
    {
        uint4 v;
        __half2* h = reinterpret_cast<__half2*>(&v);
#pragma unroll
        for (int e = 0; e < 4; ++e) h[e] = __floats2half2_rn(f[2 * e], f[2 * e + 1]);
        __stcs(reinterpret_cast<uint4*>(p) + g, v);
    }
};
template <>
struct Elem<HX_BF16> {  // source only
    using T = uint16_t;
    __device__ static float bits(uint32_t b) { return __uint_as_float(b << 16); }
    __device__ static float get(const T* p, int64_t i) { return bits(p[i]); }
    __device__ static void get8(const T* p, int64_t g, float (&f)[8])
    {
        const uint4 v = __ldcs(reinterpret_cast<const uint4*>(p) + g);
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            f[2 * e] = __uint_as_float(w[e] << 16);          // low half: element 2e
            f[2 * e + 1] = __uint_as_float(w[e] & 0xffff0000u);  // high half: element 2e + 1
        }
    }
};

// units [0, groups) are 8-element groups, units [groups, groups + tail) single
// elements 8 * groups + (u - groups)
template <int SRC, int DST>
__global__ void __launch_bounds__(kConvThreads)
    convert_kernel(void* dst, const void* src, int64_t groups, int64_t tail)
{
    using S = Elem<SRC>;
    using D = Elem<DST>;
    const typename S::T* s = static_cast<const typename S::T*>(src);
    typename D::T* d = static_cast<typename D::T*>(dst);
    const int64_t units = groups + tail;
    const int64_t stride = (int64_t)gridDim.x * kConvThreads;
    for (int64_t u = (int64_t)blockIdx.x * kConvThreads + threadIdx.x; u < units; u += stride) {
        if (u < groups) {
            float f[8];
            S::get8(s, u, f);
            D::put8(d, u, f);
        } else {
            const int64_t i = 8 * groups + (u - groups);
            D::put(d, i, S::get(s, i));
        }
    }
}

static int elem_bytes(int dtype)
{
    switch (dtype) {
    case HX_FP32: return 4;
    case HX_FP16: return 2;
    case HX_BF16: return 2;
    default: return 0;
    }
}

template <int SRC, int DST>
static int launch_convert(void* dst, const void* src, size_t n, cudaStream_t stream)
{
    const bool aligned = ((reinterpret_cast<uintptr_t>(dst) | reinterpret_cast<uintptr_t>(src)) & 15) == 0;
    const int64_t groups = aligned ? (int64_t)(n / 8) : 0;
    const int64_t tail = (int64_t)n - 8 * groups;
    const int64_t units = groups + tail;
    const int blocks = (int)std::max<int64_t>(
        1, std::min<int64_t>((units + kConvThreads - 1) / kConvThreads, (int64_t)num_sms() * 8));
    convert_kernel<SRC, DST><<<blocks, kConvThreads, 0, stream>>>(dst, src, groups, tail);
    return check_launch("convert_kernel");
}

}  // namespace hx

using namespace hx;

extern "C" int hx_convert(void* dst, int dst_dtype, const void* src, int src_dtype, size_t n,
                          hx_stream_t stream_)
{
    HX_NVTX_RANGE("hx_convert");
    const int sb = elem_bytes(src_dtype), db = elem_bytes(dst_dtype);
    if (!sb || !db || dst_dtype == HX_BF16)
        return fail(HX_ERR_INVALID, "hx_convert: unsupported dtypes %d -> %d", src_dtype, dst_dtype);
    if (n == 0) return HX_OK;
    if (!dst || !src) return fail(HX_ERR_INVALID, "hx_convert: null pointer");
    if (n > (SIZE_MAX >> 3)) return fail(HX_ERR_INVALID, "hx_convert: %zu elements", n);
    const uintptr_t d0 = reinterpret_cast<uintptr_t>(dst), s0 = reinterpret_cast<uintptr_t>(src);
    const uintptr_t d1 = d0 + n * db, s1 = s0 + n * sb;
    if (dst != src && d0 < s1 && s0 < d1)
        return fail(HX_ERR_INVALID, "hx_convert: source and destination overlap");
    if (dst == src && sb != db)
        return fail(HX_ERR_INVALID, "hx_convert: in place needs equal element sizes");
    if ((d0 % db) || (s0 % sb))
        return fail(HX_ERR_INVALID, "hx_convert: pointer not aligned to its element size");
    cudaStream_t stream = (cudaStream_t)stream_;
    if (src_dtype == dst_dtype) {
        if (dst == src) return HX_OK;
        HX_CUDA_TRY(cudaMemcpyAsync(dst, src, n * db, cudaMemcpyDeviceToDevice, stream));
        return HX_OK;
    }
    if (src_dtype == HX_BF16 && dst_dtype == HX_FP16) return launch_convert<HX_BF16, HX_FP16>(dst, src, n, stream);
    if (src_dtype == HX_BF16 && dst_dtype == HX_FP32) return launch_convert<HX_BF16, HX_FP32>(dst, src, n, stream);
    if (src_dtype == HX_FP32 && dst_dtype == HX_FP16) return launch_convert<HX_FP32, HX_FP16>(dst, src, n, stream);
    return launch_convert<HX_FP16, HX_FP32>(dst, src, n, stream);
}
