// device_context.h — per-device state shared by the C++ operators: a device
// [0, n) int32 ramp (positions and lengths are passed to the C ABI as device
// pointers into it), the split-K workspace, a cuBLAS handle, RoPE tables
// keyed by their parameters and cache handles over caller tensors.
#pragma once
#include <cublas_v2.h>

#include "base/config.h"
#include "hx_kv.h"

namespace hxinfer {
namespace detail {

// Device pointer to int32 values [0, n) (valid until a larger n is asked for).
const int32_t* ramp(int n);
// Device pointer to n int32 zeros (sequence ids of a one-sequence batch; valid
// until a larger n is asked for).
const int32_t* zeros(int n);
// Device workspace of at least `bytes` bytes.
void* workspace(size_t bytes);
cublasHandle_t cublas();
// RoPE table for (base, head_dim, YaRN fields of config) covering max_pos.
const hx_rope_table* rope_table(const ModelConfig& config, float base, int head_dim, int max_pos);
// Cache handle over caller k/v memory ([hkv][capacity][hd] fp16 inside).
hx_kv_cache* wrapped_cache(void* k, void* v, int hkv, int hd, int capacity);
void forget_cache(void* k);

}  // namespace detail
}  // namespace hxinfer
