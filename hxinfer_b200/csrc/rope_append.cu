// rope_append.cu — K1: fused QKV bias + NeoX RoPE + K/V cache append, and the
// in-place RoPE behind the kept rope_cuda operator.
//
// Replaces, in one launch per layer step, the reference chain
//   add_bias_cuda_fp16/fp32 x3        hxinfer-engine/src/op/cuda/bias_add.cu:6-30
//   rope_kernel_cuda_neox(_fp16) x2   hxinfer-engine/src/op/cuda/rope_cuda.cu:46-96,127-148
//   kv_cache_update_kernel(_fp16)     hxinfer-engine/src/op/cuda/attention_score_cuda.cu:7-15,85-93
//
// Numerics: the bias add rounds like the reference (fp16 __hadd, or fp32 add);
// the rotation uses the cos/sin the reference CPU op computes (read from a
// host-built table) and evaluates x1*c - x2*s and x2*c + x1*s with separately
// rounded multiplies and adds, the order of rope_cpu.cpp:29-30 without FMA
// contraction, so the rotated values equal rope_cpu's bit for bit.
#include "hx_common.cuh"

namespace hx {

// ld / ld_bias / st / rotate (the K1 numerics) live in hx_common.cuh, shared
// with the append-and-decode kernel.

// grid (token, head group): each CTA takes heads_per_cta consecutive head
// slots of one token, one thread per NeoX pair (d, d + head_dim/2), so every
// load of a token's step is issued at once.  Slots: [0, hq) = q heads,
// [hq, hq+hkv) = k heads, [hq+hkv, hq+2hkv) = v heads.
template <typename T, typename TO>
__global__ void rope_append_kernel(KVView view, const T* __restrict__ q, const T* __restrict__ k,
                                   const T* __restrict__ v, const T* __restrict__ bq,
                                   const T* __restrict__ bk, const T* __restrict__ bv,
                                   const int32_t* __restrict__ seq_ids,
                                   const int32_t* __restrict__ positions, int hq,
                                   const float2* __restrict__ table, int table_max_pos,
                                   TO* __restrict__ q_out, int heads_per_cta, int* status)
{
    pdl_trigger();
    pdl_wait();  // inputs come from the previous kernel on the stream
    const int i = blockIdx.x;
    const int hd = view.hd, half = hd / 2, hkv = view.hkv;
    const int q_heads = q ? hq : 0;
    const int slot = blockIdx.y * heads_per_cta + (int)threadIdx.x / half;
    const int d = (int)threadIdx.x % half;
    if ((int)threadIdx.x >= heads_per_cta * half || slot >= q_heads + 2 * hkv) return;
    const int seq = seq_ids[i], pos = positions[i];
    if (seq < 0 || seq >= view.max_seqs || pos < 0 || pos >= view.capacity ||
        (table && pos >= table_max_pos)) {
        if (threadIdx.x == 0) record_status(status, HX_ERR_CAPACITY);
        return;
    }
    const float2* cs_row = table ? table + (int64_t)pos * half : nullptr;
    if (slot < q_heads) {
        const int64_t base = ((int64_t)i * hq + slot) * hd + d;
        const T* b = bq ? bq + (int64_t)slot * hd + d : nullptr;
        float x1 = ld_bias(q + base, b), x2 = ld_bias(q + base + half, b ? b + half : nullptr);
        if (cs_row) rotate(x1, x2, cs_row[d], x1, x2);
        if (q_out) {
            st(q_out + base, x1);
            st(q_out + base + half, x2);
        }
        return;
    }
    const bool is_k = slot < q_heads + hkv;
    const int h = is_k ? slot - q_heads : slot - q_heads - hkv;
    const T* src = (is_k ? k : v) + ((int64_t)i * hkv + h) * hd + d;
    const T* bias = is_k ? bk : bv;
    const T* b = bias ? bias + (int64_t)h * hd + d : nullptr;
    float x1 = ld_bias(src, b), x2 = ld_bias(src + half, b ? b + half : nullptr);
    if (is_k && cs_row) rotate(x1, x2, cs_row[d], x1, x2);
    const int64_t off = token_offset(view, seq, h, pos);
    if (off < 0) {
        record_status(status, HX_ERR_CAPACITY);
        return;
    }
    __half* dst = reinterpret_cast<__half*>((is_k ? view.k : view.v) + off);
    dst[d] = __float2half_rn(x1);
    dst[d + half] = __float2half_rn(x2);
}

// In-place RoPE of q [rows][hq*hd] and k [rows][hkv*hd] at one position.
template <typename T>
__global__ void rope_inplace_kernel(T* __restrict__ q, T* __restrict__ k, int rows, int hq,
                                    int hkv, int hd, const float2* __restrict__ cs_row)
{
    const int half = hd / 2;
    const int64_t items = (int64_t)rows * (hq + hkv) * half;
    for (int64_t it = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; it < items;
         it += (int64_t)gridDim.x * blockDim.x) {
        const int d = (int)(it % half);
        const int64_t rs = it / half;
        const int slot = (int)(rs % (hq + hkv));
        const int64_t row = rs / (hq + hkv);
        T* base = slot < hq ? q + (row * hq + slot) * hd : k + (row * hkv + (slot - hq)) * hd;
        float x1 = ld(base + d), x2 = ld(base + d + half);
        rotate(x1, x2, cs_row[d], x1, x2);
        st(base + d, x1);
        st(base + d + half, x2);
    }
}

}  // namespace hx

using namespace hx;

extern "C" int hx_rope_append(hx_kv_cache* c, int layer, const void* q, const void* k,
                              const void* v, int dtype, const void* bq, const void* bk,
                              const void* bv, const int32_t* seq_ids, const int32_t* positions,
                              int n_tokens, int num_q_heads, const hx_rope_table* table,
                              void* q_out, int q_out_dtype, hx_stream_t stream)
{
    HX_NVTX_RANGE("hx_rope_append");
    if (!c) return fail(HX_ERR_INVALID, "null cache");
    if (layer < 0 || layer >= c->cfg.num_layers) return fail(HX_ERR_INVALID, "layer %d out of range", layer);
    if (!k || !v || !seq_ids || !positions) return fail(HX_ERR_INVALID, "null k/v/seq_ids/positions");
    if (n_tokens < 0) return fail(HX_ERR_INVALID, "n_tokens < 0");
    const int hd = c->cfg.head_dim;
    if (q && (num_q_heads < 1 || num_q_heads % c->cfg.num_kv_heads))
        return fail(HX_ERR_INVALID, "num_q_heads %d is not a multiple of kv heads %d", num_q_heads,
                    c->cfg.num_kv_heads);
    if (table && table->cfg.head_dim != hd)
        return fail(HX_ERR_INVALID, "rope table head_dim %d != cache head_dim %d", table->cfg.head_dim, hd);
    if (dtype != HX_FP16 && dtype != HX_FP32) return fail(HX_ERR_INVALID, "dtype %d", dtype);
    if (q_out && q_out_dtype != HX_FP16 && q_out_dtype != HX_FP32)
        return fail(HX_ERR_INVALID, "q_out dtype %d", q_out_dtype);
    if (n_tokens == 0) return HX_OK;
    if (int rc = check_device(c->device, "the cache")) return rc;
    if (table)
        if (int rc = check_device(table->device, "the rope table")) return rc;
    KVView view = make_view(c, layer);
    const float2* tab = table ? table->d_cos_sin : nullptr;
    const int tmax = table ? table->cfg.max_pos : 0;
    const int half = hd / 2;
    const int threads = 256;
    const int heads_per_cta = std::max(1, threads / half);
    const int slots = (q ? num_q_heads : 0) + 2 * c->cfg.num_kv_heads;
    const dim3 grid(n_tokens, (slots + heads_per_cta - 1) / heads_per_cta);
    cudaStream_t s = (cudaStream_t)stream;
    int* sw = status_word();
    const bool ov = (c->cfg.flags & HX_KV_OVERLAP_LAUNCH) != 0;
    const bool q16 = !q_out || q_out_dtype == HX_FP16;
    if (dtype == HX_FP16) {
        if (q16)
            launch_kernel(rope_append_kernel<__half, __half>, grid, dim3(threads), 0, s, ov,
                view, (const __half*)q, (const __half*)k, (const __half*)v, (const __half*)bq,
                (const __half*)bk, (const __half*)bv, seq_ids, positions, num_q_heads, tab, tmax,
                (__half*)q_out, heads_per_cta, sw);
        else
            launch_kernel(rope_append_kernel<__half, float>, grid, dim3(threads), 0, s, ov,
                view, (const __half*)q, (const __half*)k, (const __half*)v, (const __half*)bq,
                (const __half*)bk, (const __half*)bv, seq_ids, positions, num_q_heads, tab, tmax,
                (float*)q_out, heads_per_cta, sw);
    } else {
        if (q16)
            launch_kernel(rope_append_kernel<float, __half>, grid, dim3(threads), 0, s, ov,
                view, (const float*)q, (const float*)k, (const float*)v, (const float*)bq,
                (const float*)bk, (const float*)bv, seq_ids, positions, num_q_heads, tab, tmax,
                (__half*)q_out, heads_per_cta, sw);
        else
            launch_kernel(rope_append_kernel<float, float>, grid, dim3(threads), 0, s, ov,
                view, (const float*)q, (const float*)k, (const float*)v, (const float*)bq,
                (const float*)bk, (const float*)bv, seq_ids, positions, num_q_heads, tab, tmax,
                (float*)q_out, heads_per_cta, sw);
    }
    return check_launch("rope_append_kernel");
}

extern "C" int hx_rope_qk(void* q, void* k, int dtype, int rows, int num_q_heads,
                          int num_kv_heads, int head_dim, int step, const hx_rope_table* table,
                          hx_stream_t stream)
{
    HX_NVTX_RANGE("hx_rope_qk");
    if (!q || !k || !table) return fail(HX_ERR_INVALID, "null q/k/table");
    if (rows < 0 || num_q_heads < 1 || num_kv_heads < 1) return fail(HX_ERR_INVALID, "bad shape");
    if (head_dim != table->cfg.head_dim)
        return fail(HX_ERR_INVALID, "head_dim %d != rope table head_dim %d", head_dim,
                    table->cfg.head_dim);
    if (step < 0 || step >= table->cfg.max_pos)
        return fail(HX_ERR_CAPACITY, "step %d outside the rope table [0, %d)", step, table->cfg.max_pos);
    if (rows == 0) return HX_OK;
    if (int rc = check_device(table->device, "the rope table")) return rc;
    const float2* cs = table->d_cos_sin + (int64_t)step * (head_dim / 2);
    int64_t items = (int64_t)rows * (num_q_heads + num_kv_heads) * (head_dim / 2);
    int blocks = (int)std::min<int64_t>((items + 255) / 256, 4096);
    cudaStream_t s = (cudaStream_t)stream;
    if (dtype == HX_FP16)
        rope_inplace_kernel<__half><<<blocks, 256, 0, s>>>((__half*)q, (__half*)k, rows,
                                                           num_q_heads, num_kv_heads, head_dim, cs);
    else if (dtype == HX_FP32)
        rope_inplace_kernel<float><<<blocks, 256, 0, s>>>((float*)q, (float*)k, rows, num_q_heads,
                                                          num_kv_heads, head_dim, cs);
    else
        return fail(HX_ERR_INVALID, "dtype %d", dtype);
    return check_launch("rope_inplace_kernel");
}
