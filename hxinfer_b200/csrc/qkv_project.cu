// qkv_project.cu — the QKV projection fused with bias + NeoX RoPE + K/V append.
//
// Replaces, for the decode step of one layer, the reference chain
//   matmul_qkv_cuda: three cublasGemmEx GEMVs      hxinfer-engine/src/op/cuda/matmul_cuda.cu:106-189
//   add_bias_cuda_fp16/fp32 x3                     hxinfer-engine/src/op/cuda/bias_add.cu:20-30
//   RoPE of q and k, K/V cache append              (K1, rope_append.cu)
// with one launch that reads each weight row once.
//
// Weights are the reference's fp16 [out_features][hidden] row-major tensors
// (wq, wk, wv).  Each output element is a dot product over `hidden` with fp32
// accumulation (CUBLAS_COMPUTE_32F in the reference), rounded to the
// projection dtype (fp16 or fp32, the dtype the reference's q/k/v tensors
// have), then the bias is added with the reference's rounding and the rest is
// K1's arithmetic.  Only the order of the fp32 accumulation differs from
// cuBLAS's.
//
// (For 4-8 tokens, qkv_rope_append_mma_kernel below does the dot products on
// the tensor cores instead.)
//
// Grid: (head slot x 4, token group).  A CTA owns 16 NeoX pairs (d, d + 64)
// of one head, i.e. 32 weight rows, so the rotation needs no exchange between
// CTAs; 36-48 heads x 4 = 144-192 CTAs cover the SMs.  Eight warps take four
// rows each; lanes stride over 16-byte weight chunks (eight halves) and the
// CTA's tokens are staged in shared memory as fp16.  Bound: HBM (the weights).
#include "hx_common.cuh"

namespace hx {

constexpr int kQkvThreads = 256;
constexpr int kQkvRows = 32;  // weight rows per CTA: pairs d and d + 64, d in a 16-wide quarter

__device__ __forceinline__ float dot8(const uint4& w, const uint4& x)
{
    const __half2* wh = reinterpret_cast<const __half2*>(&w);
    const __half2* xh = reinterpret_cast<const __half2*>(&x);
    float s = 0.f;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        const float2 a = __half22float2(wh[e]);
        const float2 b = __half22float2(xh[e]);
        s = fmaf(a.x, b.x, s);
        s = fmaf(a.y, b.y, s);
    }
    return s;
}

// The projection result rounded like the reference's q/k/v tensor, plus its
// bias with the reference's rounding (bias_add.cu:6-11 for fp16).
template <typename TP>
__device__ __forceinline__ float proj_bias(float acc, const TP* b);
template <>
__device__ __forceinline__ float proj_bias<__half>(float acc, const __half* b)
{
    const __half h = __float2half_rn(acc);
    return b ? __half2float(__hadd(h, *b)) : __half2float(h);
}
template <>
__device__ __forceinline__ float proj_bias<float>(float acc, const float* b)
{
    return b ? __fadd_rn(acc, *b) : acc;
}

template <typename TO>
__device__ __forceinline__ void st_out(TO* p, float v);
template <>
__device__ __forceinline__ void st_out<__half>(__half* p, float v)
{
    *p = __float2half_rn(v);
}
template <>
__device__ __forceinline__ void st_out<float>(float* p, float v)
{
    *p = v;
}

// Shared tail of the projection kernels: one thread per (NeoX pair, token);
// res[lr][t] holds the fp32 dot products of local row lr (d, or d + 64 for
// lr >= 16) for token t0 + t.
template <int NTOK, typename TP, typename TO>
__device__ __forceinline__ void qkv_epilogue(const KVView& view, const float (*res)[NTOK], int slot,
                                             int qtr, int t0, int nt, const TP* bq, const TP* bk,
                                             const TP* bv, const int32_t* seq_ids,
                                             const int32_t* positions, int hq,
                                             const float2* table, int table_max_pos, TO* q_out,
                                             int* status)
{
    const int hkv = view.hkv;
    const int i = threadIdx.x & 15, tt = threadIdx.x >> 4;
    if (tt >= nt) return;
    const int t = t0 + tt;
    const int d = 16 * qtr + i;
    const int seq = seq_ids[t], pos = positions[t];
    if (seq < 0 || seq >= view.max_seqs || pos < 0 || pos >= view.capacity ||
        (table && pos >= table_max_pos)) {
        if (i == 0) record_status(status, HX_ERR_CAPACITY);
        return;
    }
    const float2* cs_row = table ? table + (int64_t)pos * 64 : nullptr;
    if (slot < hq) {
        const TP* b = bq ? bq + (int64_t)slot * 128 + d : nullptr;
        float x1 = proj_bias<TP>(res[i][tt], b), x2 = proj_bias<TP>(res[16 + i][tt], b ? b + 64 : nullptr);
        if (cs_row) {
            const float2 cs = cs_row[d];
            const float o1 = __fsub_rn(__fmul_rn(x1, cs.x), __fmul_rn(x2, cs.y));
            const float o2 = __fadd_rn(__fmul_rn(x2, cs.x), __fmul_rn(x1, cs.y));
            x1 = o1;
            x2 = o2;
        }
        if (q_out) {
            const int64_t base = ((int64_t)t * hq + slot) * 128 + d;
            st_out<TO>(q_out + base, x1);
            st_out<TO>(q_out + base + 64, x2);
        }
        return;
    }
    const bool is_k = slot < hq + hkv;
    const int h = is_k ? slot - hq : slot - hq - hkv;
    const TP* bias = is_k ? bk : bv;
    const TP* b = bias ? bias + (int64_t)h * 128 + d : nullptr;
    float x1 = proj_bias<TP>(res[i][tt], b), x2 = proj_bias<TP>(res[16 + i][tt], b ? b + 64 : nullptr);
    if (is_k && cs_row) {
        const float2 cs = cs_row[d];
        const float o1 = __fsub_rn(__fmul_rn(x1, cs.x), __fmul_rn(x2, cs.y));
        const float o2 = __fadd_rn(__fmul_rn(x2, cs.x), __fmul_rn(x1, cs.y));
        x1 = o1;
        x2 = o2;
    }
    const int64_t off = token_offset(view, seq, h, pos);
    if (off < 0) {
        record_status(status, HX_ERR_CAPACITY);
        return;
    }
    __half* dst = reinterpret_cast<__half*>((is_k ? view.k : view.v) + off);
    dst[d] = __float2half_rn(x1);
    dst[d + 64] = __float2half_rn(x2);
}

// BATCH: weight chunks per lane held in registers, as two alternating
// buffers of BATCH / 2 (see the main loop).  BATCH 8 holds
// ~200 registers, one CTA per SM, for grids that fit the SMs in one wave;
// BATCH <= 4 fits two CTAs per SM for larger grids.
template <int NTOK, int BATCH, typename TP, typename TO>
__global__ void __launch_bounds__(kQkvThreads, BATCH >= 8 ? 1 : 2)
    qkv_rope_append_kernel(KVView view, const void* __restrict__ x, int x_f32, int hidden,
                           int n_tokens, const __half* __restrict__ wq,
                           const __half* __restrict__ wk, const __half* __restrict__ wv,
                           const TP* __restrict__ bq, const TP* __restrict__ bk,
                           const TP* __restrict__ bv, const int32_t* __restrict__ seq_ids,
                           const int32_t* __restrict__ positions, int hq,
                           const float2* __restrict__ table, int table_max_pos,
                           TO* __restrict__ q_out, int* status)
{
    extern __shared__ uint4 smem_x[];  // [NTOK][hidden / 8] fp16 chunks
    __shared__ float res[kQkvRows][NTOK];
    pdl_trigger();
    const int slot = blockIdx.x / 4, qtr = blockIdx.x % 4;
    const int t0 = blockIdx.y * NTOK;
    const int nt = min(NTOK, n_tokens - t0);
    const int hkv = view.hkv;
    const int chunks = hidden / 8;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    // weight rows of this CTA: local row lr -> head row d (lr < 16) or d + 64
    const __half* wslot = slot < hq ? wq + (int64_t)slot * 128 * hidden
                        : slot < hq + hkv ? wk + (int64_t)(slot - hq) * 128 * hidden
                                          : wv + (int64_t)(slot - hq - hkv) * 128 * hidden;
    const uint4* wrow[4];
#pragma unroll
    for (int r = 0; r < 4; ++r) {
        const int lr = 4 * warp + r;
        const int d = 16 * qtr + (lr & 15) + (lr >= 16 ? 64 : 0);
        wrow[r] = reinterpret_cast<const uint4*>(wslot + (int64_t)d * hidden);
    }
    // the weights do not depend on the previous kernel: start them streaming
#pragma unroll
    for (int r = 0; r < 4; ++r)
        if (lane < chunks) asm volatile("prefetch.global.L2 [%0];" ::"l"(wrow[r] + lane));

    pdl_wait();  // x, seq_ids and positions come from the previous kernel
    for (int e = threadIdx.x; e < nt * chunks; e += kQkvThreads) {
        const int t = e / chunks, c = e - t * chunks;
        const int64_t src = (int64_t)(t0 + t) * hidden + 8 * c;
        uint4 v;
        if (x_f32) {
            const float4 a = *reinterpret_cast<const float4*>(static_cast<const float*>(x) + src);
            const float4 b = *reinterpret_cast<const float4*>(static_cast<const float*>(x) + src + 4);
            v = make_uint4(pack_half2(a.x, a.y), pack_half2(a.z, a.w), pack_half2(b.x, b.y),
                           pack_half2(b.z, b.w));
        } else {
            v = *reinterpret_cast<const uint4*>(static_cast<const __half*>(x) + src);
        }
        smem_x[t * chunks + c] = v;
    }
    __syncthreads();

    float acc[4][NTOK];
#pragma unroll
    for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int t = 0; t < NTOK; ++t) acc[r][t] = 0.f;
    // The weights are the only HBM traffic and one lane's arithmetic per chunk
    // is small, so the loop is latency-bound unless many loads are in flight.
    // Two buffers of BATCH / 2 chunks x 4 rows (64 B per chunk), used
    // alternately: the next buffer's loads are issued before the current one
    // is consumed, so a lane always has loads in flight (for 1-2 tokens
    // 64 KB per SM: 4 x 64 B x 256 threads in one CTA, or 2 x 64 B x 256
    // threads in each of two).  With one batch issued and then consumed, the
    // memory system idled while each batch was used.
    constexpr int kHalf = BATCH / 2;
    auto load = [&](uint4 (&w)[kHalf][4], int c0) {
#pragma unroll
        for (int u = 0; u < kHalf; ++u) {
            const int c = c0 + 32 * u;
#pragma unroll
            for (int r = 0; r < 4; ++r)  // read once: do not keep in L1/L2
                w[u][r] = c < chunks ? __ldcs(wrow[r] + c) : make_uint4(0u, 0u, 0u, 0u);
        }
    };
    auto use = [&](const uint4 (&w)[kHalf][4], int c0) {
#pragma unroll
        for (int u = 0; u < kHalf; ++u) {
            const int c = c0 + 32 * u;
            if (c >= chunks) break;
#pragma unroll
            for (int t = 0; t < NTOK; ++t) {
                if (t < nt) {
                    const uint4 xv = smem_x[t * chunks + c];
#pragma unroll
                    for (int r = 0; r < 4; ++r) acc[r][t] += dot8(w[u][r], xv);
                }
            }
        }
    };
    uint4 wa[kHalf][4], wb[kHalf][4];
    load(wa, lane);
    for (int c0 = lane; c0 < chunks; c0 += 64 * kHalf) {
        load(wb, c0 + 32 * kHalf);
        use(wa, c0);
        load(wa, c0 + 64 * kHalf);
        use(wb, c0 + 32 * kHalf);
    }
#pragma unroll
    for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int t = 0; t < NTOK; ++t) {
            float s = acc[r][t];
#pragma unroll
            for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
            if (lane == 0) res[4 * warp + r][t] = s;
        }
    __syncthreads();

    qkv_epilogue<NTOK, TP, TO>(view, res, slot, qtr, t0, nt, bq, bk, bv, seq_ids, positions, hq,
                               table, table_max_pos, q_out, status);
}

// Tensor-core variant for 3-8 tokens (the CUDA-core kernel binds on FMAs
// there): mma.sync m16n8k16 with the tokens as the M side (rows >= 8 zero)
// and eight weight rows as the N side.  Warp (row group rg, half kh) takes
// rows 8rg..8rg+7 and half of `hidden`.  The k index is permuted inside each
// 32-wide window so that a lane's single 16-byte load of its weight row (and
// of its token's activations) feeds both k-steps of the window without
// shuffles: logical k 2t+e (+8) of step s is physical 8t + 4s + e (+2), the
// same mapping for both operands, so the dot products are unchanged.
template <int NTOK, typename TP, typename TO>
__global__ void __launch_bounds__(kQkvThreads)
    qkv_rope_append_mma_kernel(KVView view, const void* __restrict__ x, int x_f32, int hidden,
                               int n_tokens, const __half* __restrict__ wq,
                               const __half* __restrict__ wk, const __half* __restrict__ wv,
                               const TP* __restrict__ bq, const TP* __restrict__ bk,
                               const TP* __restrict__ bv, const int32_t* __restrict__ seq_ids,
                               const int32_t* __restrict__ positions, int hq,
                               const float2* __restrict__ table, int table_max_pos,
                               TO* __restrict__ q_out, int* status)
{
    static_assert(NTOK <= 8, "tokens are the M side of one m16 tile");
    extern __shared__ uint4 smem_x[];  // [8][hidden / 8] fp16 chunks, rows >= nt zero
    __shared__ float part[2][kQkvRows][NTOK];
    __shared__ float res[kQkvRows][NTOK];
    pdl_trigger();
    const int slot = blockIdx.x / 4, qtr = blockIdx.x % 4;
    const int t0 = blockIdx.y * NTOK;
    const int nt = min(NTOK, n_tokens - t0);
    const int hkv = view.hkv;
    const int chunks = hidden / 8;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, t4 = lane & 3;
    const int rg = warp & 3, kh = warp >> 2;

    const __half* wslot = slot < hq ? wq + (int64_t)slot * 128 * hidden
                        : slot < hq + hkv ? wk + (int64_t)(slot - hq) * 128 * hidden
                                          : wv + (int64_t)(slot - hq - hkv) * 128 * hidden;
    const int lr = 8 * rg + g;  // this lane's weight row
    const int d = 16 * qtr + (lr & 15) + (lr >= 16 ? 64 : 0);
    const uint4* wrow = reinterpret_cast<const uint4*>(wslot + (int64_t)d * hidden);
    const int windows = hidden / 32;
    const int w0 = kh * windows / 2, w1 = (kh + 1) * windows / 2;
    asm volatile("prefetch.global.L2 [%0];" ::"l"(wrow + 4 * w0 + t4));

    pdl_wait();  // x, seq_ids and positions come from the previous kernel
    for (int e = threadIdx.x; e < 8 * chunks; e += kQkvThreads) {
        const int t = e / chunks, c = e - t * chunks;
        uint4 v = make_uint4(0, 0, 0, 0);
        if (t < nt) {
            const int64_t src = (int64_t)(t0 + t) * hidden + 8 * c;
            if (x_f32) {
                const float4 a = *reinterpret_cast<const float4*>(static_cast<const float*>(x) + src);
                const float4 b = *reinterpret_cast<const float4*>(static_cast<const float*>(x) + src + 4);
                v = make_uint4(pack_half2(a.x, a.y), pack_half2(a.z, a.w), pack_half2(b.x, b.y),
                               pack_half2(b.z, b.w));
            } else {
                v = *reinterpret_cast<const uint4*>(static_cast<const __half*>(x) + src);
            }
        }
        smem_x[t * chunks + c] = v;
    }
    __syncthreads();

    float acc0[4] = {0.f, 0.f, 0.f, 0.f}, acc1[4] = {0.f, 0.f, 0.f, 0.f};
    const uint4* xrow = smem_x + g * chunks;  // this lane's token (M row g)
#pragma unroll 8
    for (int wdw = w0; wdw < w1; ++wdw) {
        const uint4 w = __ldcs(wrow + 4 * wdw + t4);  // read once
        const uint4 xv = xrow[4 * wdw + t4];
        // step 0: physical 8t4 + {0,1} and + {2,3}; step 1: + {4,5} and + {6,7}
        const uint32_t a0[4] = {xv.x, 0u, xv.y, 0u};
        const uint32_t a1[4] = {xv.z, 0u, xv.w, 0u};
        mma_16816(acc0, a0, w.x, w.y);
        mma_16816(acc1, a1, w.z, w.w);
    }
    // acc[0..1]: token g, rows 8rg + 2t4 (+1); acc[2..3]: tokens g + 8 (none)
    if (g < NTOK) {
        part[kh][8 * rg + 2 * t4][g] = acc0[0] + acc1[0];
        part[kh][8 * rg + 2 * t4 + 1][g] = acc0[1] + acc1[1];
    }
    __syncthreads();
    for (int e = threadIdx.x; e < kQkvRows * NTOK; e += kQkvThreads) {
        const int row = e / NTOK, t = e % NTOK;
        res[row][t] = part[0][row][t] + part[1][row][t];
    }
    __syncthreads();
    qkv_epilogue<NTOK, TP, TO>(view, res, slot, qtr, t0, nt, bq, bk, bv, seq_ids, positions, hq,
                               table, table_max_pos, q_out, status);
}

template <int NTOK, typename TP, typename TO>
static int launch_qkv(const hx_kv_cache* c, const KVView& view, const void* x, int x_f32,
                      int hidden, int n, const void* wq, const void* wk, const void* wv,
                      const void* bq, const void* bk, const void* bv, const int32_t* seq_ids,
                      const int32_t* positions, int hq, const hx_rope_table* table, void* q_out,
                      cudaStream_t stream)
{
    // 4-8 tokens: the tensor-core kernel (whole 32-wide k windows needed)
    const bool mma = NTOK >= 4 && hidden % 32 == 0;
    const dim3 grid((hq + 2 * view.hkv) * 4, (n + NTOK - 1) / NTOK);
    // 1-2 tokens: 8-chunk batches when the grid is one wave of single CTAs
    // per SM, else 4-chunk batches at two CTAs per SM (same bytes in flight)
    const bool one_wave = (int64_t)grid.x * grid.y <= num_sms();
    const int variant = mma ? 2 : (NTOK <= 2 && one_wave) ? 1 : 0;
    constexpr int kSmallBatch = NTOK <= 2 ? 4 : 2, kBigBatch = NTOK <= 2 ? 8 : kSmallBatch;
    auto kernel = variant == 2   ? qkv_rope_append_mma_kernel<NTOK, TP, TO>
                  : variant == 1 ? qkv_rope_append_kernel<NTOK, kBigBatch, TP, TO>
                                 : qkv_rope_append_kernel<NTOK, kSmallBatch, TP, TO>;
    const size_t smem = (size_t)(mma ? 8 : NTOK) * hidden * 2;
    static std::atomic<bool> attr_set[64][3];  // per device; set again on ordinals past 63
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64 || !attr_set[dev][variant].load(std::memory_order_acquire)) {
        HX_CUDA_TRY(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (mma ? 8 : NTOK) * 8192 * 2));
        if (dev >= 0 && dev < 64) attr_set[dev][variant].store(true, std::memory_order_release);
    }
    const bool ov = (c->cfg.flags & HX_KV_OVERLAP_LAUNCH) != 0;
    cudaError_t e = launch_kernel(
        kernel, grid, dim3(kQkvThreads), smem, stream, ov, view, x, x_f32, hidden, n,
        (const __half*)wq, (const __half*)wk, (const __half*)wv, (const TP*)bq, (const TP*)bk,
        (const TP*)bv, seq_ids, positions, hq, table ? (const float2*)table->d_cos_sin : nullptr,
        table ? table->cfg.max_pos : 0, (TO*)q_out, status_word());
    if (e != cudaSuccess) return cuda_fail(e, "qkv_rope_append_kernel launch");
    return check_launch("qkv_rope_append_kernel");
}

template <typename TP, typename TO>
static int launch_qkv_n(const hx_kv_cache* c, const KVView& view, const void* x, int x_f32,
                        int hidden, int n, const void* wq, const void* wk, const void* wv,
                        const void* bq, const void* bk, const void* bv, const int32_t* seq_ids,
                        const int32_t* positions, int hq, const hx_rope_table* table,
                        void* q_out, cudaStream_t s)
{
    if (n == 1)
        return launch_qkv<1, TP, TO>(c, view, x, x_f32, hidden, n, wq, wk, wv, bq, bk, bv,
                                     seq_ids, positions, hq, table, q_out, s);
    if (n == 2)
        return launch_qkv<2, TP, TO>(c, view, x, x_f32, hidden, n, wq, wk, wv, bq, bk, bv,
                                     seq_ids, positions, hq, table, q_out, s);
    if (n <= 4)
        return launch_qkv<4, TP, TO>(c, view, x, x_f32, hidden, n, wq, wk, wv, bq, bk, bv,
                                     seq_ids, positions, hq, table, q_out, s);
    return launch_qkv<8, TP, TO>(c, view, x, x_f32, hidden, n, wq, wk, wv, bq, bk, bv, seq_ids,
                                 positions, hq, table, q_out, s);
}

}  // namespace hx

using namespace hx;

extern "C" int hx_qkv_rope_append(hx_kv_cache* c, int layer, const void* x, int x_dtype,
                                  int hidden, const void* wq, const void* wk, const void* wv,
                                  int proj_dtype, const void* bq, const void* bk, const void* bv,
                                  const int32_t* seq_ids, const int32_t* positions, int n_tokens,
                                  int num_q_heads, const hx_rope_table* table, void* q_out,
                                  int q_out_dtype, hx_stream_t stream)
{
    HX_NVTX_RANGE("hx_qkv_rope_append");
    if (!c) return fail(HX_ERR_INVALID, "null cache");
    if (layer < 0 || layer >= c->cfg.num_layers) return fail(HX_ERR_INVALID, "layer %d out of range", layer);
    if (c->cfg.head_dim != 128)
        return fail(HX_ERR_UNSUPPORTED, "the fused projection needs head_dim 128 (have %d)", c->cfg.head_dim);
    if (n_tokens < 0) return fail(HX_ERR_INVALID, "n_tokens < 0");
    if (n_tokens == 0) return HX_OK;
    if (!x || !wq || !wk || !wv || !seq_ids || !positions)
        return fail(HX_ERR_INVALID, "null x / weights / seq_ids / positions");
    if (hidden < 8 || hidden % 8 || hidden > 8192)
        return fail(HX_ERR_INVALID, "hidden %d must be a multiple of 8 in [8, 8192]", hidden);
    const int hkv = c->cfg.num_kv_heads;
    if (num_q_heads < hkv || num_q_heads % hkv)
        return fail(HX_ERR_INVALID, "num_q_heads %d must be a multiple of kv heads %d", num_q_heads, hkv);
    if ((x_dtype != HX_FP16 && x_dtype != HX_FP32) || (proj_dtype != HX_FP16 && proj_dtype != HX_FP32) ||
        (q_out && q_out_dtype != HX_FP16 && q_out_dtype != HX_FP32))
        return fail(HX_ERR_INVALID, "x / projection / q_out dtype");
    auto misaligned = [](const void* ptr) { return reinterpret_cast<uintptr_t>(ptr) % 16 != 0; };
    if (misaligned(x) || misaligned(wq) || misaligned(wk) || misaligned(wv))
        return fail(HX_ERR_INVALID, "x and the weights must be 16-byte aligned");
    if (table && (table->cfg.head_dim != 128))
        return fail(HX_ERR_INVALID, "rope table head_dim %d != 128", table->cfg.head_dim);
    if (int rc = check_device(c->device, "the cache")) return rc;
    if (table)
        if (int rc = check_device(table->device, "the rope table")) return rc;
    const KVView view = make_view(c, layer);
    cudaStream_t s = (cudaStream_t)stream;
    const int xf = x_dtype == HX_FP32;
    const bool o32 = q_out_dtype == HX_FP32;
    if (proj_dtype == HX_FP16)
        return o32 ? launch_qkv_n<__half, float>(c, view, x, xf, hidden, n_tokens, wq, wk, wv, bq, bk, bv,
                                                 seq_ids, positions, num_q_heads, table, q_out, s)
                   : launch_qkv_n<__half, __half>(c, view, x, xf, hidden, n_tokens, wq, wk, wv, bq, bk,
                                                  bv, seq_ids, positions, num_q_heads, table, q_out, s);
    return o32 ? launch_qkv_n<float, float>(c, view, x, xf, hidden, n_tokens, wq, wk, wv, bq, bk, bv,
                                            seq_ids, positions, num_q_heads, table, q_out, s)
               : launch_qkv_n<float, __half>(c, view, x, xf, hidden, n_tokens, wq, wk, wv, bq, bk, bv,
                                             seq_ids, positions, num_q_heads, table, q_out, s);
}
