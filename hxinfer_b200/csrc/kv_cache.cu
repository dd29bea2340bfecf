// kv_cache.cu — paged head-major KV cache, block allocator, RoPE tables,
// status reporting and the small utility kernels of libhxkv.
//
// Replaces the per-layer token-major cache tensors that AttentionLayer
// allocates with cudaMalloc (hxinfer-engine/include/layer/attention.h:49-51,
// allocator_cuda.cu:6-19).  Layout: one pool
//   [layer][K|V][block][kv_head][64 positions][head_dim] fp16
// so every (block, kv_head) tile is one contiguous, 128-byte aligned run
// that a single TMA box pair covers; a block table maps each sequence's
// logical blocks to physical ones.
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "hx_common.cuh"

namespace hx {

static thread_local std::string t_last_error;

int fail(int code, const char* fmt, ...)
{
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    t_last_error = buf;
    return code;
}

int cuda_fail(cudaError_t e, const char* what)
{
    if (e == cudaSuccess) return HX_OK;
    return fail(e == cudaErrorMemoryAllocation ? HX_ERR_OOM : HX_ERR_CUDA, "%s: %s", what,
                cudaGetErrorString(e));
}

int check_launch(const char* what)
{
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, what);
    return HX_OK;
}

int check_device(int device, const char* what)
{
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
    if (dev != device)
        return fail(HX_ERR_INVALID, "%s lives on device %d but device %d is current", what, device,
                    dev);
    return HX_OK;
}

static std::mutex g_status_mu;
static int* g_status[64] = {nullptr};

int* status_word()
{
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
    std::lock_guard<std::mutex> lk(g_status_mu);
    if (!g_status[dev]) {
        int* p = nullptr;
        if (cudaMalloc(&p, sizeof(int)) != cudaSuccess) return nullptr;
        if (cudaMemset(p, 0, sizeof(int)) != cudaSuccess) return nullptr;
        g_status[dev] = p;
    }
    return g_status[dev];
}

int num_sms()
{
    static std::atomic<int> cached[64];  // zero = not yet read
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64) {
        const int c = cached[dev].load(std::memory_order_relaxed);
        if (c) return c;
    }
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
    if (dev >= 0 && dev < 64) cached[dev].store(n, std::memory_order_relaxed);
    return n;
}

KVView make_view(const hx_kv_cache* c, int layer)
{
    KVView v{};
    v.k = c->k0 + (int64_t)layer * c->layer_stride;
    v.v = c->v0 + (int64_t)layer * c->layer_stride;
    v.table = c->d_table;
    v.mbps = c->mbps;
    v.hkv = c->cfg.num_kv_heads;
    v.hd = c->cfg.head_dim;
    v.capacity = c->cfg.max_tokens_per_seq;
    v.max_seqs = c->cfg.max_seqs;
    v.block_stride = c->block_stride;
    v.head_stride = c->head_stride;
    const int64_t row_bytes = (int64_t)c->cfg.head_dim * 2;
    v.k_row0 = (v.k - c->tm_k_base) / row_bytes;
    v.v_row0 = (v.v - c->tm_v_base) / row_bytes;
    return v;
}

// ---------------------------------------------------------------- tensor maps

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn()
{
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    return fn;
}

// [rows][head_dim] fp16 viewed through 64x64 boxes with 128-byte swizzle.
int encode_rows_map(CUtensorMap* tm, void* base, int head_dim, uint64_t rows)
{
    EncodeTiledFn fn = encode_fn();
    if (!fn) return fail(HX_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
    cuuint64_t gdim[2] = {(cuuint64_t)head_dim, (cuuint64_t)rows};
    cuuint64_t gstride[1] = {(cuuint64_t)head_dim * 2};
    cuuint32_t box[2] = {64, 64};
    cuuint32_t estride[2] = {1, 1};
    CUresult r = fn(tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, base, gdim, gstride, box, estride,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(HX_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    return HX_OK;
}

// ---------------------------------------------------------------- kernels

struct TableChunk {
    int32_t n;
    int32_t ids[960];
};

__global__ void table_update_kernel(int32_t* dst, TableChunk chunk)
{
    for (int i = threadIdx.x; i < chunk.n; i += blockDim.x) dst[i] = chunk.ids[i];
}

// grid (n, hkv, 2): copies one head row of K (z=0) or V (z=1) into the cache.
template <typename T>
__global__ void kv_write_kernel(KVView view, int seq, int start, int n, const T* __restrict__ k,
                               const T* __restrict__ v, int* status)
{
    const int i = blockIdx.x, h = blockIdx.y, which = blockIdx.z;
    const T* src = (which == 0 ? k : v) + ((int64_t)i * view.hkv + h) * view.hd;
    int64_t off = token_offset(view, seq, h, start + i);
    if (off < 0) {
        if (threadIdx.x == 0) record_status(status, HX_ERR_CAPACITY);
        return;
    }
    __half* dst = reinterpret_cast<__half*>((which == 0 ? view.k : view.v) + off);
    for (int d = threadIdx.x; d < view.hd; d += blockDim.x) dst[d] = __float2half_rn((float)src[d]);
}

template <>
__global__ void kv_write_kernel<__half>(KVView view, int seq, int start, int n,
                                        const __half* __restrict__ k,
                                        const __half* __restrict__ v, int* status)
{
    const int i = blockIdx.x, h = blockIdx.y, which = blockIdx.z;
    const __half* src = (which == 0 ? k : v) + ((int64_t)i * view.hkv + h) * view.hd;
    int64_t off = token_offset(view, seq, h, start + i);
    if (off < 0) {
        if (threadIdx.x == 0) record_status(status, HX_ERR_CAPACITY);
        return;
    }
    __half* dst = reinterpret_cast<__half*>((which == 0 ? view.k : view.v) + off);
    for (int d = threadIdx.x; d < view.hd; d += blockDim.x) dst[d] = src[d];
}

__global__ void kv_read_kernel(KVView view, int seq, int start, int n, __half* __restrict__ k,
                               __half* __restrict__ v, int* status)
{
    const int i = blockIdx.x, h = blockIdx.y, which = blockIdx.z;
    __half* dst = (which == 0 ? k : v);
    if (!dst) return;
    dst += ((int64_t)i * view.hkv + h) * view.hd;
    int64_t off = token_offset(view, seq, h, start + i);
    if (off < 0) {
        if (threadIdx.x == 0) record_status(status, HX_ERR_CAPACITY);
        return;
    }
    const __half* src = reinterpret_cast<const __half*>((which == 0 ? view.k : view.v) + off);
    for (int d = threadIdx.x; d < view.hd; d += blockDim.x) dst[d] = src[d];
}

__device__ __forceinline__ uint64_t mix64(uint64_t z)
{
    z += 0x9e3779b97f4a7c15ull;
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
    return z ^ (z >> 31);
}

// Writes N(0,1) fp16 values (Box-Muller on a counter hash) over n8 16-byte
// groups of 8 halves.
__global__ void fill_normal_kernel(uint4* __restrict__ dst, uint64_t n8, uint64_t seed)
{
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    for (uint64_t g = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; g < n8; g += stride) {
        uint32_t w[4];
#pragma unroll
        for (int p = 0; p < 4; ++p) {
            uint64_t r = mix64(seed ^ mix64(g * 4 + p));
            float u1 = ((uint32_t)(r >> 40) + 1u) * (1.0f / 16777216.0f);  // (0, 1]
            float u2 = (uint32_t)(r & 0xffffffu) * (1.0f / 16777216.0f);   // [0, 1)
            float rad = sqrtf(-2.0f * __logf(u1));
            float s, c;
            __sincosf(6.283185307179586f * u2, &s, &c);
            w[p] = pack_half2(rad * c, rad * s);
        }
        dst[g] = make_uint4(w[0], w[1], w[2], w[3]);
    }
}

}  // namespace hx

using namespace hx;

// ---------------------------------------------------------------- C ABI

extern "C" const char* hx_status_string(int s)
{
    switch (s) {
    case HX_OK: return "ok";
    case HX_ERR_INVALID: return "invalid argument";
    case HX_ERR_CAPACITY: return "capacity exceeded";
    case HX_ERR_OOM: return "out of memory";
    case HX_ERR_CUDA: return "CUDA error";
    case HX_ERR_NCCL: return "collective error";
    case HX_ERR_TIMEOUT: return "device wait timed out";
    case HX_ERR_NOT_FOUND: return "not found";
    case HX_ERR_UNSUPPORTED: return "unsupported";
    default: return "unknown status";
    }
}

extern "C" const char* hx_last_error(void) { return t_last_error.c_str(); }

extern "C" int hx_device_status(int clear)
{
    int* w = status_word();
    if (!w) return fail(HX_ERR_CUDA, "no device status word");
    HX_CUDA_TRY(cudaDeviceSynchronize());
    int v = 0;
    HX_CUDA_TRY(cudaMemcpy(&v, w, sizeof v, cudaMemcpyDeviceToHost));
    if (clear) {
        HX_CUDA_TRY(cudaMemset(w, 0, sizeof(int)));
        // the reset must land before later launches on non-blocking streams run
        HX_CUDA_TRY(cudaDeviceSynchronize());
    }
    if (v != HX_OK) fail(v, "a kernel recorded: %s", hx_status_string(v));
    return v;
}

static int validate_cfg(const hx_kv_config* c)
{
    if (!c) return fail(HX_ERR_INVALID, "null config");
    if (c->num_layers < 1 || c->num_kv_heads < 1 || c->max_seqs < 1 || c->max_tokens_per_seq < 1)
        return fail(HX_ERR_INVALID, "config fields must be positive");
    if (c->head_dim < 2 || c->head_dim > kMaxHeadDim || (c->head_dim & 1))
        return fail(HX_ERR_INVALID, "head_dim %d must be even and <= %d", c->head_dim, kMaxHeadDim);
    if (c->num_blocks < 0) return fail(HX_ERR_INVALID, "num_blocks < 0");
    return HX_OK;
}

extern "C" int hx_kv_create(const hx_kv_config* cfg, hx_kv_cache** out)
{
    if (!out) return fail(HX_ERR_INVALID, "null out");
    *out = nullptr;
    if (int rc = validate_cfg(cfg)) return rc;
    auto* c = new (std::nothrow) hx_kv_cache();
    if (!c) return fail(HX_ERR_OOM, "host allocation");
    c->cfg = *cfg;
    cudaGetDevice(&c->device);
    c->mbps = (cfg->max_tokens_per_seq + kBlockTokens - 1) / kBlockTokens;
    c->num_blocks = cfg->num_blocks ? cfg->num_blocks : (int64_t)cfg->max_seqs * c->mbps;
    c->head_stride = (int64_t)kBlockTokens * cfg->head_dim * 2;
    c->block_stride = c->head_stride * cfg->num_kv_heads;
    c->kv_stride = c->block_stride * c->num_blocks;
    c->layer_stride = 2 * c->kv_stride;
    c->pool_bytes = (size_t)c->layer_stride * cfg->num_layers;
    cudaError_t e = cudaMalloc(&c->pool, c->pool_bytes);
    if (e != cudaSuccess) {
        delete c;
        return fail(HX_ERR_OOM, "pool of %zu bytes: %s", (size_t)0 + (size_t)c->pool_bytes,
                    cudaGetErrorString(e));
    }
    c->k0 = c->pool;
    c->v0 = c->pool + c->kv_stride;
    size_t tbytes = sizeof(int32_t) * (size_t)cfg->max_seqs * c->mbps;
    e = cudaMalloc(&c->d_table, tbytes);
    if (e == cudaSuccess) e = cudaMemset(c->d_table, 0xff, tbytes);
    if (e == cudaSuccess) e = cudaMemset(c->pool, 0, c->pool_bytes);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
        int rc = cuda_fail(e, "cache allocation");
        hx_kv_destroy(c);
        return rc;
    }
    c->h_table.assign((size_t)cfg->max_seqs * c->mbps, -1);
    c->n_mapped.assign(cfg->max_seqs, 0);
    c->free_list.resize(c->num_blocks);
    for (int64_t b = 0; b < c->num_blocks; ++b) c->free_list[b] = (int32_t)(c->num_blocks - 1 - b);
    c->tm_k_base = c->tm_v_base = c->pool;
    if (cfg->head_dim == 128) {
        uint64_t rows = c->pool_bytes / (cfg->head_dim * 2);
        if (rows < (1ull << 31)) {
            if (int rc = encode_rows_map(&c->tm_k, c->pool, cfg->head_dim, rows)) {
                hx_kv_destroy(c);
                return rc;
            }
            c->tm_v = c->tm_k;
            c->has_tmap = true;
        }
    }
    if (int rc = decode_prepare_device(c)) {
        hx_kv_destroy(c);
        return rc;
    }
    *out = c;
    return HX_OK;
}

extern "C" int hx_kv_wrap(void* k_base, void* v_base, int num_kv_heads, int head_dim,
                          int capacity, hx_kv_cache** out)
{
    if (!out) return fail(HX_ERR_INVALID, "null out");
    *out = nullptr;
    if (!k_base || !v_base) return fail(HX_ERR_INVALID, "null cache pointer");
    hx_kv_config cfg{};
    cfg.num_layers = 1;
    cfg.num_kv_heads = num_kv_heads;
    cfg.head_dim = head_dim;
    cfg.max_seqs = 1;
    cfg.max_tokens_per_seq = capacity;
    if (int rc = validate_cfg(&cfg)) return rc;
    if ((reinterpret_cast<uintptr_t>(k_base) | reinterpret_cast<uintptr_t>(v_base)) & 15)
        return fail(HX_ERR_INVALID, "cache pointers must be 16-byte aligned");
    auto* c = new (std::nothrow) hx_kv_cache();
    if (!c) return fail(HX_ERR_OOM, "host allocation");
    c->cfg = cfg;
    c->wrapped = true;
    cudaGetDevice(&c->device);
    c->mbps = (capacity + kBlockTokens - 1) / kBlockTokens;
    c->num_blocks = c->mbps;
    c->head_stride = (int64_t)capacity * head_dim * 2;  // contiguous [kv_head][capacity][hd]
    c->block_stride = (int64_t)kBlockTokens * head_dim * 2;
    c->layer_stride = 0;
    c->k0 = static_cast<char*>(k_base);
    c->v0 = static_cast<char*>(v_base);
    c->tm_k_base = c->k0;
    c->tm_v_base = c->v0;
    c->n_mapped.assign(1, c->mbps);
    if (head_dim == 128) {
        uint64_t rows = (uint64_t)num_kv_heads * capacity;
        int rc = encode_rows_map(&c->tm_k, c->k0, head_dim, rows);
        if (!rc) rc = encode_rows_map(&c->tm_v, c->v0, head_dim, rows);
        if (rc) {
            delete c;
            return rc;
        }
        c->has_tmap = true;
    }
    if (int rc = decode_prepare_device(c)) {
        delete c;
        return rc;
    }
    *out = c;
    return HX_OK;
}

extern "C" int hx_kv_destroy(hx_kv_cache* c)
{
    if (!c) return HX_OK;
    if (c->pool) cudaFree(c->pool);
    if (c->d_table) cudaFree(c->d_table);
    delete c;
    return HX_OK;
}

extern "C" int hx_kv_get_info(const hx_kv_cache* c, hx_kv_info* o)
{
    if (!c || !o) return fail(HX_ERR_INVALID, "null argument");
    o->num_layers = c->cfg.num_layers;
    o->num_kv_heads = c->cfg.num_kv_heads;
    o->head_dim = c->cfg.head_dim;
    o->max_seqs = c->cfg.max_seqs;
    o->max_blocks_per_seq = c->mbps;
    o->num_blocks = c->num_blocks;
    o->free_blocks = (int64_t)c->free_list.size();
    o->pool = c->pool;
    o->pool_bytes = c->pool_bytes;
    o->layer_stride_bytes = c->layer_stride;
    o->kv_stride_bytes = c->kv_stride;
    o->block_stride_bytes = c->block_stride;
    o->head_stride_bytes = c->head_stride;
    o->block_table = c->d_table;
    return HX_OK;
}

static int push_table_range(hx_kv_cache* c, int seq, int first, int count, cudaStream_t stream)
{
    for (int done = 0; done < count;) {
        TableChunk ch;
        ch.n = std::min(count - done, 960);
        std::memcpy(ch.ids, &c->h_table[(size_t)seq * c->mbps + first + done], sizeof(int32_t) * ch.n);
        table_update_kernel<<<1, 256, 0, stream>>>(c->d_table + (size_t)seq * c->mbps + first + done, ch);
        if (int rc = check_launch("table_update_kernel")) return rc;
        done += ch.n;
    }
    return HX_OK;
}

extern "C" int hx_kv_reserve(hx_kv_cache* c, int seq, int n_tokens, hx_stream_t stream)
{
    if (!c) return fail(HX_ERR_INVALID, "null cache");
    if (seq < 0 || seq >= c->cfg.max_seqs) return fail(HX_ERR_INVALID, "seq %d out of range", seq);
    if (n_tokens < 0 || n_tokens > c->cfg.max_tokens_per_seq)
        return fail(HX_ERR_CAPACITY, "%d positions exceed the per-sequence capacity %d", n_tokens,
                    c->cfg.max_tokens_per_seq);
    if (c->wrapped) return HX_OK;  // fully mapped by construction
    if (int rc = check_device(c->device, "the cache")) return rc;
    int need = (n_tokens + kBlockTokens - 1) / kBlockTokens;
    int have = c->n_mapped[seq];
    if (need <= have) return HX_OK;
    if ((int64_t)(need - have) > (int64_t)c->free_list.size())
        return fail(HX_ERR_CAPACITY, "pool exhausted: need %d blocks, %zu free", need - have,
                    c->free_list.size());
    for (int b = have; b < need; ++b) {
        c->h_table[(size_t)seq * c->mbps + b] = c->free_list.back();
        c->free_list.pop_back();
    }
    c->n_mapped[seq] = need;
    return push_table_range(c, seq, have, need - have, (cudaStream_t)stream);
}

extern "C" int hx_kv_release(hx_kv_cache* c, int seq, hx_stream_t stream)
{
    if (!c) return fail(HX_ERR_INVALID, "null cache");
    if (seq < 0 || seq >= c->cfg.max_seqs) return fail(HX_ERR_INVALID, "seq %d out of range", seq);
    if (c->wrapped) return HX_OK;
    if (int rc = check_device(c->device, "the cache")) return rc;
    int have = c->n_mapped[seq];
    for (int b = 0; b < have; ++b) {
        int32_t& e = c->h_table[(size_t)seq * c->mbps + b];
        c->free_list.push_back(e);
        e = -1;
    }
    c->n_mapped[seq] = 0;
    return push_table_range(c, seq, 0, have, (cudaStream_t)stream);
}

static int check_range(const hx_kv_cache* c, int layer, int seq, int start, int n)
{
    if (!c) return fail(HX_ERR_INVALID, "null cache");
    if (layer < 0 || layer >= c->cfg.num_layers) return fail(HX_ERR_INVALID, "layer %d out of range", layer);
    if (seq < 0 || seq >= c->cfg.max_seqs) return fail(HX_ERR_INVALID, "seq %d out of range", seq);
    if (start < 0 || n < 0 || (int64_t)start + n > (int64_t)c->n_mapped[seq] * kBlockTokens ||
        (int64_t)start + n > c->cfg.max_tokens_per_seq)
        return fail(HX_ERR_CAPACITY, "positions [%d, %d) not reserved for seq %d", start, start + n, seq);
    return check_device(c->device, "the cache");
}

extern "C" int hx_kv_write(hx_kv_cache* c, int layer, int seq, int start, int n, const void* k,
                           const void* v, int dtype, hx_stream_t stream)
{
    if (int rc = check_range(c, layer, seq, start, n)) return rc;
    if (!k || !v) return fail(HX_ERR_INVALID, "null k/v");
    if (n == 0) return HX_OK;
    KVView view = make_view(c, layer);
    dim3 grid(n, c->cfg.num_kv_heads, 2);
    int threads = std::min(128, c->cfg.head_dim);
    if (dtype == HX_FP16)
        kv_write_kernel<__half><<<grid, threads, 0, (cudaStream_t)stream>>>(
            view, seq, start, n, (const __half*)k, (const __half*)v, status_word());
    else if (dtype == HX_FP32)
        kv_write_kernel<float><<<grid, threads, 0, (cudaStream_t)stream>>>(
            view, seq, start, n, (const float*)k, (const float*)v, status_word());
    else
        return fail(HX_ERR_INVALID, "dtype %d", dtype);
    return check_launch("kv_write_kernel");
}

extern "C" int hx_kv_read(const hx_kv_cache* c, int layer, int seq, int start, int n, void* k,
                          void* v, hx_stream_t stream)
{
    if (int rc = check_range(c, layer, seq, start, n)) return rc;
    if (n == 0 || (!k && !v)) return HX_OK;
    KVView view = make_view(c, layer);
    dim3 grid(n, c->cfg.num_kv_heads, 2);
    kv_read_kernel<<<grid, std::min(128, c->cfg.head_dim), 0, (cudaStream_t)stream>>>(
        view, seq, start, n, (__half*)k, (__half*)v, status_word());
    return check_launch("kv_read_kernel");
}

extern "C" int hx_kv_fill_normal(hx_kv_cache* c, uint64_t seed, hx_stream_t stream)
{
    if (!c) return fail(HX_ERR_INVALID, "null cache");
    if (int rc = check_device(c->device, "the cache")) return rc;
    auto launch = [&](void* base, size_t bytes, uint64_t s) {
        uint64_t n8 = bytes / 16;
        int blocks = num_sms() * 8;
        fill_normal_kernel<<<blocks, 256, 0, (cudaStream_t)stream>>>((uint4*)base, n8, s);
        return check_launch("fill_normal_kernel");
    };
    if (!c->wrapped) return launch(c->pool, c->pool_bytes, seed);
    size_t bytes = (size_t)c->cfg.num_kv_heads * c->cfg.max_tokens_per_seq * c->cfg.head_dim * 2;
    if (int rc = launch(c->k0, bytes, seed)) return rc;
    return launch(c->v0, bytes, seed ^ 0x5bd1e995ull);
}

// ---------------------------------------------------------------- RoPE tables

// YaRN helpers: the formulas of the reference's host code
// (hxinfer-engine/src/op/cuda/rope_cuda.cu:9-35).
static float yarn_correction_dim(int num_rotations, int dim, float base, int max_pos)
{
    const double pi = 3.14159265358979323846;
    double q = max_pos / ((double)(num_rotations * 2.0f) * pi);
    return (dim * logf((float)q)) / (2.0f * logf(base));
}

extern "C" int hx_rope_table_create(const hx_rope_config* cfg, hx_rope_table** out)
{
    if (!cfg || !out) return fail(HX_ERR_INVALID, "null argument");
    *out = nullptr;
    if (cfg->head_dim < 2 || (cfg->head_dim & 1) || cfg->head_dim > kMaxHeadDim || cfg->max_pos < 1)
        return fail(HX_ERR_INVALID, "bad rope config (head_dim %d, max_pos %d)", cfg->head_dim,
                    cfg->max_pos);
    const int half = cfg->head_dim / 2;
    std::vector<float> yarn(half, 1.0f);
    float attn_factor = 1.0f;
    if (cfg->use_yarn) {
        float low = yarn_correction_dim((int)cfg->yarn_beta_fast, cfg->head_dim, cfg->theta,
                                        cfg->yarn_orig_max_pos);
        float high = yarn_correction_dim((int)cfg->yarn_beta_slow, cfg->head_dim, cfg->theta,
                                         cfg->yarn_orig_max_pos);
        low = fmaxf(low, 0.0f);
        high = fminf(high, (float)(half - 1));
        float span = high - low;
        if (span <= 0.0f) span = 1.0f;
        for (int d = 0; d < half; d++) {
            float ramp = ((float)d - low) / span;
            ramp = fmaxf(0.0f, fminf(1.0f, ramp));
            yarn[d] = 1.0f - ramp * (1.0f - 1.0f / cfg->yarn_factor);
        }
        attn_factor = cfg->yarn_factor <= 1.0f ? 1.0f : 0.1f * logf(cfg->yarn_factor) + 1.0f;
    }
    // The angle and cos/sin are the expressions of rope_cpu.cpp:22-25 (or of
    // rope_cuda.cu:56-61 with YaRN), evaluated by the host libm so the table
    // holds exactly the values the reference CPU op rotates with.
    std::vector<float> freq(half);
    for (int d = 0; d < half; d++) {
        float scale = 1.0f / powf(cfg->theta, (float)(2 * d) / cfg->head_dim);
        if (cfg->use_yarn) scale *= yarn[d];
        freq[d] = scale;
    }
    std::vector<float2> host((size_t)cfg->max_pos * half);
    for (int p = 0; p < cfg->max_pos; p++) {
        for (int d = 0; d < half; d++) {
            float angle = p * freq[d];
            float c = cosf(angle), s = sinf(angle);
            if (cfg->use_yarn) {
                c = c * attn_factor;
                s = s * attn_factor;
            }
            host[(size_t)p * half + d] = make_float2(c, s);
        }
    }
    auto* t = new (std::nothrow) hx_rope_table();
    if (!t) return fail(HX_ERR_OOM, "host allocation");
    t->cfg = *cfg;
    cudaGetDevice(&t->device);
    size_t bytes = sizeof(float2) * host.size();
    cudaError_t e = cudaMalloc(&t->d_cos_sin, bytes);
    if (e == cudaSuccess) e = cudaMemcpy(t->d_cos_sin, host.data(), bytes, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
        int rc = cuda_fail(e, "rope table upload");
        hx_rope_table_destroy(t);
        return rc;
    }
    *out = t;
    return HX_OK;
}

extern "C" int hx_rope_table_destroy(hx_rope_table* t)
{
    if (!t) return HX_OK;
    if (t->d_cos_sin) cudaFree(t->d_cos_sin);
    delete t;
    return HX_OK;
}

extern "C" uint64_t hx_prefix_hash(const int32_t* tokens, size_t n)
{
    uint64_t h = 0xcbf29ce484222325ull;  // FNV-1a 64 offset basis
    for (size_t i = 0; i < n; i++) {
        h ^= (uint64_t)(int64_t)tokens[i];
        h *= 0x100000001b3ull;  // FNV-1a 64 prime
    }
    return h;
}
