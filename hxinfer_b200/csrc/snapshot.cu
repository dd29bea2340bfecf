// snapshot.cu — K4: prefix-cache snapshot / restore copies on the device.
//
// Replaces the host std::memcpy of PrefixCacheManager::store / restore
// (hxinfer-engine/include/cache/prefix_cache.h:78-89, 135-147), which copies
// the first prefix_len rows of every layer's K and V.  Here one launch copies
// all layers: each (layer, K|V, kv head, block) run is contiguous in both the
// cache and the snapshot, so a CTA streams it with 16-byte vectors (2-byte
// elements when head_dim*2 is not a multiple of 16), streaming cache hints.
// Snapshot layout: [layer][K|V][kv_head][prefix_len][head_dim] fp16, dense.  Positions >= prefix_len are never read or written.
#include "hx_common.cuh"

namespace hx {

// Per-layer K and V base addresses of up to kSnapMaxLayers one-layer caches
// (passed by value: no device table to allocate).  n = 0: the layers are the
// layers of one cache, layer_stride apart.
constexpr int kSnapMaxLayers = 64;
struct LayerBases {
    int n;
    char* k[kSnapMaxLayers];
    char* v[kSnapMaxLayers];
};

__device__ __forceinline__ char* layer_base(const KVView& v0, const LayerBases& lb,
                                            int64_t layer_stride, int64_t layer, int kv)
{
    if (lb.n) return kv ? lb.v[layer] : lb.k[layer];
    return (kv ? v0.v : v0.k) + layer * layer_stride;
}

// One work item = the positions of one block of one (layer, K|V, kv head):
// a contiguous run of up to 64 rows in the cache and in the snapshot.  A CTA
// copies it with every thread holding four 16-byte vectors in flight.
// Row bytes (head_dim * 2) must be a multiple of 16 here.
template <bool TO_SNAPSHOT>
__global__ void __launch_bounds__(256)
    snapshot_block_kernel(KVView v0, int64_t layer_stride, const LayerBases lb, int layers, int seq,
                          int prefix_len, uint4* __restrict__ snap, int* status)
{
    const int row_vecs = v0.hd * 2 / 16;
    const int nblk = (prefix_len + kBlockTokens - 1) / kBlockTokens;
    const int64_t items = (int64_t)layers * 2 * v0.hkv * nblk;
    for (int64_t it = blockIdx.x; it < items; it += gridDim.x) {
        const int blk = (int)(it % nblk);
        const int64_t plane = it / nblk;  // (layer, kv, head)
        const int h = (int)(plane % v0.hkv);
        const int64_t lkv = plane / v0.hkv;
        const int kv = (int)(lkv & 1);
        const int64_t layer = lkv >> 1;
        const int64_t pb = phys_block(v0, seq, blk);
        if (pb < 0) {
            if (threadIdx.x == 0) record_status(status, HX_ERR_CAPACITY);
            continue;
        }
        const int rows = min(kBlockTokens, prefix_len - blk * kBlockTokens);
        const int nvec = rows * row_vecs;
        uint4* cache = reinterpret_cast<uint4*>(layer_base(v0, lb, layer_stride, layer, kv) +
                                                pb * v0.block_stride + (int64_t)h * v0.head_stride);
        uint4* dst = snap + (plane * prefix_len + (int64_t)blk * kBlockTokens) * row_vecs;
        uint4* from = TO_SNAPSHOT ? cache : dst;
        uint4* to = TO_SNAPSHOT ? dst : cache;
        for (int base = 0; base < nvec; base += 4 * 256) {
            uint4 x[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int e = base + u * 256 + threadIdx.x;
                if (e < nvec) x[u] = __ldcs(from + e);
            }
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int e = base + u * 256 + threadIdx.x;
                if (e < nvec) __stcs(to + e, x[u]);
            }
        }
    }
}

// Any even head_dim: one 2-byte element per work unit.
template <bool TO_SNAPSHOT>
__global__ void snapshot_elem_kernel(KVView v0, int64_t layer_stride, const LayerBases lb, int layers,
                                     int seq, int prefix_len, uint16_t* __restrict__ snap, int* status)
{
    const int hd = v0.hd;
    const int64_t total = (int64_t)layers * 2 * v0.hkv * prefix_len * hd;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t u = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; u < total; u += stride) {
        const int d = (int)(u % hd);
        const int64_t row = u / hd;
        const int pos = (int)(row % prefix_len);
        const int64_t plane = row / prefix_len;
        const int h = (int)(plane % v0.hkv);
        const int64_t lkv = plane / v0.hkv;
        const int64_t off = token_offset(v0, seq, h, pos);
        if (off < 0) {
            record_status(status, HX_ERR_CAPACITY);
            continue;
        }
        uint16_t* cache = reinterpret_cast<uint16_t*>(
                              layer_base(v0, lb, layer_stride, lkv >> 1, (int)(lkv & 1)) + off) + d;
        if (TO_SNAPSHOT)
            snap[u] = *cache;
        else
            *cache = snap[u];
    }
}

// Copies `layers` layers: those of cache c (lb.n == 0) or the one-layer
// caches whose bases lb holds (c is the first of them, for the geometry).
template <bool TO_SNAPSHOT>
static int launch_copy(const hx_kv_cache* c, const LayerBases& lb, int layers, int seq,
                       int prefix_len, void* buf, cudaStream_t stream)
{
    KVView v = make_view(c, 0);
    const int hd_bytes = c->cfg.head_dim * 2;
    if (hd_bytes % 16 == 0) {
        const int nblk = (prefix_len + kBlockTokens - 1) / kBlockTokens;
        const int64_t items = (int64_t)layers * 2 * c->cfg.num_kv_heads * nblk;
        // one CTA per run (grid-stride only past 2^20 runs): a fixed grid of
        // 16 CTAs per SM left a partial last round of runs (7168 runs over 2368
        // CTAs for a 28-layer, 2048-position snapshot)
        const int blocks = (int)std::min<int64_t>(items, int64_t(1) << 20);
        snapshot_block_kernel<TO_SNAPSHOT><<<blocks, 256, 0, stream>>>(
            v, c->layer_stride, lb, layers, seq, prefix_len, (uint4*)buf, status_word());
        return check_launch("snapshot_block_kernel");
    }
    const int64_t units = (int64_t)layers * 2 * c->cfg.num_kv_heads * prefix_len * c->cfg.head_dim;
    const int blocks = (int)std::max<int64_t>(1, std::min<int64_t>((units + 255) / 256, (int64_t)num_sms() * 16));
    snapshot_elem_kernel<TO_SNAPSHOT><<<blocks, 256, 0, stream>>>(
        v, c->layer_stride, lb, layers, seq, prefix_len, (uint16_t*)buf, status_word());
    return check_launch("snapshot_elem_kernel");
}

}  // namespace hx

using namespace hx;

extern "C" size_t hx_snapshot_bytes(const hx_kv_cache* c, int prefix_len)
{
    if (!c || prefix_len < 0) return 0;
    return (size_t)c->cfg.num_layers * 2 * c->cfg.num_kv_heads * prefix_len * c->cfg.head_dim * 2;
}

// The copy kernels read and write the snapshot buffer directly: it must be
// device, managed or mapped pinned memory.  A pageable host pointer would be
// an illegal address on the device, so one that the runtime reports as
// unregistered (or as pinned but unmapped) host memory is refused here,
// before any launch.  A pointer the query cannot classify is passed on as
// before.
static int check_device_accessible(const void* p)
{
    cudaPointerAttributes a{};
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();  // the query's error is not sticky: clear it for later calls
        return HX_OK;
    }
    if (a.type == cudaMemoryTypeUnregistered || (a.type == cudaMemoryTypeHost && !a.devicePointer))
        return fail(HX_ERR_INVALID, "snapshot buffer is pageable host memory; pass device, managed "
                                    "or mapped pinned memory");
    return HX_OK;
}

static int check_snapshot_args(const hx_kv_cache* c, int seq, int prefix_len, const void* buf,
                               size_t bytes)
{
    if (!c) return fail(HX_ERR_INVALID, "null cache");
    if (seq < 0 || seq >= c->cfg.max_seqs) return fail(HX_ERR_INVALID, "seq %d out of range", seq);
    if (prefix_len < 0 || prefix_len > c->cfg.max_tokens_per_seq)
        return fail(HX_ERR_CAPACITY, "prefix_len %d outside [0, %d]", prefix_len, c->cfg.max_tokens_per_seq);
    if ((int64_t)prefix_len > (int64_t)c->n_mapped[seq] * kBlockTokens)
        return fail(HX_ERR_CAPACITY, "seq %d holds only %d reserved positions", seq,
                    c->n_mapped[seq] * kBlockTokens);
    if (prefix_len > 0 && !buf) return fail(HX_ERR_INVALID, "null snapshot buffer");
    if (bytes < hx_snapshot_bytes(c, prefix_len))
        return fail(HX_ERR_INVALID, "snapshot buffer of %zu bytes < %zu needed", bytes,
                    hx_snapshot_bytes(c, prefix_len));
    if (reinterpret_cast<uintptr_t>(buf) & 15) return fail(HX_ERR_INVALID, "snapshot buffer not 16-byte aligned");
    if (prefix_len == 0) return HX_OK;
    if (int rc = check_device(c->device, "the cache")) return rc;
    return check_device_accessible(buf);
}

extern "C" int hx_kv_snapshot(const hx_kv_cache* c, int seq, int prefix_len, void* dst,
                              size_t dst_bytes, hx_stream_t stream)
{
    HX_NVTX_RANGE("hx_kv_snapshot");
    if (int rc = check_snapshot_args(c, seq, prefix_len, dst, dst_bytes)) return rc;
    if (prefix_len == 0) return HX_OK;
    LayerBases none{};
    return launch_copy<true>(c, none, c->cfg.num_layers, seq, prefix_len, dst, (cudaStream_t)stream);
}

extern "C" int hx_kv_restore(hx_kv_cache* c, int seq, int prefix_len, const void* src,
                             size_t src_bytes, hx_stream_t stream)
{
    HX_NVTX_RANGE("hx_kv_restore");
    if (int rc = check_snapshot_args(c, seq, prefix_len, src, src_bytes)) return rc;
    if (prefix_len == 0) return HX_OK;
    LayerBases none{};
    return launch_copy<false>(c, none, c->cfg.num_layers, seq, prefix_len, const_cast<void*>(src),
                              (cudaStream_t)stream);
}

// ------------------------------------------------------------ layers of separate caches

// All caches: one-layer caches made by hx_kv_wrap with the geometry of the
// first, on its device; fills lb with their bases.
static int check_layer_caches(const hx_kv_cache* const* caches, int n, int prefix_len,
                              const void* buf, size_t bytes, LayerBases& lb)
{
    if (!caches || n < 1) return fail(HX_ERR_INVALID, "no caches");
    if (n > kSnapMaxLayers) return fail(HX_ERR_INVALID, "%d caches; at most %d per call", n, kSnapMaxLayers);
    const hx_kv_cache* c0 = caches[0];
    for (int i = 0; i < n; ++i) {
        const hx_kv_cache* c = caches[i];
        if (!c) return fail(HX_ERR_INVALID, "null cache %d", i);
        if (!c->wrapped || c->cfg.num_layers != 1 || c->cfg.num_kv_heads != c0->cfg.num_kv_heads ||
            c->cfg.head_dim != c0->cfg.head_dim || c->cfg.max_tokens_per_seq != c0->cfg.max_tokens_per_seq ||
            c->device != c0->device)
            return fail(HX_ERR_INVALID, "cache %d is not a one-layer wrapped cache shaped like cache 0", i);
        lb.k[i] = c->k0;
        lb.v[i] = c->v0;
    }
    lb.n = n;
    if (prefix_len < 0 || prefix_len > c0->cfg.max_tokens_per_seq)
        return fail(HX_ERR_CAPACITY, "prefix_len %d outside [0, %d]", prefix_len, c0->cfg.max_tokens_per_seq);
    const size_t need = (size_t)n * hx_snapshot_bytes(c0, prefix_len);
    if (prefix_len > 0 && !buf) return fail(HX_ERR_INVALID, "null snapshot buffer");
    if (bytes < need) return fail(HX_ERR_INVALID, "snapshot buffer of %zu bytes < %zu needed", bytes, need);
    if (reinterpret_cast<uintptr_t>(buf) & 15) return fail(HX_ERR_INVALID, "snapshot buffer not 16-byte aligned");
    if (prefix_len == 0) return HX_OK;
    if (int rc = check_device(c0->device, "the caches")) return rc;
    return check_device_accessible(buf);
}

extern "C" int hx_kv_snapshot_layers(const hx_kv_cache* const* caches, int n_caches, int prefix_len,
                                     void* dst, size_t dst_bytes, hx_stream_t stream)
{
    HX_NVTX_RANGE("hx_kv_snapshot_layers");
    LayerBases lb{};
    if (int rc = check_layer_caches(caches, n_caches, prefix_len, dst, dst_bytes, lb)) return rc;
    if (prefix_len == 0) return HX_OK;
    return launch_copy<true>(caches[0], lb, n_caches, 0, prefix_len, dst, (cudaStream_t)stream);
}

extern "C" int hx_kv_restore_layers(hx_kv_cache* const* caches, int n_caches, int prefix_len,
                                    const void* src, size_t src_bytes, hx_stream_t stream)
{
    HX_NVTX_RANGE("hx_kv_restore_layers");
    LayerBases lb{};
    if (int rc = check_layer_caches(caches, n_caches, prefix_len, src, src_bytes, lb)) return rc;
    if (prefix_len == 0) return HX_OK;
    return launch_copy<false>(caches[0], lb, n_caches, 0, prefix_len, const_cast<void*>(src),
                              (cudaStream_t)stream);
}
