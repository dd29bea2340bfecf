// snapshot.cu — K4: prefix-cache snapshot / restore copies on the device.
//
// Replaces the host std::memcpy of PrefixCacheManager::store / restore
// (hxinfer-engine/include/cache/prefix_cache.h:78-89, 135-147), which copies
// the first prefix_len rows of every layer's K and V.  Here one launch copies
// all layers: 16-byte vector loads/stores (2-byte elements when head_dim*2 is
// not a multiple of 16), grid-stride over the payload, so the copy runs at
// HBM copy speed.  Snapshot layout: [layer][K|V][kv_head][prefix_len][head_dim]
// fp16, dense.  Positions >= prefix_len are never read or written.
#include "hx_common.cuh"

namespace hx {

// One work unit = `unit` bytes of one position row of one (layer, K|V, head).
template <typename U, bool TO_SNAPSHOT>
__global__ void snapshot_copy_kernel(KVView v0, int64_t layer_stride, int layers, int seq,
                                     int prefix_len, U* __restrict__ snap, int* status)
{
    const int hd_bytes = v0.hd * 2;
    const int per_row = hd_bytes / (int)sizeof(U);
    const int64_t rows_per_plane = (int64_t)v0.hkv * prefix_len;
    const int64_t total = (int64_t)layers * 2 * rows_per_plane * per_row;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t u = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; u < total; u += stride) {
        const int sub = (int)(u % per_row);
        const int64_t row = u / per_row;
        const int pos = (int)(row % prefix_len);
        const int64_t hp = row / prefix_len;  // (layer, kv, head)
        const int h = (int)(hp % v0.hkv);
        const int64_t lkv = hp / v0.hkv;
        const int kv = (int)(lkv & 1);
        const int64_t layer = lkv >> 1;
        const int64_t off = token_offset(v0, seq, h, pos);
        if (off < 0) {
            record_status(status, HX_ERR_CAPACITY);
            continue;
        }
        char* base = (kv ? v0.v : v0.k) + layer * layer_stride + off;
        U* cache = reinterpret_cast<U*>(base) + sub;
        if (TO_SNAPSHOT)
            snap[u] = *cache;
        else
            *cache = snap[u];
    }
}

template <bool TO_SNAPSHOT>
static int launch_copy(const hx_kv_cache* c, int seq, int prefix_len, void* buf,
                       cudaStream_t stream)
{
    KVView v = make_view(c, 0);
    const int hd_bytes = c->cfg.head_dim * 2;
    const int64_t bytes = (int64_t)c->cfg.num_layers * 2 * c->cfg.num_kv_heads * prefix_len * hd_bytes;
    const int unit = (hd_bytes % 16 == 0) ? 16 : 2;
    const int64_t units = bytes / unit;
    int blocks = (int)std::min<int64_t>((units + 255) / 256, (int64_t)num_sms() * 16);
    if (blocks < 1) blocks = 1;
    if (unit == 16)
        snapshot_copy_kernel<uint4, TO_SNAPSHOT><<<blocks, 256, 0, stream>>>(
            v, c->layer_stride, c->cfg.num_layers, seq, prefix_len, (uint4*)buf, status_word());
    else
        snapshot_copy_kernel<uint16_t, TO_SNAPSHOT><<<blocks, 256, 0, stream>>>(
            v, c->layer_stride, c->cfg.num_layers, seq, prefix_len, (uint16_t*)buf, status_word());
    return check_launch("snapshot_copy_kernel");
}

}  // namespace hx

using namespace hx;

extern "C" size_t hx_snapshot_bytes(const hx_kv_cache* c, int prefix_len)
{
    if (!c || prefix_len < 0) return 0;
    return (size_t)c->cfg.num_layers * 2 * c->cfg.num_kv_heads * prefix_len * c->cfg.head_dim * 2;
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
    return HX_OK;
}

extern "C" int hx_kv_snapshot(const hx_kv_cache* c, int seq, int prefix_len, void* dst,
                              size_t dst_bytes, hx_stream_t stream)
{
    if (int rc = check_snapshot_args(c, seq, prefix_len, dst, dst_bytes)) return rc;
    if (prefix_len == 0) return HX_OK;
    return launch_copy<true>(c, seq, prefix_len, dst, (cudaStream_t)stream);
}

extern "C" int hx_kv_restore(hx_kv_cache* c, int seq, int prefix_len, const void* src,
                             size_t src_bytes, hx_stream_t stream)
{
    if (int rc = check_snapshot_args(c, seq, prefix_len, src, src_bytes)) return rc;
    if (prefix_len == 0) return HX_OK;
    return launch_copy<false>(c, seq, prefix_len, const_cast<void*>(src), (cudaStream_t)stream);
}
