// dist.cu — gather endpoints for multi-GPU decode (one process per GPU).
//
// Each rank allocates one device region: its gather buffer, then a 256-byte
// block of flag words, [0, world) = the epoch each rank last posted here.
// The region is exported with a CUDA IPC handle and mapped by every other
// rank, so the decode kernels of rank r store rows straight into rank q's
// buffer (decode_attention.cu: store_rows).  hx_dist_wait then runs one warp
// after them on the stream: it fences at system scope, posts this rank's
// epoch into every peer's flags[rank] with release stores, and polls the
// local flags with acquire loads until every peer's epoch has arrived, so
// rows a peer stored before its own post are visible here afterwards.
//
// The reference engine has no multi-GPU path (hxinfer-engine runs one
// device); this replaces the NCCL all-gather a sharded decode would issue
// after every layer.

#include <cuda_runtime.h>

#include <cstring>

#include "hx_common.cuh"

namespace hx {

constexpr size_t kFlagBytes = 256;

struct DistHandle {
    cudaIpcMemHandle_t mem;
    uint64_t bytes;
    int32_t rank, world;
};

static size_t round_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

__device__ __forceinline__ uint32_t ld_acquire_sys(const unsigned int* p)
{
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

struct PeerFlags {
    unsigned int* slot[kHxMaxRanks];  // peer r's flags[rank]; null for this rank
};

// One warp, launched as a programmatic dependent of the kernel before it on
// the stream: it becomes resident early, and griddepcontrol.wait returns once
// that kernel (and, through it, the decode kernels, whose last grid always
// waits for its predecessor) has completed with its stores performed.  Then
// lane r < world (r != rank) fences, posts `epoch` to peer r, and waits for
// flags[r] to reach `epoch` (mod 2^32 comparison), bounded by
// kWaitTimeoutNs of %globaltimer.
__global__ void dist_wait_kernel(const unsigned int* flags, PeerFlags peers, int world, int rank,
                                 uint32_t epoch, int* status)
{
    pdl_trigger();
    pdl_wait();
    const int r = threadIdx.x;
    bool ok = true;
    if (r < world && r != rank) {
        __threadfence_system();
        asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(peers.slot[r]), "r"(epoch)
                     : "memory");
        const uint64_t t0 = globaltimer_ns();
        while ((int32_t)(ld_acquire_sys(flags + r) - epoch) < 0) {
            if (globaltimer_ns() - t0 > kWaitTimeoutNs) {
                ok = false;
                break;
            }
        }
    }
    if (!ok) record_status(status, HX_ERR_TIMEOUT);
}

}  // namespace hx

using namespace hx;

extern "C" size_t hx_dist_handle_bytes(void) { return sizeof(DistHandle); }

extern "C" int hx_dist_create(int rank, int world, size_t buffer_bytes, hx_dist** out)
{
    if (!out) return fail(HX_ERR_INVALID, "null out");
    *out = nullptr;
    if (world < 1 || world > kHxMaxRanks || rank < 0 || rank >= world)
        return fail(HX_ERR_INVALID, "rank %d / world %d outside 1..%d ranks", rank, world,
                    kHxMaxRanks);
    if (buffer_bytes == 0) return fail(HX_ERR_INVALID, "empty gather buffer");
    auto* d = new (std::nothrow) hx_dist;
    if (!d) return fail(HX_ERR_OOM, "host allocation");
    d->rank = rank;
    d->world = world;
    d->bytes = buffer_bytes;
    cudaError_t e = cudaGetDevice(&d->device);
    const size_t total = round_up(buffer_bytes, kFlagBytes) + kFlagBytes;
    if (e == cudaSuccess) e = cudaMalloc(reinterpret_cast<void**>(&d->buf), total);
    if (e == cudaSuccess) e = cudaMemset(d->buf, 0, total);
    if (e != cudaSuccess) {
        if (d->buf) cudaFree(d->buf);
        delete d;
        return cuda_fail(e, "gather buffer allocation");
    }
    d->flags = reinterpret_cast<unsigned int*>(d->buf + round_up(buffer_bytes, kFlagBytes));
    d->peer_buf[rank] = d->buf;
    d->peer_flags[rank] = d->flags;
    d->connected = world == 1;
    *out = d;
    return HX_OK;
}

extern "C" int hx_dist_export(const hx_dist* d, void* handle)
{
    if (!d || !handle) return fail(HX_ERR_INVALID, "null endpoint or handle");
    DistHandle h{};
    HX_CUDA_TRY(cudaIpcGetMemHandle(&h.mem, d->buf));
    h.bytes = d->bytes;
    h.rank = d->rank;
    h.world = d->world;
    std::memcpy(handle, &h, sizeof h);
    return HX_OK;
}

extern "C" int hx_dist_connect(hx_dist* d, const void* handles)
{
    if (!d || !handles) return fail(HX_ERR_INVALID, "null endpoint or handles");
    if (d->connected) return d->world == 1 ? HX_OK : fail(HX_ERR_INVALID, "already connected");
    const auto* hs = static_cast<const DistHandle*>(handles);
    for (int r = 0; r < d->world; ++r) {
        DistHandle h;
        std::memcpy(&h, hs + r, sizeof h);
        if (h.rank != r || h.world != d->world || h.bytes != d->bytes)
            return fail(HX_ERR_INVALID, "handle %d is rank %d of %d with %llu bytes; expected rank "
                        "%d of %d with %zu", r, h.rank, h.world, (unsigned long long)h.bytes, r,
                        d->world, d->bytes);
    }
    for (int r = 0; r < d->world; ++r) {
        if (r == d->rank) continue;
        DistHandle h;
        std::memcpy(&h, hs + r, sizeof h);
        void* p = nullptr;
        cudaError_t e = cudaIpcOpenMemHandle(&p, h.mem, cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess) {
            for (int q = 0; q < r; ++q)
                if (q != d->rank && d->peer_buf[q]) {
                    cudaIpcCloseMemHandle(d->peer_buf[q]);
                    d->peer_buf[q] = nullptr;
                    d->peer_flags[q] = nullptr;
                }
            return cuda_fail(e, "cudaIpcOpenMemHandle of a peer's gather buffer");
        }
        d->peer_buf[r] = static_cast<char*>(p);
        d->peer_flags[r] =
            reinterpret_cast<unsigned int*>(d->peer_buf[r] + round_up(d->bytes, kFlagBytes));
    }
    d->connected = true;
    return HX_OK;
}

extern "C" int hx_dist_destroy(hx_dist* d)
{
    if (!d) return HX_OK;
    int rc = HX_OK;
    for (int r = 0; r < d->world; ++r) {
        if (r == d->rank || !d->peer_buf[r]) continue;
        cudaError_t e = cudaIpcCloseMemHandle(d->peer_buf[r]);
        if (e != cudaSuccess && rc == HX_OK) rc = cuda_fail(e, "cudaIpcCloseMemHandle");
    }
    if (d->buf) {
        cudaError_t e = cudaFree(d->buf);
        if (e != cudaSuccess && rc == HX_OK) rc = cuda_fail(e, "cudaFree of the gather buffer");
    }
    delete d;
    return rc;
}

extern "C" void* hx_dist_buffer(const hx_dist* d) { return d ? d->buf : nullptr; }

extern "C" int hx_dist_wait(hx_dist* d, uint32_t epoch, hx_stream_t stream)
{
    HX_NVTX_RANGE("hx_dist_wait");
    if (!d || !d->connected) return fail(HX_ERR_INVALID, "gather endpoint is not connected");
    if (d->world == 1) return HX_OK;
    if (int rc = check_device(d->device, "the gather endpoint")) return rc;
    PeerFlags peers{};
    for (int r = 0; r < d->world; ++r)
        if (r != d->rank) peers.slot[r] = d->peer_flags[r] + d->rank;
    cudaError_t e = launch_kernel(dist_wait_kernel, dim3(1), dim3(32), 0, (cudaStream_t)stream,
                                  true, (const unsigned int*)d->flags, peers, d->world, d->rank,
                                  epoch, status_word());
    if (e != cudaSuccess) return cuda_fail(e, "dist_wait_kernel launch");
    return check_launch("dist_wait_kernel");
}
