// hx_internal.h — host-side state shared by the translation units of libhxkv.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <nvtx3/nvToolsExt.h>
#include <string>
#include <vector>

#include "../../include/hx_kv.h"

namespace hx {

constexpr int kBlockTokens = 64;  // positions per cache block
constexpr int kMaxHeadDim = 256;

// What a kernel needs to address one layer of a cache (passed by value).
struct KVView {
    char* k;                 // K base of this layer
    char* v;                 // V base of this layer
    const int32_t* table;    // [max_seqs][mbps] physical block ids; nullptr = identity
    int32_t mbps;            // max blocks per sequence
    int32_t hkv;             // kv heads in this cache
    int32_t hd;              // head_dim
    int32_t capacity;        // positions per sequence
    int32_t max_seqs;
    int64_t block_stride;    // bytes between physical blocks
    int64_t head_stride;     // bytes between kv heads inside a block
    int64_t k_row0, v_row0;  // tensor-map row (unit: hd*2 bytes) of k / v
};

}  // namespace hx

struct hx_kv_cache {
    hx_kv_config cfg{};
    bool wrapped = false;
    int device = 0;
    int32_t mbps = 0;  // max blocks per sequence
    int64_t num_blocks = 0;
    char* pool = nullptr;
    size_t pool_bytes = 0;
    char* k0 = nullptr;  // layer-0 K base
    char* v0 = nullptr;  // layer-0 V base
    int64_t layer_stride = 0, kv_stride = 0, block_stride = 0, head_stride = 0;
    int32_t* d_table = nullptr;
    std::vector<int32_t> h_table;   // host mirror of the block table
    std::vector<int32_t> n_mapped;  // blocks mapped per sequence
    std::vector<int32_t> free_list;
    bool has_tmap = false;
    CUtensorMap tm_k{}, tm_v{};     // 2-D [rows][head_dim] fp16, box 64x64, 128B swizzle
    char* tm_k_base = nullptr;
    char* tm_v_base = nullptr;
    // Set up at creation on the cache's device (decode_prepare_device): the
    // device status word and the device address of the no-allocation decode
    // scratch, so hx_decode_attention_noalloc makes no set-up calls.
    int* status = nullptr;
    void* noalloc_scratch = nullptr;
};

// Peer-to-peer gather of decode outputs across the GPUs of one node: every
// rank owns a gather buffer and a flag word per rank, exported by CUDA IPC
// and mapped into every other rank.
constexpr int kHxMaxRanks = 8;

struct hx_dist {
    int rank = 0, world = 1, device = 0;
    size_t bytes = 0;
    char* buf = nullptr;                 // local gather buffer
    unsigned int* flags = nullptr;       // local [world] epochs posted by each rank
    char* peer_buf[kHxMaxRanks] = {};    // every rank's buffer (own at [rank])
    unsigned int* peer_flags[kHxMaxRanks] = {};
    bool connected = false;
};

struct hx_rope_table {
    hx_rope_config cfg{};
    float2* d_cos_sin = nullptr;  // [max_pos][head_dim/2] (cos, sin)
    int device = 0;
};

namespace hx {

// Records the message for hx_last_error() and returns `code`.
int fail(int code, const char* fmt, ...);
// Maps a CUDA error to HX_ERR_CUDA with its message (HX_OK if none).
int cuda_fail(cudaError_t e, const char* what);
// Checks the launch that was just issued.
int check_launch(const char* what);
// HX_ERR_INVALID unless `device` is the calling thread's current device.
// Every entry point that launches on a cache, table or endpoint calls it
// before any launch: a tensor map or block table of one GPU used from a
// kernel on another would read that GPU's memory as peer memory.
int check_device(int device, const char* what);
// Device status word of the current device (allocated on first use).
int* status_word();
int num_sms();
KVView make_view(const hx_kv_cache* c, int layer);
// Per-device set-up of the decode path for a new cache, on its device:
// kernel attributes and module loading, the device status word, and the
// no-allocation scratch address (stored in the cache).
int decode_prepare_device(hx_kv_cache* c);

}  // namespace hx

#define HX_CUDA_TRY(expr)                                            \
    do {                                                             \
        cudaError_t _e = (expr);                                     \
        if (_e != cudaSuccess) return hx::cuda_fail(_e, #expr);      \
    } while (0)

namespace hx {
// An NVTX range named after the C ABI call it covers: the call shows on a
// profiler's timeline and `ncu --nvtx --nvtx-include "<name>/"` selects its
// kernels.  Without a tool attached a push/pop is one pointer check.
struct NvtxRange {
    explicit NvtxRange(const char* name) { nvtxRangePushA(name); }
    ~NvtxRange() { nvtxRangePop(); }
    NvtxRange(const NvtxRange&) = delete;
    NvtxRange& operator=(const NvtxRange&) = delete;
};
}  // namespace hx
#define HX_NVTX_RANGE(name) ::hx::NvtxRange hx_nvtx_range_(name)
