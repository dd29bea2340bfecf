/*
 * hx_kv.h — C ABI of the B200 (sm_100a) KV-cache hot path for hxinfer.
 *
 * The library (hxinfer_b200/libhxkv.so) replaces, behind hxinfer's own operator
 * and layer interfaces, the reference engine's
 *   - KV append + decode attention  hxinfer-engine/src/op/cuda/attention_score_cuda.cu:7-214
 *                                   (declared hxinfer-engine/include/op/math_ops.h:67-73)
 *   - RoPE                          hxinfer-engine/src/op/cuda/rope_cuda.cu:46-152,
 *                                   hxinfer-engine/src/op/cpu/rope_cpu.cpp:5-39
 *                                   (declared math_ops.h:28-30)
 *   - QKV bias add                  hxinfer-engine/src/op/cuda/bias_add.cu:20-30
 *   - the per-layer K/V cache       hxinfer-engine/include/layer/attention.h:49-51,82-84
 *   - PrefixCacheManager copies     hxinfer-engine/include/cache/prefix_cache.h:58-151
 *
 * Conventions
 *   - Every entry point returns an int status (HX_OK = 0, else HX_ERR_*); the
 *     message of the last failure on the calling thread is in hx_last_error().
 *     Nothing is printed.
 *   - Every launch takes a CUDA stream and never synchronises it.  Kernel-side
 *     faults (an out-of-range position, a missing cache block, a bounded wait
 *     that ran out) are recorded in a per-device status word that
 *     hx_device_status() reads back.
 *   - Pointers marked "device" are CUDA device pointers; sizes are in elements
 *     unless the name ends in _bytes.  No torch or C++ types cross this ABI.
 *   - A cache handle is thread-compatible: one host thread at a time per
 *     handle; concurrency comes from streams.
 *
 * KV layout in HBM (head-major, 128-byte aligned blocks)
 *   One pool per cache: [layer][K|V][block][kv_head][64 tokens][head_dim] fp16.
 *   A block holds 64 consecutive positions of one sequence; a per-sequence
 *   block table maps logical block -> physical block.  Each (block, kv_head)
 *   tile is a contiguous 64*head_dim*2-byte run (16 KiB at head_dim 128),
 *   which is one TMA tile of the decode kernel.
 */
#ifndef HX_KV_H
#define HX_KV_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

struct CUstream_st;
typedef struct CUstream_st* hx_stream_t; /* same type as cudaStream_t */

enum hx_status {
    HX_OK = 0,
    HX_ERR_INVALID = 1,     /* bad argument, shape or dtype */
    HX_ERR_CAPACITY = 2,    /* position / length / pool capacity exceeded */
    HX_ERR_OOM = 3,         /* device or host allocation failed */
    HX_ERR_CUDA = 4,        /* a CUDA runtime call failed */
    HX_ERR_NCCL = 5,        /* a collective failed */
    HX_ERR_TIMEOUT = 6,     /* a bounded device-side wait ran out */
    HX_ERR_NOT_FOUND = 7,   /* unknown sequence or snapshot */
    HX_ERR_UNSUPPORTED = 8  /* valid request this build does not implement */
};

/* Element types; FP32 and FP16 are the reference's DataType codes
 * (hxinfer-engine/include/base/config.h:5-10).  BF16 is a checkpoint source
 * format only (safetensors "BF16"), accepted by hx_convert alone. */
enum hx_dtype { HX_FP32 = 1, HX_FP16 = 3, HX_BF16 = 16 };

const char* hx_status_string(int status);
/* Message of the last failed call on this thread ("" if none). */
const char* hx_last_error(void);
/* Reads (and, if clear != 0, resets) the device-side status word of the
 * current device.  Synchronises the device.  Returns HX_OK or the first
 * HX_ERR_* a kernel recorded since the last reset. */
int hx_device_status(int clear);

/* ------------------------------------------------------------ KV cache */

typedef struct hx_kv_cache hx_kv_cache;

typedef struct {
    int32_t num_layers;
    int32_t num_kv_heads;        /* heads held by this cache (a shard may hold a subset) */
    int32_t head_dim;            /* even, <= 256; 128 takes the TMA decode path */
    int32_t max_seqs;
    int32_t max_tokens_per_seq;  /* per-sequence capacity in positions */
    int64_t num_blocks;          /* physical 64-token blocks; 0 = max_seqs * ceil(max_tokens/64) */
    int32_t flags;               /* HX_KV_* bits below; 0 = none */
} hx_kv_config;

/* hx_kv_config.flags
 *
 * HX_KV_OVERLAP_LAUNCH: hx_rope_append and hx_decode_attention on this cache
 * are launched as programmatic dependents, so a launch can begin while the
 * kernel before it on the stream is still finishing.  hx_rope_append reads
 * nothing before that kernel has finished.  hx_decode_attention reads
 * `lengths`, `seq_ids`, the block table and cache positions below each
 * sequence's newest position (lengths[i] - 1) early; the kernel launched just
 * before it on the stream must therefore write none of those -- it may write
 * q and each sequence's newest position, which is exactly what the decode
 * step hx_rope_append -> hx_decode_attention does.  Without the flag every
 * launch waits for the previous kernel to finish. */
enum { HX_KV_OVERLAP_LAUNCH = 1 };

typedef struct {
    int32_t num_layers, num_kv_heads, head_dim, max_seqs, max_blocks_per_seq;
    int64_t num_blocks, free_blocks;
    void* pool;                  /* device; NULL for a wrapped cache */
    size_t pool_bytes;
    int64_t layer_stride_bytes, kv_stride_bytes, block_stride_bytes, head_stride_bytes;
    int32_t* block_table;        /* device [max_seqs][max_blocks_per_seq], -1 = unmapped */
} hx_kv_info;

/* Allocates the pool and block table (replaces the per-layer cache tensors of
 * AttentionLayer, attention.h:49-51). */
int hx_kv_create(const hx_kv_config* cfg, hx_kv_cache** out);

/* Wraps caller memory as a one-layer, one-sequence cache with the contiguous
 * head-major layout [num_kv_heads][capacity][head_dim] fp16 for K and V.
 * This is how the kept operator attention_score_cuda(q, k, v, k_cache,
 * v_cache, out, config, pos) (math_ops.h:67-73) uses the caller's k_cache /
 * v_cache tensors: storage stays opaque to the caller. */
int hx_kv_wrap(void* k_base, void* v_base, int num_kv_heads, int head_dim, int capacity,
               hx_kv_cache** out);

int hx_kv_destroy(hx_kv_cache* cache);
int hx_kv_get_info(const hx_kv_cache* cache, hx_kv_info* out);

/* Makes sequence `seq` able to hold n_tokens positions, mapping blocks from
 * the pool's free list; the block-table row is updated on `stream`. */
int hx_kv_reserve(hx_kv_cache* cache, int seq, int n_tokens, hx_stream_t stream);
/* Returns every block of `seq` to the free list. */
int hx_kv_release(hx_kv_cache* cache, int seq, hx_stream_t stream);

/* Copies n token rows (token-major [n][num_kv_heads*head_dim], dtype
 * HX_FP16 or HX_FP32, device) into positions [start, start+n) of (layer, seq)
 * without rotation; fp32 input is rounded to fp16 (RNE). */
int hx_kv_write(hx_kv_cache* cache, int layer, int seq, int start, int n, const void* k,
                const void* v, int dtype, hx_stream_t stream);
/* Gathers positions [start, start+n) of (layer, seq) into token-major fp16
 * rows [n][num_kv_heads*head_dim] (device); k or v may be NULL. */
int hx_kv_read(const hx_kv_cache* cache, int layer, int seq, int start, int n, void* k, void* v,
               hx_stream_t stream);
/* Fills every block of the pool with N(0,1) values rounded to fp16, from a
 * counter-based generator keyed by `seed` (synthetic benchmark caches). */
int hx_kv_fill_normal(hx_kv_cache* cache, uint64_t seed, hx_stream_t stream);

/* ------------------------------------------------------------ RoPE */

typedef struct hx_rope_table hx_rope_table;

typedef struct {
    int32_t head_dim;
    int32_t max_pos;            /* positions [0, max_pos) */
    float theta;                /* base; ModelConfig::rope_theta (config.h:41) */
    int32_t use_yarn;           /* ModelConfig::rope_use_yarn (config.h:43) */
    float yarn_factor, yarn_beta_fast, yarn_beta_slow;
    int32_t yarn_orig_max_pos;
} hx_rope_config;

/* Builds the device cos/sin table [max_pos][head_dim/2] holding exactly the
 * cos/sin values rope_cpu computes (rope_cpu.cpp:22-25), or with use_yarn the
 * YaRN-scaled values of rope_cuda (rope_cuda.cu:56-61, 112-121). */
int hx_rope_table_create(const hx_rope_config* cfg, hx_rope_table** out);
int hx_rope_table_destroy(hx_rope_table* table);

/* In-place NeoX RoPE of q [rows][num_q_heads*head_dim] and k
 * [rows][num_kv_heads*head_dim] (device, HX_FP16 or HX_FP32) at one position
 * `step`.  Replaces rope_cuda (rope_cuda.cu:98-152); the result equals
 * rope_cpu (rope_cpu.cpp:5-39) bit for bit. */
int hx_rope_qk(void* q, void* k, int dtype, int rows, int num_q_heads, int num_kv_heads,
               int head_dim, int step, const hx_rope_table* table, hx_stream_t stream);

/* K1: fused QKV bias + RoPE + K/V append.  For each token i:
 *   q' = rope(q[i] + bq), k' = rope(k[i] + bk), v' = v[i] + bv,
 *   cache(layer, seq_ids[i], positions[i]) <- (k', v') in fp16,
 *   q_out[i] <- q' in q_out_dtype.
 * q/k/v rows as in the reference ([n][Hq*hd], [n][Hkv*hd]) in `dtype`;
 * biases (same dtype) may be NULL; table may be NULL (no rotation: a plain
 * append, as attention_score_cuda.cu:7-15 does); q/q_out may be NULL.
 * The fp16 bias add rounds like bias_add.cu:6-11 (__hadd).
 * seq_ids/positions: device int32 [n_tokens]. */
int hx_rope_append(hx_kv_cache* cache, int layer, const void* q, const void* k, const void* v,
                   int dtype, const void* bq, const void* bk, const void* bv,
                   const int32_t* seq_ids, const int32_t* positions, int n_tokens,
                   int num_q_heads, const hx_rope_table* table, void* q_out, int q_out_dtype,
                   hx_stream_t stream);

/* ------------------------------------------------------------ attention */

/* The QKV projection fused with K1 (a step beyond the reference's K1
 * boundary: replaces matmul_qkv_cuda's three cublasGemmEx GEMVs,
 * matmul_cuda.cu:106-189, and the bias adds in front of hx_rope_append).
 * For each token i: q = Wq x[i], k = Wk x[i], v = Wv x[i] (fp32 accumulate,
 * rounded to proj_dtype, the dtype the reference's q/k/v tensors have), then
 * exactly hx_rope_append's bias + RoPE + append on those values.
 * x: device [n_tokens][hidden] fp16 or fp32 (fp32 is rounded to fp16 first,
 * as the reference does); wq/wk/wv: device fp16 [Hq*128][hidden],
 * [Hkv*128][hidden] row-major (the reference's weight tensors); biases in
 * proj_dtype, may be NULL.  x and the weights 16-byte aligned; hidden a
 * multiple of 8, at most 8192; head_dim 128.  Reads each weight row once per
 * group of 8 tokens: meant for decode batches. */
int hx_qkv_rope_append(hx_kv_cache* cache, int layer, const void* x, int x_dtype, int hidden,
                       const void* wq, const void* wk, const void* wv, int proj_dtype,
                       const void* bq, const void* bk, const void* bv, const int32_t* seq_ids,
                       const int32_t* positions, int n_tokens, int num_q_heads,
                       const hx_rope_table* table, void* q_out, int q_out_dtype,
                       hx_stream_t stream);

/* Workspace bytes hx_decode_attention needs for n_seqs sequences: a fixed
 * 64 KiB block of per-segment arrival counters followed by the split-K
 * partial results.  Device memory owned by the caller.  Zero-fill it once
 * before its first use (e.g. cudaMemsetAsync); every call leaves the counters
 * zero again, so later calls, on any cache and any n_seqs up to the size the
 * buffer was made for, need no clearing.  Calls that share one workspace must
 * not overlap on the GPU. */
size_t hx_decode_workspace_bytes(const hx_kv_cache* cache, int n_seqs, int num_q_heads);

/* K2: split-K GQA decode attention over the cache (replaces
 * attention_score_kernel, attention_score_cuda.cu:17-83,95-161).
 * q: device [n_seqs][num_q_heads*head_dim] (rotated) in q_dtype;
 * seq_ids, lengths: device int32 [n_seqs] (lengths = positions attended, >= 1);
 * out: device [n_seqs][num_q_heads*head_dim] in out_dtype.
 * q head h reads kv head h / (num_q_heads / num_kv_heads).
 * One launch when the call has at least 64 (sequence, kv head) pairs and at
 * most 8 q heads per kv head (the decode kernel merges its own split-K
 * pieces); otherwise the split-K kernel and its combine kernel. */
int hx_decode_attention(const hx_kv_cache* cache, int layer, const void* q, int q_dtype,
                        const int32_t* seq_ids, const int32_t* lengths, int n_seqs,
                        int num_q_heads, float scale, void* out, int out_dtype, void* workspace,
                        size_t workspace_bytes, hx_stream_t stream);

/* The new token of every sequence of an append-and-decode call (one token
 * per sequence, at position lengths[s] - 1): its raw K and V rows and the
 * optional biases, all in `dtype` (HX_FP16 or HX_FP32, also the dtype of q),
 * and the optional RoPE table (NULL: no rotation). */
typedef struct {
    const void* k;                 /* device [n_seqs][num_kv_heads*head_dim] */
    const void* v;                 /* device [n_seqs][num_kv_heads*head_dim] */
    const void* bq;                /* [num_q_heads*head_dim] or NULL */
    const void* bk;                /* [num_kv_heads*head_dim] or NULL */
    const void* bv;                /* [num_kv_heads*head_dim] or NULL */
    int32_t dtype;
    const hx_rope_table* table;
} hx_append_spec;

/* K1 + K2 in one launch: for every sequence, the bias and RoPE of q and k,
 * the append of the token's K/V row at position lengths[s] - 1, then decode
 * attention over lengths[s] positions.  Replaces the reference's
 * attention_score_cuda (attention_score_cuda.cu:163-214), which appends
 * curr_k / curr_v and attends in one host call, together with the bias adds
 * and rope_cuda in front of it (attention.cpp:21-35).  q: the raw q rows
 * [n_seqs][num_q_heads*head_dim] in append->dtype.  Equal bit for bit, in
 * the cache and in out, to hx_rope_append (positions lengths - 1, q_out
 * fp16) followed by hx_decode_attention; the cache must be as hx_decode_
 * attention needs it (head_dim 128, at most 16 q heads per kv head; else
 * HX_ERR_UNSUPPORTED).  The workspace is hx_decode_workspace_bytes, with its
 * rules. */
int hx_append_decode_attention(hx_kv_cache* cache, int layer, const void* q,
                               const hx_append_spec* append, const int32_t* seq_ids,
                               const int32_t* lengths, int n_seqs, int num_q_heads, float scale,
                               void* out, int out_dtype, void* workspace, size_t workspace_bytes,
                               hx_stream_t stream);

/* K3: causal prefill attention on the tcgen05 tensor cores.  Query rows
 * i in [0, n) sit at positions start + i of sequence `seq` and attend to
 * positions [0, start + i] of the cache (their own K/V must already be
 * appended, e.g. by hx_rope_append).  q: device fp16 [n][num_q_heads*128]
 * (rotated), 16-byte aligned; out: [n][num_q_heads*128] in out_dtype.
 * head_dim must be 128.  The reference prefills one token per forward call
 * (hxinfer demos/bench_1024.cpp:62-70), i.e. attention_score_cuda.cu:17-83 once
 * per position; this is the same function of the inputs in one launch. */
int hx_prefill_attention(const hx_kv_cache* cache, int layer, const void* q, int seq, int start,
                         int n, int num_q_heads, float scale, void* out, int out_dtype,
                         hx_stream_t stream);

/* The same decode attention as hx_decode_attention, for callers that cannot
 * allocate device memory (code inside an allocator or an out-of-memory
 * handler, hosts that reserve all device memory up front, plug-in hosts that
 * forbid cudaMalloc): no workspace argument, and no cudaMalloc, cudaFree or
 * other allocating call.  No counterpart exists in the reference engine.
 * Its split-K scratch is a fixed 4 MiB array inside the library, which every
 * GPU that loads the library keeps until exit; calls needing more
 * (hx_decode_workspace_bytes > 4 MiB) fail with HX_ERR_CAPACITY.  The array's
 * device address, the kernels' attributes and the device status word are
 * set up once per device by hx_kv_create / hx_kv_wrap, on the cache's device,
 * where allocating is allowed; this entry point itself makes no set-up call.
 * All calls share the array and it keeps the last call's contents (its
 * counters are back at zero after every call): calls that overlap on the GPU
 * race.  Kernel-side faults are recorded in the device status word as for
 * hx_decode_attention. */
int hx_decode_attention_noalloc(const hx_kv_cache* cache, int layer, const void* q, int q_dtype,
                                const int32_t* seq_ids, const int32_t* lengths, int n_seqs,
                                int num_q_heads, float scale, void* out, int out_dtype,
                                hx_stream_t stream);

/* ------------------------------------------------------------ multi-GPU gather
 *
 * K5: decode attention sharded over the GPUs of one node (one process per
 * GPU), with the all-gather of the per-rank outputs fused into the decode
 * kernels.  Each rank owns a gather buffer; the decode and combine kernels
 * store every output row of this rank into every rank's buffer over NVLink
 * peer memory (16-byte stores, no bulk copy).  hx_dist_wait then posts this
 * rank's epoch into a flag word on every other rank and holds the stream
 * until every other rank's epoch has arrived.  The
 * reference engine is single-GPU; this replaces an NCCL all-gather issued
 * after each decode call.
 *
 * Set-up, on every rank (with the current device set to the rank's GPU):
 *   hx_dist_create -> hx_dist_export -> exchange the handles (any host-side
 *   all-gather, e.g. torch.distributed over a store) -> hx_dist_connect.
 * All ranks must run on GPUs of one node that can access each other's memory
 * (cudaDeviceCanAccessPeer), in different processes. */
typedef struct hx_dist hx_dist;

/* Bytes of the IPC handle blob hx_dist_export writes. */
size_t hx_dist_handle_bytes(void);
/* Allocates this rank's gather buffer (buffer_bytes, zeroed) and flag words on
 * the current device.  1 <= world <= 8, 0 <= rank < world. */
int hx_dist_create(int rank, int world, size_t buffer_bytes, hx_dist** out);
/* Writes this rank's IPC handles (hx_dist_handle_bytes bytes) to `handle`. */
int hx_dist_export(const hx_dist* dist, void* handle);
/* Maps every other rank's buffer and flags.  handles: world blobs of
 * hx_dist_handle_bytes each, in rank order (this rank's own is ignored). */
int hx_dist_connect(hx_dist* dist, const void* handles);
/* Unmaps the peers and frees this rank's buffer.  Every rank must have
 * finished its last gathering call (e.g. a host barrier after a device
 * synchronise) before any rank destroys its endpoint. */
int hx_dist_destroy(hx_dist* dist);
/* Device address of this rank's gather buffer. */
void* hx_dist_buffer(const hx_dist* dist);

/* hx_decode_attention for this rank's shard, with the outputs written into
 * every rank's gather buffer.  The output is a matrix starting at byte
 * out_offset (a multiple of 16) of each buffer, [rows][out_row_heads*128] in
 * out_dtype: q head qh of local sequence s goes to row out_rows[s] (device
 * int32 [n_seqs]), column block out_head0 + qh.  The ranks' (row, column)
 * blocks must not overlap.  n_seqs may be 0 (nothing is written).
 *
 * The call does not wait for the other ranks: follow it by hx_dist_wait
 * before reading the buffer.  A region of the buffer may be written again
 * once every rank has consumed it; with two regions used alternately that
 * holds when each rank consumes a region before its next gathering call. */
int hx_decode_attention_gather(const hx_kv_cache* cache, int layer, const void* q, int q_dtype,
                               const int32_t* seq_ids, const int32_t* lengths, int n_seqs,
                               int num_q_heads, float scale, hx_dist* dist, size_t out_offset,
                               const int32_t* out_rows, int out_row_heads, int out_head0,
                               int out_dtype, void* workspace, size_t workspace_bytes,
                               hx_stream_t stream);
/* hx_append_decode_attention with the outputs placed as
 * hx_decode_attention_gather places them. */
int hx_append_decode_attention_gather(hx_kv_cache* cache, int layer, const void* q,
                                      const hx_append_spec* append, const int32_t* seq_ids,
                                      const int32_t* lengths, int n_seqs, int num_q_heads,
                                      float scale, hx_dist* dist, size_t out_offset,
                                      const int32_t* out_rows, int out_row_heads, int out_head0,
                                      int out_dtype, void* workspace, size_t workspace_bytes,
                                      hx_stream_t stream);
/* Exchanges `epoch` with every other rank: once everything launched before
 * it on `stream` has completed, posts `epoch` to every other rank and holds
 * the stream until every other rank has posted it here (one warp; rows a
 * rank stored before its post are then visible).  Every rank calls it with
 * the same epoch, greater (mod 2^32) than its previous one, after the same
 * gathering calls.  The wait is bounded (4 s); when it runs out the kernel
 * records HX_ERR_TIMEOUT in the device status word and returns, so the host
 * finds the failure through hx_device_status. */
int hx_dist_wait(hx_dist* dist, uint32_t epoch, hx_stream_t stream);

/* ------------------------------------------------------------ prefix snapshots */

/* Bytes of a snapshot of the first prefix_len positions of one sequence:
 * layers * 2 * num_kv_heads * prefix_len * head_dim * 2. */
size_t hx_snapshot_bytes(const hx_kv_cache* cache, int prefix_len);

/* K4: copies positions [0, prefix_len) of every layer's K and V of `seq` into
 * dst (device, layout [layer][K|V][kv_head][prefix_len][head_dim] fp16).
 * dst (and src of hx_kv_restore) must be device, managed or mapped pinned
 * memory; pageable host memory is refused with HX_ERR_INVALID.
 * Replaces the host memcpy of PrefixCacheManager::store (prefix_cache.h:78-89). */
int hx_kv_snapshot(const hx_kv_cache* cache, int seq, int prefix_len, void* dst,
                   size_t dst_bytes, hx_stream_t stream);
/* Copies a snapshot back into positions [0, prefix_len) of `seq` (which must
 * be reserved for prefix_len positions); later positions are untouched.
 * Replaces PrefixCacheManager::restore's memcpy (prefix_cache.h:135-147). */
int hx_kv_restore(hx_kv_cache* cache, int seq, int prefix_len, const void* src,
                  size_t src_bytes, hx_stream_t stream);

/* hx_kv_snapshot over the layers of a model whose layers each hold their own
 * cache (AttentionLayer keeps one [seq_len, kv_dim] K and V tensor per layer,
 * attention.h:49-51, each wrapped by hx_kv_wrap): ONE launch copies
 * positions [0, prefix_len) of every cache in caches[0 .. n_caches), into dst
 * laid out [cache][K|V][kv_head][prefix_len][head_dim] fp16 -- the bytes of
 * n_caches consecutive hx_kv_snapshot calls.  Every cache must come from
 * hx_kv_wrap with the shape of caches[0], on the current device; at most 64
 * caches per call.  Replaces the per-layer memcpy loop of
 * PrefixCacheManager::store (prefix_cache.h:78-89). */
int hx_kv_snapshot_layers(const hx_kv_cache* const* caches, int n_caches, int prefix_len,
                          void* dst, size_t dst_bytes, hx_stream_t stream);
/* The inverse copy, one launch (PrefixCacheManager::restore,
 * prefix_cache.h:135-147); positions >= prefix_len are untouched. */
int hx_kv_restore_layers(hx_kv_cache* const* caches, int n_caches, int prefix_len,
                         const void* src, size_t src_bytes, hx_stream_t stream);

/* ------------------------------------------------------------ weight loading */

/* Converts n elements of src (device memory, src_dtype) into dst (device
 * memory, dst_dtype) on `stream`: BF16->FP16, BF16->FP32, FP32->FP16,
 * FP16->FP32, or a copy when the dtypes are equal.  Narrowing to FP16 rounds
 * to nearest even, overflowing to infinity, as __float2half does in the
 * reference's CPU loops; widening is exact.  dst may equal src when both
 * element sizes are equal (BF16->FP16 in place); otherwise the two ranges
 * must not overlap.  n = 0 is a no-op.
 * Replaces the CPU conversion loops of SafetensorsReader::get_tensor_gpu
 * (model_loaders/src/safetensors_loader.cpp:12-27, 124-197). */
int hx_convert(void* dst, int dst_dtype, const void* src, int src_dtype, size_t n,
               hx_stream_t stream);

/* FNV-1a 64 of the token ids (PrefixCacheManager::compute_hash,
 * prefix_cache.h:42-49); host function. */
uint64_t hx_prefix_hash(const int32_t* tokens, size_t n);

#ifdef __cplusplus
}
#endif
#endif /* HX_KV_H */
