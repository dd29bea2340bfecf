// decode_attention.cu — K2: split-K (flash-decoding) GQA/MHA decode attention
// over the paged head-major KV cache, and its combine kernel.
//
// Replaces attention_score_kernel(_fp16) (hxinfer-engine/src/op/cuda/
// attention_score_cuda.cu:17-83, 95-161): there one CTA per q head walks all
// positions with scores staged in shared memory (so it cannot run past ~12k
// positions) and re-reads K/V once per q head.  Here:
//
//  * Work is the flat list of 64-position tiles over all (sequence, kv head)
//    segments; CTA c of C takes tiles [c*T/C, (c+1)*T/C), so every CTA
//    streams the same number of bytes whatever the lengths.  C is one CTA
//    per SM (6-stage ring) or, for calls with many segments, two CTAs per SM
//    (3-stage rings) so that one CTA's tail overlaps the other's streaming.
//  * Warp 4 (producer) streams each tile's K and V (2 x 16 KiB) with TMA
//    (cp.async.bulk.tensor, 64x64 boxes, 128-byte swizzle, L2 evict-first)
//    into the mbarrier ring; no multicast.
//  * Warps 0-3 (consumers) each own 16 positions of every tile.  The MMAs
//    (mma.sync m16n8k16, fp16 in, fp32 accumulate) run transposed: the
//    warp's positions are the M side and the GQA group's q rows the N side
//    (8 rows per n-tile), so each K/V tile is read from HBM once per group
//    and a group of up to 8 rows needs no padding: S^T = K Q^T, then
//    O^T += V^T P^T with P^T moved into operand layout by movmatrix.  The
//    softmax is online (running max and sum per row, warp-shuffle reductions
//    over the lanes that share a row).
//  * At the end of each piece (the part of a segment inside one CTA) the four
//    warps merge in the shared memory of the stage they just consumed.  A
//    piece that is a whole segment writes the normalised output; otherwise
//    it writes (O, m, l) to a workspace slot, and the pieces are merged by
//    log-sum-exp: in wide calls (few pieces per segment) by the CTA whose
//    arrival completes the segment, counted in a per-segment counter; in
//    narrow calls (batch 1: dozens of pieces per segment) by
//    decode_combine_kernel, one CTA per segment and q row, launched as a
//    programmatic dependent.
//
// Workspace: a fixed 64 KiB block of per-segment counters (zero between
// calls), then the slots: slot (seq*hkv + kv_head) holds the piece that
// starts at a segment's first tile; slot (n_segments + c) holds CTA c's first
// piece when that piece starts inside a segment, so slots = n_segments + C.
// Every slot a merge reads is written earlier in the same call.
#include <cfloat>
#include <mutex>

#include "hx_common.cuh"

namespace hx {

// Two launch shapes of the same kernel:
//  * narrow: one CTA per SM with a 6-stage ring;
//  * wide: two CTAs per SM, each with a 3-stage ring (the same bytes in
//    flight per SM), so one CTA's end-of-range merge, its exit and the next
//    CTA's start overlap the other CTA's streaming.  It needs the 8-row GQA
//    tile (the 16-row one has too many registers for two CTAs) and pays off
//    when every CTA has many tiles; with few segments (batch-1 long context)
//    its shorter ring loses, so calls with fewer than kWideMinSegments
//    (sequence, kv head) segments use the narrow shape.
constexpr int kWideMinSegments = 64;
constexpr int kDecConsumerWarps = 4;
constexpr int kDecThreads = (kDecConsumerWarps + 1) * 32;
constexpr int kHalfTileBytes = 64 * 64 * 2;       // one 64x64 fp16 TMA box
constexpr int kTileBytes = 2 * kHalfTileBytes;     // 64 positions x 128 dims
constexpr uint32_t kStageTxBytes = 2 * kTileBytes; // K + V
constexpr int kMaxPieces = 300;  // bound on split-K pieces per segment (needs C + 2 <= it)

struct DecodeParams {
    KVView view;
    const void* q;             // [n_seqs][hq*128], fp16 or fp32
    const int32_t* seq_ids;
    const int32_t* lengths;
    int n_seqs, hq, group, q_f32;
    float scale_log2;          // softmax scale * log2(e)
    void* out;                 // first destination (== outs[0])
    // Output placement: q head qh of sequence s goes to row out_rows[s]
    // (s when out_rows is null), column block out_head0 + qh, of a matrix
    // [rows][out_hq * head_dim] in every destination outs[0..n_outs).  A plain
    // call has one destination, out_hq == hq and out_head0 == 0; a gathering
    // call also writes each other rank's buffer.
    void* outs[kHxMaxRanks];
    int n_outs;
    const int32_t* out_rows;
    int out_hq, out_head0;
    int out_row_limit;         // rows the destinations hold; a row beyond is skipped and recorded
    int out_vec;               // every destination is 16-byte aligned: rows go out as 16-byte stores
    int out_f32;
    float* ws_o;               // [slots][group][128]
    float2* ws_ml;             // [slots][group] (m, l)
    int* status;
    // Folded combine (wide calls): one arrival counter per segment.  The CTA
    // that completes a segment's last piece merges its pieces itself and
    // returns the counter to zero; null = the separate combine kernel merges.
    unsigned int* fold_cnt;
    // Append-and-decode (k_new != null): every sequence s brings one new
    // token, at position lengths[s] - 1.  q is then its raw q rows (bias and
    // RoPE still to apply) and k_new / v_new its raw K / V rows
    // [n_seqs][hkv * 128], in q's dtype like the optional biases.  The CTA
    // whose range holds a segment's newest tile writes the token's K and V
    // row into the cache before loading that tile; every CTA applies the bias
    // and the rotation to its q rows as it loads them.  The arithmetic is K1's,
    // so cache and output equal hx_rope_append followed by
    // hx_decode_attention bit for bit.
    const void* k_new;
    const void* v_new;
    const void* bq;
    const void* bk;
    const void* bv;
    const float2* rope;        // [rope_max_pos][64] (cos, sin), or null: no rotation
    int rope_max_pos;
};

constexpr int kMinTilesPerCta = 2;  // small problems use fewer CTAs, hence fewer pieces

// The CTA's slice of the flat tile list, computed once by the producer warp.
struct Sched {
    int s, h, j, tiles, len, seq;  // cursor at the first tile
    int count;                     // tiles in this CTA's range
    int g_first;                   // global index of the first tile
    int total;                     // tiles over all segments
    int n_eff;                     // CTAs that received work
    int odd_lengths;               // some length is < 1 or above the capacity
};

template <int ROWS, int STAGES>
struct DecodeSmem {
    // [stage][K|V]: two 64x64 boxes each.  At the end of a piece the stage
    // just consumed also holds the warps' O partials (merge_o), before it is
    // released to the producer.
    uint8_t stage[STAGES][2][kTileBytes];
    float merge_m[kDecConsumerWarps][ROWS];
    float merge_l[kDecConsumerWarps][ROWS];
    uint64_t full[STAGES];
    uint64_t empty[STAGES];
    Sched sched;
    int fold_ca;               // folded combine: first CTA of the segment to merge, or -1
    int fold_np;               // and its number of pieces
    int cstart[kMaxPieces];    // first global tile of CTA c, c in [0, n_eff]
};

__device__ __forceinline__ int tiles_of(int len) { return (len + kBlockTokens - 1) / kBlockTokens; }

__device__ __forceinline__ int clamp_len(int len, int cap) { return len < 0 ? 0 : (len > cap ? cap : len); }

// Position of the CTA's tile range within the segment list.
struct Cursor {
    int s, h, j, tiles, len, seq;
};

__device__ __forceinline__ void cursor_load(Cursor& c, const DecodeParams& p, int s)
{
    c.s = s;
    c.len = s < p.n_seqs ? clamp_len(p.lengths[s], p.view.capacity) : 0;
    c.tiles = tiles_of(c.len);
    c.seq = s < p.n_seqs ? p.seq_ids[s] : 0;
}

__device__ __forceinline__ void cursor_next(Cursor& c, const DecodeParams& p)
{
    if (++c.j < c.tiles) return;
    c.j = 0;
    if (++c.h < p.view.hkv) return;
    c.h = 0;
    int s = c.s + 1;
    cursor_load(c, p, s);
    // skip empty sequences (length 0 has no tiles)
    while (c.tiles == 0 && s < p.n_seqs) cursor_load(c, p, ++s);
}

// Producer-warp planning, all lanes: total tiles T, the number of CTAs that
// get work (n_eff = min(grid, ceil(T / kMinTilesPerCta))), every CTA's first
// tile (cstart, so later piece arithmetic is a shared-memory lookup), and
// this CTA's starting cursor.
template <typename Smem>
__device__ void plan_cta(const DecodeParams& p, int cta, int grid, Smem& sm)
{
    const int lane = threadIdx.x & 31;
    const int hkv = p.view.hkv;
    long long total = 0;
    bool odd = false;
    // The first kPlanRounds x 32 sequences' lengths and ids are loaded
    // together and kept, so a call of up to 128 sequences plans with one
    // round of global loads.
    constexpr int kPlanRounds = 4;
    int len_r[kPlanRounds], sid_r[kPlanRounds];
#pragma unroll
    for (int r = 0; r < kPlanRounds; ++r) {
        const int s = 32 * r + lane;
        len_r[r] = s < p.n_seqs ? p.lengths[s] : 1;
        sid_r[r] = s < p.n_seqs ? p.seq_ids[s] : 0;
    }
    // the kept value of round base / 32, else a load (calls of more than 128 sequences)
    auto kept = [&](const int (&arr)[kPlanRounds], int base, const int* src, int dflt) {
        int v = dflt;
#pragma unroll
        for (int r = 0; r < kPlanRounds; ++r)
            if (base == 32 * r) v = arr[r];
        if (base >= 32 * kPlanRounds) v = base + lane < p.n_seqs ? src[base + lane] : dflt;
        return v;
    };
    for (int base = 0; base < p.n_seqs; base += 32) {
        const int s = base + lane;
        const int len = kept(len_r, base, p.lengths, 1);
        odd |= len < 1 || len > p.view.capacity;
        int t = tiles_of(clamp_len(len, p.view.capacity)) * (s < p.n_seqs);
#pragma unroll
        for (int o = 16; o; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
        total += t;
    }
    odd = __any_sync(0xffffffffu, odd);
    total *= hkv;
    if (total >= (1ll << 31) / kMaxPieces) {
        // the int tile arithmetic below would overflow: refuse the work
        if (lane == 0) record_status(p.status, HX_ERR_CAPACITY);
        total = 0;
    }
    const int T = (int)total;
    const int want = (T + kMinTilesPerCta - 1) / kMinTilesPerCta;
    const int n_eff = max(1, min(grid, want));
    // T < 2^31 / kMaxPieces, so T * c fits in 32 bits
    for (int c = lane; c <= n_eff; c += 32) sm.cstart[c] = (int)((unsigned)T * (unsigned)c / (unsigned)n_eff);
    __syncwarp();
    Sched sc{};
    sc.total = T;
    sc.n_eff = n_eff;
    sc.odd_lengths = odd;
    sc.s = p.n_seqs;
    if (cta < n_eff) {
        sc.g_first = sm.cstart[cta];
        sc.count = sm.cstart[cta + 1] - sc.g_first;
    }
    if (sc.count > 0) {
        const int g0 = sc.g_first;
        int run = 0;  // tiles before the current chunk
        for (int base = 0; base < p.n_seqs; base += 32) {
            const int s = base + lane;
            const int len = s < p.n_seqs ? clamp_len(kept(len_r, base, p.lengths, 1), p.view.capacity) : 0;
            const int sid = kept(sid_r, base, p.seq_ids, 0);
            const int t = tiles_of(len) * hkv;
            int incl = t;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int y = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o) incl += y;
            }
            const unsigned hit = __ballot_sync(0xffffffffu, run + incl > g0);
            if (hit) {
                const int src = __ffs(hit) - 1;
                const int before = run + __shfl_sync(0xffffffffu, incl - t, src);
                const int off = g0 - before;
                sc.s = base + src;
                sc.len = __shfl_sync(0xffffffffu, len, src);
                sc.tiles = tiles_of(sc.len);
                sc.seq = __shfl_sync(0xffffffffu, sid, src);
                sc.h = off / sc.tiles;
                sc.j = off % sc.tiles;
                break;
            }
            run += __shfl_sync(0xffffffffu, incl, 31);
        }
    }
    if (lane == 0) sm.sched = sc;
}

// The CTA whose non-empty range [cstart[c], cstart[c+1]) holds global tile g.
__device__ __forceinline__ int cta_of_tile(const int* cstart, int n_eff, int g)
{
    int lo = 0, hi = n_eff - 1;
    while (lo < hi) {  // largest c with cstart[c] <= g
        const int mid = (lo + hi + 1) >> 1;
        if (cstart[mid] <= g) lo = mid;
        else hi = mid - 1;
    }
    return lo;
}

// Index, in q-head units, of the first q head of sequence s in the output,
// or -1 (recorded) when its row lies outside the destinations.
__device__ __forceinline__ int64_t out_head_base(const DecodeParams& p, int s)
{
    const int row = p.out_rows ? p.out_rows[s] : s;
    if (row < 0 || row >= p.out_row_limit) {
        record_status(p.status, HX_ERR_CAPACITY);
        return -1;
    }
    return (int64_t)row * p.out_hq + p.out_head0;
}

// Stores n_rows finished rows (fp32 in shared memory, 128 dims each, row r
// at src + r * src_stride) as q heads qh0 .. qh0 + n_rows - 1 of sequence s
// into every destination, threads tid, tid + nthr, ... each taking one
// 16-byte chunk of one row of one destination at a time (so a row crosses
// NVLink as full 16-byte writes).  Rounds like store_out.
__device__ void store_rows(const DecodeParams& p, int s, int qh0, const float* src, int src_stride,
                           int n_rows, int tid, int nthr)
{
    const int64_t base = out_head_base(p, s);
    if (base < 0) return;
    if (!p.out_vec) {
        for (int idx = tid; idx < n_rows * 128; idx += nthr) {
            const int r = idx / 128, d = idx % 128;
            const float val = src[r * src_stride + d];
            const int64_t oi = (base + qh0 + r) * 128 + d;
            for (int k = 0; k < p.n_outs; ++k) {
                if (p.out_f32) static_cast<float*>(p.outs[k])[oi] = val;
                else static_cast<__half*>(p.outs[k])[oi] = __float2half_rn(val);
            }
        }
        return;
    }
    const int chunks = p.out_f32 ? 32 : 16;  // 16-byte chunks per row
    const int per_dest = n_rows * chunks;
    for (int idx = tid; idx < p.n_outs * per_dest; idx += nthr) {
        const int k = idx / per_dest, rem = idx - k * per_dest;
        const int r = rem / chunks, c = rem - r * chunks;
        const float* f = src + r * src_stride;
        const int64_t row = (base + qh0 + r) * 128;
        if (p.out_f32) {
            *reinterpret_cast<float4*>(static_cast<float*>(p.outs[k]) + row + 4 * c) =
                *reinterpret_cast<const float4*>(f + 4 * c);
        } else {
            const float4 a = *reinterpret_cast<const float4*>(f + 8 * c);
            const float4 b = *reinterpret_cast<const float4*>(f + 8 * c + 4);
            *reinterpret_cast<uint4*>(static_cast<__half*>(p.outs[k]) + row + 8 * c) =
                make_uint4(pack_half2(a.x, a.y), pack_half2(a.z, a.w), pack_half2(b.x, b.y),
                           pack_half2(b.z, b.w));
        }
    }
}

// Sequences with no positions attend to nothing: their rows are zeros.
__device__ void zero_empty_outputs(const DecodeParams& p)
{
    const int lane = threadIdx.x & 31;
    for (int s = 0; s < p.n_seqs; ++s) {
        const int len = p.lengths[s];
        if (len >= 1 && len <= p.view.capacity) continue;
        if (lane == 0) record_status(p.status, HX_ERR_CAPACITY);
        if (len >= 1) continue;  // over capacity: clamped, still attended
        const int64_t base = out_head_base(p, s);
        if (base < 0) continue;
        for (int e = lane; e < p.hq * 128; e += 32) {
            const int64_t oi = base * 128 + e;
            for (int k = 0; k < p.n_outs; ++k) {
                if (p.out_f32) static_cast<float*>(p.outs[k])[oi] = 0.f;
                else static_cast<__half*>(p.outs[k])[oi] = __float2half_rn(0.f);
            }
        }
    }
}

// Folded combine: merges the np pieces of segment `seg` (slot seg, then slot
// n_seg + ca + k for k = 1 .. np-1, as the decode kernel writes them) by
// log-sum-exp for every q row of the group, and writes the normalised rows
// to dst ([group][128] fp32 in shared memory).  Warp w takes rows w, w + 4,
// ...; lane i dims 4i .. 4i+3.  Loads go to L2 (the pieces come from other
// SMs), four pieces at a time, merged online.
__device__ void fold_merge_rows(const DecodeParams& p, int seg, int n_seg, int ca, int np,
                                float* dst, int w, int lane)
{
    for (int r = w; r < p.group; r += kDecConsumerWarps) {
        float M = -INFINITY, L = 0.f;
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int j0 = 0; j0 < np; j0 += 4) {
            float2 ml[4];
            float4 ov[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const int j = j0 + k;
                ml[k] = make_float2(-INFINITY, 0.f);
                ov[k] = make_float4(0.f, 0.f, 0.f, 0.f);
                if (j < np) {
                    const int64_t slot = j == 0 ? seg : (int64_t)n_seg + ca + j;
                    ml[k] = __ldcg(&p.ws_ml[slot * p.group + r]);
                    ov[k] = __ldcg(reinterpret_cast<const float4*>(p.ws_o + (slot * p.group + r) * 128) + lane);
                }
            }
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const float Mn = fmaxf(M, ml[k].x);
                const float Mu = Mn == -INFINITY ? 0.f : Mn;
                const float a = fast_exp2(M - Mu), b = fast_exp2(ml[k].x - Mu);
                L = L * a + ml[k].y * b;
                acc.x = acc.x * a + ov[k].x * b;
                acc.y = acc.y * a + ov[k].y * b;
                acc.z = acc.z * a + ov[k].z * b;
                acc.w = acc.w * a + ov[k].w * b;
                M = Mn;
            }
        }
        *reinterpret_cast<float4*>(dst + r * 128 + 4 * lane) =
            make_float4(acc.x / L, acc.y / L, acc.z / L, acc.w / L);
    }
}

// Append-and-decode, producer warp: writes the new token of sequence slot s
// (cache sequence seq) for kv head h at position pos into physical block pb,
// with K1's bias rounding and rotation; lane l takes the pairs (l, l + 64) and
// (l + 32, l + 96).
template <typename T>
__device__ void append_new_token(const DecodeParams& p, int s, int h, int pos, int64_t pb, int lane)
{
    const KVView& v = p.view;
    const int64_t src = ((int64_t)s * v.hkv + h) * 128;
    const T* k = static_cast<const T*>(p.k_new) + src;
    const T* vv = static_cast<const T*>(p.v_new) + src;
    const T* bk = p.bk ? static_cast<const T*>(p.bk) + (int64_t)h * 128 : nullptr;
    const T* bv = p.bv ? static_cast<const T*>(p.bv) + (int64_t)h * 128 : nullptr;
    const float2* cs = p.rope ? p.rope + (int64_t)pos * 64 : nullptr;
    const int64_t off = pb * v.block_stride + (int64_t)h * v.head_stride + (int64_t)(pos % kBlockTokens) * 256;
    __half* kd = reinterpret_cast<__half*>(v.k + off);
    __half* vd = reinterpret_cast<__half*>(v.v + off);
    // every load first (one round of latency), then the stores
    float kx[4], vx[4];
    float2 c2[2] = {make_float2(1.f, 0.f), make_float2(1.f, 0.f)};
#pragma unroll
    for (int u = 0; u < 4; ++u) {
        const int d = lane + 32 * u;  // u = 0, 1: x1 of pair lane + 32u; u = 2, 3: its x2
        kx[u] = ld_bias(k + d, bk ? bk + d : nullptr);
        vx[u] = ld_bias(vv + d, bv ? bv + d : nullptr);
    }
    if (cs) {
        c2[0] = cs[lane];
        c2[1] = cs[lane + 32];
#pragma unroll
        for (int u = 0; u < 2; ++u) rotate(kx[u], kx[u + 2], c2[u], kx[u], kx[u + 2]);
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
        kd[lane + 32 * u] = __float2half_rn(kx[u]);
        vd[lane + 32 * u] = __float2half_rn(vx[u]);
    }
}

// Append-and-decode, consumers: this lane's B-operand words of q row r of
// the piece (q head qh of sequence slot s), with K1's bias and rotation.  The
// lane holds dims 16kk + 2t4 + 8half (+1); the NeoX partner of a dim below 64
// sits at kk + 4 of the same lane, so the rotation needs no exchange.
template <typename T>
__device__ __forceinline__ void load_q_new(const DecodeParams& p, int s, int qh, const float2* cs,
                                           int t4, uint32_t (&qw)[8][2])
{
    const int64_t base = ((int64_t)s * p.hq + qh) * 128;
    const T* q = static_cast<const T*>(p.q) + base;
    const T* b = p.bq ? static_cast<const T*>(p.bq) + (int64_t)qh * 128 : nullptr;
    float x[8][2][2];
#pragma unroll
    for (int kk = 0; kk < 8; ++kk)
#pragma unroll
        for (int half = 0; half < 2; ++half)
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                const int d = 16 * kk + 2 * t4 + 8 * half + e;
                x[kk][half][e] = ld_bias(q + d, b ? b + d : nullptr);
            }
    if (cs) {
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
#pragma unroll
            for (int half = 0; half < 2; ++half)
#pragma unroll
                for (int e = 0; e < 2; ++e)
                    rotate(x[kk][half][e], x[kk + 4][half][e], cs[16 * kk + 2 * t4 + 8 * half + e],
                           x[kk][half][e], x[kk + 4][half][e]);
    }
#pragma unroll
    for (int kk = 0; kk < 8; ++kk)
#pragma unroll
        for (int half = 0; half < 2; ++half) qw[kk][half] = pack_half2(x[kk][half][0], x[kk][half][1]);
}

template <int ROWS, int STAGES, int CTAS_PER_SM>
__global__ void __launch_bounds__(kDecThreads, CTAS_PER_SM)
    decode_attention_kernel(const __grid_constant__ CUtensorMap tm_k,
                            const __grid_constant__ CUtensorMap tm_v, const DecodeParams p)
{
    constexpr int kDecStages = STAGES;
    extern __shared__ uint8_t smem_raw[];
    auto& sm = *reinterpret_cast<DecodeSmem<ROWS, STAGES>*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int cta = blockIdx.x, n_ctas = gridDim.x;
    const int n_seg = p.n_seqs * p.view.hkv;

    // With HX_KV_OVERLAP_LAUNCH this kernel may start before the previous one
    // on the stream (normally hx_rope_append) has finished.  Until pdl_wait()
    // it reads only lengths, seq_ids, the block table and cache positions
    // below each sequence's newest one; q, the newest position and every write
    // come after it.
    pdl_trigger();
    if (threadIdx.x == 0) {
        for (int i = 0; i < kDecStages; ++i) {
            mbar_init(&sm.full[i], 1);
            mbar_init(&sm.empty[i], kDecConsumerWarps);
        }
        fence_mbar_init();
    }
    if (warp == kDecConsumerWarps) plan_cta(p, cta, n_ctas, sm);
    __syncthreads();
    const Sched sc = sm.sched;
    const int count = sc.count;
    if (cta == 0 && warp == 0 && sc.odd_lengths) {
        // only when the plan saw an empty or over-capacity sequence, so the
        // common call adds no load after the wait to CTA 0's critical path
        pdl_wait();
        zero_empty_outputs(p);
    }
    if (count <= 0) return;
    const int g_first = sc.g_first, n_eff = sc.n_eff;
    Cursor cur{sc.s, sc.h, sc.j, sc.tiles, sc.len, sc.seq};

    if (warp == kDecConsumerWarps) {
        // ------------------------------------------------------------ producer
        // The whole warp walks the tiles (the cursor is uniform across
        // lanes); lane 0 issues the copies.  Block-table entries come in
        // windows of 32 consecutive blocks of one sequence, one coalesced
        // load per window, so issuing the first ring of tiles costs one
        // round of global loads instead of one per tile.
        if (lane == 0) {
            prefetch_tensormap(&tm_k);
            prefetch_tensormap(&tm_v);
        }
        const uint64_t pol = l2_evict_first_policy();
        const KVView& v = p.view;
        bool waited = false;
        int win_seq = -1, win_j0 = 0;  // window: blocks [win_j0, win_j0 + 32) of win_seq
        int64_t win_pb = -1;           // this lane's entry: block win_j0 + lane
        for (int i = 0; i < count; ++i) {
            const int st = i % kDecStages;
            const uint32_t round = (uint32_t)(i / kDecStages);
            bool ok = true;
            if (lane == 0 && i >= kDecStages) ok = mbar_wait(&sm.empty[st], (round - 1) & 1);
            if (!__shfl_sync(0xffffffffu, ok, 0)) {
                if (lane == 0) record_status(p.status, HX_ERR_TIMEOUT);
                return;
            }
            if (!waited && cur.j == cur.tiles - 1) {
                pdl_wait();  // the segment's last tile holds the newest position
                waited = true;
            }
            if (cur.seq != win_seq || cur.j < win_j0 || cur.j >= win_j0 + 32) {
                win_seq = cur.seq;
                win_j0 = cur.j;
                win_pb = phys_block(v, win_seq, win_j0 + lane);
            }
            const int64_t pb = __shfl_sync(0xffffffffu, win_pb, cur.j - win_j0);
            if (p.k_new && cur.j == cur.tiles - 1) {
                // append-and-decode: this CTA holds the segment's newest tile,
                // so it writes the new token there before loading the tile
                // the cursor's length is the sequence's unless the plan saw an
                // empty or over-capacity one (then the raw length decides)
                const int len = sc.odd_lengths ? p.lengths[cur.s] : cur.len;
                const int pos = len - 1;
                if (len >= 1 && len <= v.capacity && pb >= 0 && (!p.rope || pos < p.rope_max_pos)) {
                    if (p.q_f32) append_new_token<float>(p, cur.s, cur.h, pos, pb, lane);
                    else append_new_token<__half>(p, cur.s, cur.h, pos, pb, lane);
                    fence_proxy_async_global();  // the writes before the tile's TMA load
                } else if (lane == 0) {
                    record_status(p.status, HX_ERR_CAPACITY);
                }
                __syncwarp();
            }
            if (lane == 0) {
                if (pb < 0) {
                    // unmapped block: no copy is issued; the consumers still get
                    // a completed phase (stale data) and the status word records it
                    record_status(p.status, HX_ERR_CAPACITY);
                    mbar_arrive(&sm.full[st]);
                } else {
                    const int64_t rel = (pb * v.block_stride + (int64_t)cur.h * v.head_stride) / 256;
                    const int row_k = (int)(v.k_row0 + rel), row_v = (int)(v.v_row0 + rel);
                    mbar_arrive_expect_tx(&sm.full[st], kStageTxBytes);
                    uint8_t* kd = sm.stage[st][0];
                    uint8_t* vd = sm.stage[st][1];
                    tma_load_2d(kd, &tm_k, 0, row_k, &sm.full[st], pol);
                    tma_load_2d(kd + kHalfTileBytes, &tm_k, 64, row_k, &sm.full[st], pol);
                    tma_load_2d(vd, &tm_v, 0, row_v, &sm.full[st], pol);
                    tma_load_2d(vd + kHalfTileBytes, &tm_v, 64, row_v, &sm.full[st], pol);
                }
            }
            cursor_next(cur, p);
        }
        if (lane != 0) return;
        // Wait for the last copies to land before the CTA may exit.
        for (int i = count > kDecStages ? count - kDecStages : 0; i < count; ++i) {
            const int st = i % kDecStages;
            if (!mbar_wait(&sm.full[st], (uint32_t)(i / kDecStages) & 1)) {
                record_status(p.status, HX_ERR_TIMEOUT);
                return;
            }
        }
        return;
    }

    // ---------------------------------------------------------------- consumers
    pdl_wait();  // q and the newest cache position come from the previous kernel
    const int g = lane >> 2, t4 = lane & 3;
    const int w = warp;
    // The MMAs run transposed: positions are the M side (16 per warp) and the
    // GQA group's q rows the N side, in NT n-tiles of 8 rows, so a group of up
    // to 8 rows needs no padding.  S^T = K Q^T, then O^T += V^T P^T.
    constexpr int NT = ROWS / 8;
    uint32_t qb[NT][8][2];  // B operand: q row 8nt+g, dims 16kk+2t4 (+8)
    float o[NT][8][4];      // O^T: dims 16mt+g (+8) x rows 8nt+2t4 (+1)
    float mrow[NT][2], lrow[NT][2];  // rows 8nt+2t4+c: running max, this lane's partial sum
    bool piece_from_seg_start = false;
    bool piece_whole = false;  // the piece is its whole segment (no other CTA shares it)
    bool dead = false;  // a bounded wait ran out
    const uint32_t stage_base = smem_u32(&sm.stage[0][0][0]);
    // ldmatrix row addresses (before swizzle) for this lane
    const int lm_mi = lane >> 3, lm_r = lane & 7;

    for (int i = 0; i < count; ++i) {
        if (i == 0 || cur.j == 0) {
            // new piece: load the packed GQA group of q rows for (s, h)
            piece_from_seg_start = (cur.j == 0);
            {
                // global tile range [a, b) of this segment: one CTA or several?
                const int a = g_first + i - cur.j, b = a + cur.tiles;
                piece_whole = cta_of_tile(sm.cstart, n_eff, a) == cta_of_tile(sm.cstart, n_eff, b - 1);
            }
            const int64_t qrow0 = ((int64_t)cur.s * p.hq + (int64_t)cur.h * p.group) * 128;
            const float2* q_cs = nullptr;  // append-and-decode: the new token's (cos, sin) row
            if (p.k_new && p.rope) {
                const int pos = cur.len - 1;  // as the producer's append (clamped lengths are an error)
                if (pos >= 0 && pos < p.rope_max_pos) q_cs = p.rope + (int64_t)pos * 64;
            }
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
                const int r = 8 * nt + g;
                if (p.k_new) {
                    if (r < p.group) {
                        const int qh = cur.h * p.group + r;
                        if (p.q_f32) load_q_new<float>(p, cur.s, qh, q_cs, t4, qb[nt]);
                        else load_q_new<__half>(p, cur.s, qh, q_cs, t4, qb[nt]);
                    } else {
#pragma unroll
                        for (int kk = 0; kk < 8; ++kk) qb[nt][kk][0] = qb[nt][kk][1] = 0u;
                    }
                }
                if (!p.k_new) {
#pragma unroll
                    for (int kk = 0; kk < 8; ++kk) {
#pragma unroll
                        for (int half = 0; half < 2; ++half) {  // dims 16kk+2t4 (+8)
                            uint32_t val = 0;
                            if (r < p.group) {
                                const int64_t idx = qrow0 + (int64_t)r * 128 + 16 * kk + 2 * t4 + 8 * half;
                                if (p.q_f32) {
                                    const float2 f = *reinterpret_cast<const float2*>(
                                        static_cast<const float*>(p.q) + idx);
                                    val = pack_half2(f.x, f.y);
                                } else {
                                    val = *reinterpret_cast<const uint32_t*>(
                                        static_cast<const __half*>(p.q) + idx);
                                }
                            }
                            qb[nt][kk][half] = val;
                        }
                    }
                }
#pragma unroll
                for (int mt = 0; mt < 8; ++mt) o[nt][mt][0] = o[nt][mt][1] = o[nt][mt][2] = o[nt][mt][3] = 0.f;
                mrow[nt][0] = mrow[nt][1] = -INFINITY;
                lrow[nt][0] = lrow[nt][1] = 0.f;
            }
        }

        const int st = i % kDecStages;
        if (!dead) {
            const bool ok = mbar_wait(&sm.full[st], (uint32_t)(i / kDecStages) & 1);
            if (__any_sync(0xffffffffu, !ok)) {
                // The tile never arrived: record it and stop waiting, but keep
                // running the loop (on stale shared memory, in bounds) so the
                // other consumer warps never wait on this one at a named
                // barrier.  The output of this call is then invalid.
                if (lane == 0) record_status(p.status, HX_ERR_TIMEOUT);
                dead = true;
            }
        }
        const int valid = min(kBlockTokens, cur.len - cur.j * kBlockTokens);
        const uint32_t kb = stage_base + st * 2 * kTileBytes;
        const uint32_t vb = kb + kTileBytes;
        const int tok0 = 16 * w;
        if (valid < tok0 + 16) {
            // Positions past the sequence end hold stale or out-of-range
            // bytes; zero this warp's V rows there so 0 * garbage cannot
            // reach the accumulators.
            uint8_t* vrow = sm.stage[st][1];
            const int lo = max(valid, tok0);
            const int nchunks = (tok0 + 16 - lo) * 16;
            for (int c = lane; c < nchunks; c += 32) {
                const int row = lo + c / 16, chunk = c % 16;
                *reinterpret_cast<uint4*>(vrow + (chunk >> 3) * kHalfTileBytes + row * 128 +
                                          (chunk & 7) * 16) = make_uint4(0, 0, 0, 0);
            }
            fence_proxy_async_smem();
            __syncwarp();
        }

        // S^T = K Q^T for this warp's 16 positions (two accumulator chains)
        float sa[NT][4], sb[NT][4];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int e = 0; e < 4; ++e) sa[nt][e] = sb[nt][e] = 0.f;
        {
            const int tok = tok0 + 8 * (lm_mi >> 1) + lm_r;
#pragma unroll
            for (int kk = 0; kk < 8; ++kk) {
                const int chunk = 2 * kk + (lm_mi & 1);
                const uint32_t addr = kb + (chunk >> 3) * kHalfTileBytes + tok * 128 +
                                      (((chunk & 7) ^ (tok & 7)) << 4);
                uint32_t r0, r1, r2, r3;
                ldmatrix_x4(r0, r1, r2, r3, addr);
                const uint32_t a[4] = {r0, r2, r1, r3};  // positions x dims fragment
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) {
                    if (kk & 1) mma_16816(sb[nt], a, qb[nt][kk][0], qb[nt][kk][1]);
                    else mma_16816(sa[nt], a, qb[nt][kk][0], qb[nt][kk][1]);
                }
            }
        }
        // online softmax per q row; this lane holds rows 8nt+2t4+c at positions
        // tok0+g (element c) and tok0+g+8 (element c+2); a row's max is
        // reduced over the eight lanes that share t4
        uint32_t pb[NT][2];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            float pr[4];
#pragma unroll
            for (int c = 0; c < 2; ++c) {
                const float x0 = (sa[nt][c] + sb[nt][c]) * p.scale_log2;
                const float x1 = (sa[nt][c + 2] + sb[nt][c + 2]) * p.scale_log2;
                const float s0 = tok0 + g < valid ? x0 : -INFINITY;
                const float s1 = tok0 + g + 8 < valid ? x1 : -INFINITY;
                float mx = fmaxf(s0, s1);
                mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
                mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
                mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
                const float mn = fmaxf(mrow[nt][c], mx);
                const float mu = mn == -INFINITY ? 0.f : mn;
                const float al = fast_exp2(mrow[nt][c] - mu);
                pr[c] = fast_exp2(s0 - mu);
                pr[c + 2] = fast_exp2(s1 - mu);
                lrow[nt][c] = lrow[nt][c] * al + (pr[c] + pr[c + 2]);
                mrow[nt][c] = mn;
#pragma unroll
                for (int mt = 0; mt < 8; ++mt) {
                    o[nt][mt][c] *= al;
                    o[nt][mt][c + 2] *= al;
                }
            }
            // P^T as the B operand of the P.V step: transpose the two 8x8
            // (positions x rows) halves in registers
            pb[nt][0] = movmatrix_trans(pack_half2(pr[0], pr[1]));
            pb[nt][1] = movmatrix_trans(pack_half2(pr[2], pr[3]));
        }

        // O^T += V^T P^T over this warp's 16 positions, 8 m-tiles of 16 dims
        {
            const int tok = tok0 + 8 * (lm_mi >> 1) + lm_r;
#pragma unroll
            for (int mt = 0; mt < 8; ++mt) {
                const int chunk = 2 * mt + (lm_mi & 1);
                const uint32_t addr = vb + (chunk >> 3) * kHalfTileBytes + tok * 128 +
                                      (((chunk & 7) ^ (tok & 7)) << 4);
                uint32_t a[4];
                ldmatrix_x4_trans(a[0], a[1], a[2], a[3], addr);
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) mma_16816(o[nt][mt], a, pb[nt][0], pb[nt][1]);
            }
        }
        __syncwarp();
        const bool seg_end = (cur.j == cur.tiles - 1);
        const bool piece_end = seg_end || i == count - 1;
        if (!piece_end && lane == 0) mbar_arrive(&sm.empty[st]);
        if (piece_end) {
            // ---- merge the four warps' partials of this piece, in the stage
            // just consumed (released only once the merge is done)
            auto merge_o = reinterpret_cast<float (*)[ROWS][128]>(&sm.stage[st][0][0]);
            asm volatile("bar.sync 1, %0;" ::"n"(kDecConsumerWarps * 32) : "memory");  // stage read by all
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
                for (int c = 0; c < 2; ++c) {
                    float lq = lrow[nt][c];
                    lq += __shfl_xor_sync(0xffffffffu, lq, 4);
                    lq += __shfl_xor_sync(0xffffffffu, lq, 8);
                    lq += __shfl_xor_sync(0xffffffffu, lq, 16);
                    const int r = 8 * nt + 2 * t4 + c;
                    if (r < p.group) {
                        if (g == 0) {
                            sm.merge_m[w][r] = mrow[nt][c];
                            sm.merge_l[w][r] = lq;
                        }
#pragma unroll
                        for (int mt = 0; mt < 8; ++mt) {
                            merge_o[w][r][16 * mt + g] = o[nt][mt][c];
                            merge_o[w][r][16 * mt + g + 8] = o[nt][mt][c + 2];
                        }
                    }
                }
            }
            asm volatile("bar.sync 1, %0;" ::"n"(kDecConsumerWarps * 32) : "memory");
            const int d = threadIdx.x;  // 0..127
            const bool whole = piece_whole;
            const int seg = cur.s * p.view.hkv + cur.h;
            const int slot = piece_from_seg_start ? seg : (n_seg + cta);
            // warp w merges rows w, w+4, ...; each lane four dims (16-byte accesses)
            for (int r = w; r < p.group; r += kDecConsumerWarps) {
                float M = -INFINITY;
#pragma unroll
                for (int ww = 0; ww < kDecConsumerWarps; ++ww) M = fmaxf(M, sm.merge_m[ww][r]);
                const float Mu = M == -INFINITY ? 0.f : M;
                float L = 0.f;
                float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
                for (int ww = 0; ww < kDecConsumerWarps; ++ww) {
                    const float wgt = fast_exp2(sm.merge_m[ww][r] - Mu);
                    L += wgt * sm.merge_l[ww][r];
                    const float4 v = *reinterpret_cast<const float4*>(&merge_o[ww][r][4 * lane]);
                    acc.x += wgt * v.x; acc.y += wgt * v.y; acc.z += wgt * v.z; acc.w += wgt * v.w;
                }
                if (whole) {
                    // row r is read and rewritten only by this warp's lanes
                    *reinterpret_cast<float4*>(&merge_o[0][r][4 * lane]) =
                        make_float4(acc.x / L, acc.y / L, acc.z / L, acc.w / L);
                } else {
                    *reinterpret_cast<float4*>(p.ws_o + ((int64_t)slot * p.group + r) * 128 + 4 * lane) = acc;
                    if (lane == 0) p.ws_ml[(int64_t)slot * p.group + r] = make_float2(M, L);
                }
            }
            if (whole) {
                asm volatile("bar.sync 1, %0;" ::"n"(kDecConsumerWarps * 32) : "memory");
                store_rows(p, cur.s, cur.h * p.group, &merge_o[0][0][0], 128, p.group, d,
                           kDecConsumerWarps * 32);
            } else if (p.fold_cnt) {
                // Folded combine: count this piece in; the CTA that brings
                // the segment's last piece merges all of its pieces.
                asm volatile("bar.sync 1, %0;" ::"n"(kDecConsumerWarps * 32) : "memory");
                if (threadIdx.x == 0) {
                    const int a = g_first + i - cur.j;  // the segment's first global tile
                    const int ca = cta_of_tile(sm.cstart, n_eff, a);
                    const int np = cta_of_tile(sm.cstart, n_eff, a + cur.tiles - 1) - ca + 1;
                    fence_acq_rel_gpu();  // this CTA's partials before the arrival
                    const unsigned old = atomicInc(p.fold_cnt + seg, (unsigned)(np - 1));
                    const bool last = old == (unsigned)(np - 1);  // the counter is back to 0
                    if (last) fence_acq_rel_gpu();  // the other pieces after it
                    sm.fold_ca = last ? ca : -1;
                    sm.fold_np = np;
                }
                asm volatile("bar.sync 1, %0;" ::"n"(kDecConsumerWarps * 32) : "memory");
                const int ca = sm.fold_ca;
                if (ca >= 0) {
                    fold_merge_rows(p, seg, n_seg, ca, sm.fold_np, &merge_o[0][0][0], w, lane);
                    asm volatile("bar.sync 1, %0;" ::"n"(kDecConsumerWarps * 32) : "memory");
                    store_rows(p, cur.s, cur.h * p.group, &merge_o[0][0][0], 128, p.group, d,
                               kDecConsumerWarps * 32);
                }
            }
            fence_proxy_async_smem();  // the producer's next copy into this stage comes after
            asm volatile("bar.sync 1, %0;" ::"n"(kDecConsumerWarps * 32) : "memory");
            if (lane == 0) mbar_arrive(&sm.empty[st]);
        }
        cursor_next(cur, p);
    }
}

// Split-K combine: one CTA (128 threads, one per dim) per (segment, q row of
// the group), launched right after the decode kernel as a programmatic
// dependent, so it is resident early and starts as soon as the decode grid
// has finished.  Segments that one CTA covered were already written by the
// decode kernel.  The pieces are slot `seg` (the one starting at the
// segment's first tile) then slot n_seg + c for each CTA c whose non-empty
// range starts inside the segment.  The four warps split the pieces and
// merge their share online (one round of loads per 32 pieces); the warps'
// results are then merged in shared memory.
//
// Items (segment, q row) are numbered seg * group + r; CTA b takes items b,
// b + gridDim.x, ...; the launch gives one CTA per item, since each item is
// a short chain of dependent loads and they overlap best as separate CTAs.
template <int kSub>  // O loads in flight per lane
__global__ void __launch_bounds__(128)
    decode_combine_kernel(const DecodeParams p, int grid_ctas)
{
    pdl_trigger();
    const int hkv = p.view.hkv;
    const int n_items = p.n_seqs * hkv * p.group;
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
    __shared__ int sh_range[4];  // a, b, T, n_eff
    __shared__ int slot_list[kMaxPieces];
    __shared__ float w_m[4], w_l[4];
    __shared__ __align__(16) float w_acc[4][128];
    __shared__ __align__(16) float row_buf[128];
    __shared__ int sh_np;
    for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
    const int seg = item / p.group, r = item % p.group;
    const int s = seg / hkv, h = seg % hkv;
    if (warp == 0) {
        int before = 0, total = 0;
        for (int base = 0; base < p.n_seqs; base += 32) {
            const int si = base + lane;
            int tl = si < p.n_seqs ? tiles_of(clamp_len(p.lengths[si], p.view.capacity)) : 0;
            int tb = si < s ? tl : 0;
#pragma unroll
            for (int o = 16; o; o >>= 1) {
                tl += __shfl_xor_sync(0xffffffffu, tl, o);
                tb += __shfl_xor_sync(0xffffffffu, tb, o);
            }
            total += tl;
            before += tb;
        }
        if (lane == 0) {
            const int tiles = tiles_of(clamp_len(p.lengths[s], p.view.capacity));
            const long long T = (long long)total * hkv;
            const int valid_T = T < (1ll << 31) / kMaxPieces ? (int)T : 0;
            const int n_eff = max(1, min(grid_ctas, (valid_T + kMinTilesPerCta - 1) / kMinTilesPerCta));
            sh_range[0] = before * hkv + h * tiles;
            sh_range[1] = sh_range[0] + tiles;
            sh_range[2] = valid_T;
            sh_range[3] = n_eff;
        }
    }
    __syncthreads();
    const int a = sh_range[0], b = sh_range[1], T = sh_range[2], n_eff = sh_range[3];
    auto cstart = [&](int c) { return (int)((unsigned)T * (unsigned)c / (unsigned)n_eff); };
    if (t == 0) sh_np = 0;
    if (t == 0 && a < b && T > 0) {
        int c = (int)((long long)a * n_eff / T);
        while (c + 1 < n_eff && cstart(c + 1) <= a) ++c;
        while (c > 0 && cstart(c) > a) --c;
        int np = 0;
        slot_list[np++] = seg;
        const int n_seg = p.n_seqs * hkv;
        for (int cc = c + 1; cc < n_eff && cstart(cc) < b && np < kMaxPieces; ++cc)
            if (cstart(cc + 1) > cstart(cc)) slot_list[np++] = n_seg + cc;
        sh_np = np;
    }
    __syncthreads();
    const int np = sh_np;  // <= 1: the decode kernel wrote this output itself
    if (np > 1) {
        pdl_wait();  // the pieces come from the decode grid
        // Warp w merges pieces w, w + 4, ... (online, in groups of 32): lane
        // i holds one piece's (m, l); each lane accumulates dims 4*lane..+3
        // of every piece's O.  All loads of a group are independent, so a
        // group costs one round of L2 latency.
        const int n_w = np > warp ? (np - warp + 3) / 4 : 0;
        float Mw = -INFINITY, Lw = 0.f;
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int base = 0; base < n_w; base += 32) {
            const int cnt = min(32, n_w - base);
            const float2 ml = lane < cnt
                ? __ldcg(&p.ws_ml[(int64_t)slot_list[warp + 4 * (base + lane)] * p.group + r])
                : make_float2(-INFINITY, 0.f);
            float4 ov[kSub];
#pragma unroll
            for (int j = 0; j < kSub; ++j)
                ov[j] = j < cnt ? __ldcg(reinterpret_cast<const float4*>(
                                      p.ws_o + ((int64_t)slot_list[warp + 4 * (base + j)] * p.group + r) * 128) + lane)
                                : make_float4(0.f, 0.f, 0.f, 0.f);
            float Mc = ml.x;
#pragma unroll
            for (int o = 16; o; o >>= 1) Mc = fmaxf(Mc, __shfl_xor_sync(0xffffffffu, Mc, o));
            const float Mn = fmaxf(Mw, Mc);
            const float Mu = Mn == -INFINITY ? 0.f : Mn;
            const float sc = fast_exp2(Mw - Mu);  // 0 while nothing is merged
            acc.x *= sc; acc.y *= sc; acc.z *= sc; acc.w *= sc;
            const float wl = fast_exp2(ml.x - Mu);  // 0 for lanes without a piece
            float lsum = wl * ml.y;
#pragma unroll
            for (int o = 16; o; o >>= 1) lsum += __shfl_xor_sync(0xffffffffu, lsum, o);
            Lw = Lw * sc + lsum;
            Mw = Mn;
            for (int j0 = 0; j0 < cnt; j0 += kSub) {
                if (j0 > 0) {
#pragma unroll
                    for (int j = 0; j < kSub; ++j)
                        ov[j] = j0 + j < cnt ? __ldcg(reinterpret_cast<const float4*>(
                                                   p.ws_o + ((int64_t)slot_list[warp + 4 * (base + j0 + j)] * p.group + r) * 128) + lane)
                                             : make_float4(0.f, 0.f, 0.f, 0.f);
                }
#pragma unroll
                for (int j = 0; j < kSub; ++j) {
                    const float wj = __shfl_sync(0xffffffffu, wl, (j0 + j) & 31);
                    if (j0 + j < cnt) {
                        acc.x += wj * ov[j].x; acc.y += wj * ov[j].y;
                        acc.z += wj * ov[j].z; acc.w += wj * ov[j].w;
                    }
                }
            }
        }
        if (lane == 0) {
            w_m[warp] = Mw;
            w_l[warp] = Lw;
        }
        *reinterpret_cast<float4*>(&w_acc[warp][4 * lane]) = acc;
        __syncthreads();
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < 4; ++w) M = fmaxf(M, w_m[w]);
        const float Mu = M == -INFINITY ? 0.f : M;
        float num = 0.f, den = 0.f;
#pragma unroll
        for (int w = 0; w < 4; ++w) {
            const float f = fast_exp2(w_m[w] - Mu);
            num += f * w_acc[w][t];
            den += f * w_l[w];
        }
        row_buf[t] = num / den;
        __syncthreads();
        store_rows(p, s, h * p.group + r, row_buf, 128, 1, t, 128);
    }
    __syncthreads();  // shared state is rewritten by the next item
    }
    // CTA 0 always waits for the decode grid, so this grid never completes
    // before it: a kernel launched after this one as a programmatic
    // dependent then also waits for the decode kernel.
    if (blockIdx.x == 0) pdl_wait();
}

// Any head_dim (<= 256), any group: one CTA of 4 warps per (sequence, q
// head); warps take positions round-robin, lanes take dims; online softmax;
// warps merge in shared memory.  Used when the TMA path does not apply.
__global__ void __launch_bounds__(128)
    decode_generic_kernel(const DecodeParams p)
{
    const int s = blockIdx.x / p.hq, qh = blockIdx.x % p.hq;
    const int kvh = qh / p.group;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const KVView& v = p.view;
    const int hd = v.hd;
    const int len = clamp_len(p.lengths[s], v.capacity), seq = p.seq_ids[s];
    constexpr int kPer = kMaxHeadDim / 32;
    float qv[kPer], acc[kPer];
    const int64_t qoff = ((int64_t)s * p.hq + qh) * hd;
#pragma unroll
    for (int e = 0; e < kPer; ++e) {
        const int d = lane + 32 * e;
        qv[e] = 0.f;
        acc[e] = 0.f;
        if (d < hd)
            qv[e] = p.q_f32 ? static_cast<const float*>(p.q)[qoff + d]
                            : __half2float(static_cast<const __half*>(p.q)[qoff + d]);
    }
    float m = -INFINITY, l = 0.f;
    for (int pos = warp; pos < len; pos += 4) {
        const int64_t off = token_offset(v, seq, kvh, pos);
        if (off < 0) {
            record_status(p.status, HX_ERR_CAPACITY);
            break;
        }
        const __half* kr = reinterpret_cast<const __half*>(v.k + off);
        const __half* vr = reinterpret_cast<const __half*>(v.v + off);
        float dot = 0.f;
#pragma unroll
        for (int e = 0; e < kPer; ++e) {
            const int d = lane + 32 * e;
            if (d < hd) dot += qv[e] * __half2float(kr[d]);
        }
#pragma unroll
        for (int o = 16; o; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
        const float sc = dot * p.scale_log2;
        const float mn = fmaxf(m, sc);
        const float al = fast_exp2(m - mn), pr = fast_exp2(sc - mn);
        l = l * al + pr;
#pragma unroll
        for (int e = 0; e < kPer; ++e) {
            const int d = lane + 32 * e;
            acc[e] = acc[e] * al + (d < hd ? pr * __half2float(vr[d]) : 0.f);
        }
        m = mn;
    }
    __shared__ float sm_m[4], sm_l[4], sm_o[4][kMaxHeadDim];
    if (lane == 0) {
        sm_m[warp] = m;
        sm_l[warp] = l;
    }
#pragma unroll
    for (int e = 0; e < kPer; ++e) {
        const int d = lane + 32 * e;
        if (d < hd) sm_o[warp][d] = acc[e];
    }
    __syncthreads();
    float M = fmaxf(fmaxf(sm_m[0], sm_m[1]), fmaxf(sm_m[2], sm_m[3]));
    const float Mu = M == -INFINITY ? 0.f : M;
    for (int d = threadIdx.x; d < hd; d += blockDim.x) {
        float L = 0.f, o = 0.f;
        for (int ww = 0; ww < 4; ++ww) {
            const float wgt = fast_exp2(sm_m[ww] - Mu);
            L += wgt * sm_l[ww];
            o += wgt * sm_o[ww][d];
        }
        const float val = L > 0.f ? o / L : 0.f;
        const int64_t base = out_head_base(p, s);
        if (base < 0) break;
        const int64_t ooff = (base + qh) * hd;
        for (int k = 0; k < p.n_outs; ++k) {
            if (p.out_f32) static_cast<float*>(p.outs[k])[ooff + d] = val;
            else static_cast<__half*>(p.outs[k])[ooff + d] = __float2half_rn(val);
        }
    }
}

// Workspace layout: [fold counters][ws_o][ws_ml].  The counter block has the
// same size in every workspace, whatever the call, so that no call's partial
// results ever land on counters another call uses: the counters stay zero
// between calls (the CTA that completes a segment returns its counter to
// zero) once the workspace has been zero-filled before its first use.
constexpr int kFoldMaxSegments = 16384;
constexpr size_t kWsHeaderBytes = kFoldMaxSegments * sizeof(unsigned int);  // 64 KiB

static size_t decode_ws_bytes(int n_seqs, int hkv, int group, int n_ctas)
{
    const size_t slots = (size_t)n_seqs * hkv + n_ctas;
    return kWsHeaderBytes + slots * group * 128 * sizeof(float) + slots * group * sizeof(float2);
}

static void bind_workspace(DecodeParams& p, void* ws, int n_ctas)
{
    const size_t slots = (size_t)p.n_seqs * p.view.hkv + n_ctas;
    char* base = static_cast<char*>(ws) + kWsHeaderBytes;
    p.ws_o = reinterpret_cast<float*>(base);
    base += slots * p.group * 128 * sizeof(float);
    p.ws_ml = reinterpret_cast<float2*>(base);
}

static bool wide_shape(int group, int n_seg) { return group <= 8 && n_seg >= kWideMinSegments; }

// Wide calls merge their split-K pieces inside the decode kernel (each
// segment has only a few pieces there, so the CTA that completes a segment
// merges it at little cost); narrow calls have many pieces per segment
// (batch 1: ~37 at 32k positions) and keep the separate combine kernel,
// which spreads that merge over one CTA per (segment, q row).
static bool folded(int group, int n_seg) { return wide_shape(group, n_seg) && n_seg <= kFoldMaxSegments; }

// CTAs of a decode launch (the split-K workspace is sized by it).
static int decode_grid(int group, int n_seg)
{
    const int per_sm = wide_shape(group, n_seg) ? 2 : 1;
    return std::min(per_sm * num_sms(), kMaxPieces - 2);
}

template <int ROWS, int STAGES>
static size_t decode_smem_bytes()
{
    return sizeof(DecodeSmem<ROWS, STAGES>) + 1024;
}

// Sets the decode kernel's shared-memory attributes on the current device,
// once per device (again on ordinals past 63).
template <int ROWS, int STAGES, int CTAS_PER_SM>
static int ensure_decode_attrs()
{
    auto kernel = decode_attention_kernel<ROWS, STAGES, CTAS_PER_SM>;
    static std::atomic<bool> attr_set[64];
    int dev = 0;
    HX_CUDA_TRY(cudaGetDevice(&dev));
    if (dev >= 0 && dev < 64 && attr_set[dev].load(std::memory_order_acquire)) return HX_OK;
    HX_CUDA_TRY(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)decode_smem_bytes<ROWS, STAGES>()));
    HX_CUDA_TRY(cudaFuncSetAttribute(kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                                     (int)cudaSharedmemCarveoutMaxShared));
    if (dev >= 0 && dev < 64) attr_set[dev].store(true, std::memory_order_release);
    return HX_OK;
}

template <int ROWS, int STAGES, int CTAS_PER_SM>
static int launch_decode(const hx_kv_cache* c, const DecodeParams& p, int n_ctas,
                         cudaStream_t stream)
{
    auto kernel = decode_attention_kernel<ROWS, STAGES, CTAS_PER_SM>;
    const size_t smem = decode_smem_bytes<ROWS, STAGES>();
    if (int rc = ensure_decode_attrs<ROWS, STAGES, CTAS_PER_SM>()) return rc;
    const bool ov = (c->cfg.flags & HX_KV_OVERLAP_LAUNCH) != 0;
    cudaError_t e = launch_kernel(kernel, dim3(n_ctas), dim3(kDecThreads), smem, stream, ov,
                                  c->tm_k, c->tm_v, p);
    if (e != cudaSuccess) return cuda_fail(e, "decode_attention_kernel launch");
    if (int rc = check_launch("decode_attention_kernel")) return rc;
    if (p.fold_cnt) return HX_OK;  // the decode kernel merged its own pieces
    const int n_items = p.n_seqs * p.view.hkv * p.group;
    // Narrow calls (few segments, many pieces each) take 12 O loads per lane
    // in one round; wide calls have 2-3 pieces per item and keep the 8-load
    // (64-register) variant, which fits beside two decode CTAs per SM.
    e = launch_kernel(n_ctas <= num_sms() ? decode_combine_kernel<12> : decode_combine_kernel<8>,
                      dim3(n_items), dim3(128), 0, stream, true, p, n_ctas);
    if (e != cudaSuccess) return cuda_fail(e, "decode_combine_kernel launch");
    return check_launch("decode_combine_kernel");
}

}  // namespace hx

using namespace hx;

extern "C" size_t hx_decode_workspace_bytes(const hx_kv_cache* c, int n_seqs, int num_q_heads)
{
    if (!c || n_seqs < 1 || num_q_heads < 1) return 0;
    const int hkv = c->cfg.num_kv_heads;
    const int group = num_q_heads / hkv < 1 ? 1 : num_q_heads / hkv;
    return decode_ws_bytes(n_seqs, hkv, group, decode_grid(group, n_seqs * hkv));
}

namespace hx {

static int validate_decode(const hx_kv_cache* c, int layer, const void* q, int q_dtype,
                           const int32_t* seq_ids, const int32_t* lengths, int n_seqs,
                           int num_q_heads, int out_dtype)
{
    if (!c) return fail(HX_ERR_INVALID, "null cache");
    if (layer < 0 || layer >= c->cfg.num_layers) return fail(HX_ERR_INVALID, "layer %d out of range", layer);
    if (n_seqs < 0 || n_seqs > c->cfg.max_seqs)
        return fail(HX_ERR_INVALID, "n_seqs %d outside [0, %d]", n_seqs, c->cfg.max_seqs);
    if (n_seqs > 0 && (!q || !seq_ids || !lengths)) return fail(HX_ERR_INVALID, "null q/seq_ids/lengths");
    const int hkv = c->cfg.num_kv_heads;
    if (num_q_heads < hkv || num_q_heads % hkv)
        return fail(HX_ERR_INVALID, "num_q_heads %d must be a multiple of kv heads %d", num_q_heads, hkv);
    if ((q_dtype != HX_FP16 && q_dtype != HX_FP32) || (out_dtype != HX_FP16 && out_dtype != HX_FP32))
        return fail(HX_ERR_INVALID, "q/out dtype");
    return check_device(c->device, "the cache");
}

// Everything but the output placement (set by the caller afterwards).
static DecodeParams base_params(const hx_kv_cache* c, int layer, const void* q, int q_dtype,
                                const int32_t* seq_ids, const int32_t* lengths, int n_seqs,
                                int num_q_heads, float scale, int out_dtype)
{
    DecodeParams p{};
    p.view = make_view(c, layer);
    p.q = q;
    p.q_f32 = q_dtype == HX_FP32;
    p.seq_ids = seq_ids;
    p.lengths = lengths;
    p.n_seqs = n_seqs;
    p.hq = num_q_heads;
    p.group = num_q_heads / c->cfg.num_kv_heads;
    p.scale_log2 = scale * 1.4426950408889634f;
    p.out_hq = num_q_heads;
    p.out_row_limit = n_seqs;
    p.out_f32 = out_dtype == HX_FP32;
    return p;
}

static bool fast_path(const hx_kv_cache* c, const DecodeParams& p)
{
    return c->has_tmap && c->cfg.head_dim == 128 && p.group <= 16;
}

// Launches the decode of a filled-in parameter block (n_seqs >= 1).  The
// fast path needs `scratch` of decode_ws_bytes, checked by the caller.
static int run_decode(const hx_kv_cache* c, DecodeParams& p, void* scratch, cudaStream_t s)
{
    if (!fast_path(c, p)) {
        decode_generic_kernel<<<p.n_seqs * p.hq, 128, 0, s>>>(p);
        return check_launch("decode_generic_kernel");
    }
    const int n_seg = p.n_seqs * p.view.hkv;
    const int n_ctas = decode_grid(p.group, n_seg);
    bind_workspace(p, scratch, n_ctas);
    if (wide_shape(p.group, n_seg)) {
        if (folded(p.group, n_seg)) p.fold_cnt = static_cast<unsigned int*>(scratch);
        return launch_decode<8, 3, 2>(c, p, n_ctas, s);
    }
    if (p.group <= 8) return launch_decode<8, 6, 1>(c, p, n_ctas, s);
    return launch_decode<16, 6, 1>(c, p, n_ctas, s);
}

static size_t needed_scratch(const hx_kv_cache* c, const DecodeParams& p)
{
    if (!fast_path(c, p)) return 0;
    return decode_ws_bytes(p.n_seqs, p.view.hkv, p.group,
                           decode_grid(p.group, p.n_seqs * p.view.hkv));
}

}  // namespace hx

extern "C" int hx_decode_attention(const hx_kv_cache* c, int layer, const void* q, int q_dtype,
                                   const int32_t* seq_ids, const int32_t* lengths, int n_seqs,
                                   int num_q_heads, float scale, void* out, int out_dtype,
                                   void* workspace, size_t workspace_bytes, hx_stream_t stream)
{
    HX_NVTX_RANGE("hx_decode_attention");
    if (int rc = validate_decode(c, layer, q, q_dtype, seq_ids, lengths, n_seqs, num_q_heads,
                                 out_dtype))
        return rc;
    if (n_seqs > 0 && !out) return fail(HX_ERR_INVALID, "null out");
    if (n_seqs == 0) return HX_OK;
    DecodeParams p = base_params(c, layer, q, q_dtype, seq_ids, lengths, n_seqs, num_q_heads,
                                 scale, out_dtype);
    p.out = out;
    p.outs[0] = out;
    p.n_outs = 1;
    p.out_vec = reinterpret_cast<uintptr_t>(out) % 16 == 0;
    p.status = status_word();
    const size_t need = needed_scratch(c, p);
    if (need && (!workspace || workspace_bytes < need))
        return fail(HX_ERR_INVALID, "workspace of %zu bytes is smaller than the %zu needed",
                    workspace_bytes, need);
    return run_decode(c, p, workspace, (cudaStream_t)stream);
}

namespace hx {

// Append-and-decode: checks the new-token inputs and puts them into p (whose
// base fields are set).  Only the fast path fuses the append.
static int append_params(const hx_kv_cache* c, const hx_append_spec* a, DecodeParams& p)
{
    if (!a) return fail(HX_ERR_INVALID, "null append spec");
    if (p.n_seqs > 0 && (!a->k || !a->v)) return fail(HX_ERR_INVALID, "null k/v rows");
    if (a->table) {
        if (a->table->cfg.head_dim != c->cfg.head_dim)
            return fail(HX_ERR_INVALID, "rope table head_dim %d != cache head_dim %d",
                        a->table->cfg.head_dim, c->cfg.head_dim);
        if (int rc = check_device(a->table->device, "the rope table")) return rc;
    }
    if (!fast_path(c, p))
        return fail(HX_ERR_UNSUPPORTED,
                    "append-and-decode needs head_dim 128 and at most 16 q heads per kv head "
                    "(hx_rope_append then hx_decode_attention cover the rest)");
    p.k_new = a->k;
    p.v_new = a->v;
    p.bq = a->bq;
    p.bk = a->bk;
    p.bv = a->bv;
    p.rope = a->table ? a->table->d_cos_sin : nullptr;
    p.rope_max_pos = a->table ? a->table->cfg.max_pos : 0;
    return HX_OK;
}

// Gathering decode, plain or with the new tokens' append (a != null): the
// rows go to every rank's buffer (the endpoints and the epoch exchange live
// in dist.cu).
static int decode_gather(const hx_kv_cache* c, int layer, const void* q, int q_dtype,
                         const hx_append_spec* a, const int32_t* seq_ids, const int32_t* lengths,
                         int n_seqs, int num_q_heads, float scale, hx_dist* dist, size_t out_offset,
                         const int32_t* out_rows, int out_row_heads, int out_head0, int out_dtype,
                         void* workspace, size_t workspace_bytes, hx_stream_t stream)
{
    if (int rc = validate_decode(c, layer, q, q_dtype, seq_ids, lengths, n_seqs, num_q_heads,
                                 out_dtype))
        return rc;
    if (!dist || !dist->connected) return fail(HX_ERR_INVALID, "gather endpoint is not connected");
    int dev = -1;
    HX_CUDA_TRY(cudaGetDevice(&dev));
    if (dev != dist->device || dev != c->device)
        return fail(HX_ERR_INVALID, "current device %d, endpoint on %d, cache on %d", dev,
                    dist->device, c->device);
    if (n_seqs > 0 && !out_rows) return fail(HX_ERR_INVALID, "null out_rows");
    if (out_head0 < 0 || out_row_heads < num_q_heads || out_head0 + num_q_heads > out_row_heads)
        return fail(HX_ERR_INVALID, "q heads [%d, %d) do not fit an output row of %d heads",
                    out_head0, out_head0 + num_q_heads, out_row_heads);
    if (out_offset % 16) return fail(HX_ERR_INVALID, "out_offset %zu is not 16-byte aligned", out_offset);
    const size_t esize = out_dtype == HX_FP32 ? 4 : 2;
    const size_t row_bytes = (size_t)out_row_heads * c->cfg.head_dim * esize;
    if (out_offset > dist->bytes || (dist->bytes - out_offset) / row_bytes < 1)
        return fail(HX_ERR_CAPACITY, "gather buffer of %zu bytes holds no row at offset %zu",
                    dist->bytes, out_offset);
    const size_t rows = (dist->bytes - out_offset) / row_bytes;
    DecodeParams p = base_params(c, layer, q, q_dtype, seq_ids, lengths, n_seqs, num_q_heads,
                                 scale, out_dtype);
    p.n_outs = 0;
    for (int r = 0; r < dist->world; ++r) {
        // own buffer first: it is the destination the single-destination paths use
        const int rr = (dist->rank + r) % dist->world;
        p.outs[p.n_outs++] = dist->peer_buf[rr] + out_offset;
    }
    p.out = p.outs[0];
    p.out_vec = 1;  // buffers from cudaMalloc, offset a multiple of 16
    p.out_rows = out_rows;
    p.out_hq = out_row_heads;
    p.out_head0 = out_head0;
    p.out_row_limit = rows > (size_t)INT32_MAX ? INT32_MAX : (int)rows;
    p.status = status_word();
    cudaStream_t s = (cudaStream_t)stream;
    if (a)
        if (int rc = append_params(c, a, p)) return rc;
    if (n_seqs == 0) return HX_OK;
    const size_t need = needed_scratch(c, p);
    if (need && (!workspace || workspace_bytes < need))
        return fail(HX_ERR_INVALID, "workspace of %zu bytes is smaller than the %zu needed",
                    workspace_bytes, need);
    return run_decode(c, p, workspace, s);
}

}  // namespace hx

extern "C" int hx_decode_attention_gather(const hx_kv_cache* c, int layer, const void* q,
                                          int q_dtype, const int32_t* seq_ids,
                                          const int32_t* lengths, int n_seqs, int num_q_heads,
                                          float scale, hx_dist* dist, size_t out_offset,
                                          const int32_t* out_rows, int out_row_heads,
                                          int out_head0, int out_dtype, void* workspace,
                                          size_t workspace_bytes, hx_stream_t stream)
{
    HX_NVTX_RANGE("hx_decode_attention_gather");
    return decode_gather(c, layer, q, q_dtype, nullptr, seq_ids, lengths, n_seqs, num_q_heads,
                         scale, dist, out_offset, out_rows, out_row_heads, out_head0, out_dtype,
                         workspace, workspace_bytes, stream);
}

extern "C" int hx_append_decode_attention(hx_kv_cache* c, int layer, const void* q,
                                          const hx_append_spec* append, const int32_t* seq_ids,
                                          const int32_t* lengths, int n_seqs, int num_q_heads,
                                          float scale, void* out, int out_dtype, void* workspace,
                                          size_t workspace_bytes, hx_stream_t stream)
{
    HX_NVTX_RANGE("hx_append_decode_attention");
    const int q_dtype = append ? append->dtype : HX_FP16;
    if (int rc = validate_decode(c, layer, q, q_dtype, seq_ids, lengths, n_seqs, num_q_heads,
                                 out_dtype))
        return rc;
    if (n_seqs > 0 && !out) return fail(HX_ERR_INVALID, "null out");
    DecodeParams p = base_params(c, layer, q, q_dtype, seq_ids, lengths, n_seqs, num_q_heads,
                                 scale, out_dtype);
    if (int rc = append_params(c, append, p)) return rc;
    if (n_seqs == 0) return HX_OK;
    p.out = out;
    p.outs[0] = out;
    p.n_outs = 1;
    p.out_vec = reinterpret_cast<uintptr_t>(out) % 16 == 0;
    p.status = status_word();
    const size_t need = needed_scratch(c, p);
    if (need && (!workspace || workspace_bytes < need))
        return fail(HX_ERR_INVALID, "workspace of %zu bytes is smaller than the %zu needed",
                    workspace_bytes, need);
    return run_decode(c, p, workspace, (cudaStream_t)stream);
}

extern "C" int hx_append_decode_attention_gather(
    hx_kv_cache* c, int layer, const void* q, const hx_append_spec* append, const int32_t* seq_ids,
    const int32_t* lengths, int n_seqs, int num_q_heads, float scale, hx_dist* dist,
    size_t out_offset, const int32_t* out_rows, int out_row_heads, int out_head0, int out_dtype,
    void* workspace, size_t workspace_bytes, hx_stream_t stream)
{
    HX_NVTX_RANGE("hx_append_decode_attention_gather");
    if (!append) return fail(HX_ERR_INVALID, "null append spec");
    return decode_gather(c, layer, q, append->dtype, append, seq_ids, lengths, n_seqs, num_q_heads,
                         scale, dist, out_offset, out_rows, out_row_heads, out_head0, out_dtype,
                         workspace, workspace_bytes, stream);
}

// ---------------------------------------------------------------- no-allocation variant
//
// For callers that cannot allocate device memory: code running inside a
// custom allocator or an out-of-memory handler, host environments that own
// the whole memory budget up front, or plug-in hosts that forbid cudaMalloc
// after start-up.  Their split-K scratch comes from a fixed array compiled
// into this library instead of a caller-supplied workspace.
//
// kNoAllocScratchBytes (4 MiB) is a hard limit: a call whose workspace would
// exceed it (see hx_decode_workspace_bytes) is rejected.  Every GPU that
// loads the library keeps this array until the process exits.
//
// In host code `g_decode_scratch` is only a host-side stand-in for the device
// array, not a device address.  Its device address is looked up with
// cudaGetSymbolAddress once per device by decode_prepare_device, which
// hx_kv_create and hx_kv_wrap run on the cache's device (where allocating is
// allowed); that set-up also sets the decode kernels' attributes, loads
// their module and allocates the device status word, so the entry point
// itself makes none of these calls.
//
// All calls share the array and it keeps the last call's contents.  Its
// first 64 KiB are the per-segment counters of the folded combine: zero when
// the module is loaded, and every call returns them to zero.  Every other
// word a call reads is written earlier in the same call, so nothing needs
// clearing; but two calls that overlap on the GPU (different streams,
// devices aside) race on the scratch.
namespace hx {
constexpr size_t kNoAllocScratchBytes = 4u << 20;
static __device__ __align__(256) unsigned char g_decode_scratch[kNoAllocScratchBytes];

int decode_prepare_device(hx_kv_cache* c)
{
    static std::mutex mu;
    static void* scratch[64] = {nullptr};
    int dev = 0;
    HX_CUDA_TRY(cudaGetDevice(&dev));
    if (dev != c->device) return fail(HX_ERR_INVALID, "cache set-up on device %d, current %d", c->device, dev);
    if (int rc = ensure_decode_attrs<8, 6, 1>()) return rc;
    if (int rc = ensure_decode_attrs<8, 3, 2>()) return rc;
    if (int rc = ensure_decode_attrs<16, 6, 1>()) return rc;
    cudaFuncAttributes fa;
    HX_CUDA_TRY(cudaFuncGetAttributes(&fa, decode_combine_kernel<12>));
    HX_CUDA_TRY(cudaFuncGetAttributes(&fa, decode_combine_kernel<8>));
    HX_CUDA_TRY(cudaFuncGetAttributes(&fa, decode_generic_kernel));
    c->status = status_word();
    if (!c->status) return fail(HX_ERR_CUDA, "device status word allocation failed");
    std::lock_guard<std::mutex> lk(mu);
    void* ptr = dev >= 0 && dev < 64 ? scratch[dev] : nullptr;
    if (!ptr) {
        HX_CUDA_TRY(cudaGetSymbolAddress(&ptr, g_decode_scratch));
        if (dev >= 0 && dev < 64) scratch[dev] = ptr;
    }
    c->noalloc_scratch = ptr;
    return HX_OK;
}
}  // namespace hx

extern "C" int hx_decode_attention_noalloc(const hx_kv_cache* c, int layer, const void* q,
                                           int q_dtype, const int32_t* seq_ids,
                                           const int32_t* lengths, int n_seqs, int num_q_heads,
                                           float scale, void* out, int out_dtype,
                                           hx_stream_t stream)
{
    HX_NVTX_RANGE("hx_decode_attention_noalloc");
    if (int rc = validate_decode(c, layer, q, q_dtype, seq_ids, lengths, n_seqs, num_q_heads,
                                 out_dtype))
        return rc;
    if (n_seqs > 0 && !out) return fail(HX_ERR_INVALID, "null out");
    if (n_seqs == 0) return HX_OK;
    DecodeParams p = base_params(c, layer, q, q_dtype, seq_ids, lengths, n_seqs, num_q_heads,
                                 scale, out_dtype);
    p.out = out;
    p.outs[0] = out;
    p.n_outs = 1;
    p.out_vec = reinterpret_cast<uintptr_t>(out) % 16 == 0;
    p.status = c->status;  // allocated when the cache was created
    const size_t need = needed_scratch(c, p);
    if (need > kNoAllocScratchBytes)
        return fail(HX_ERR_CAPACITY,
                    "this call needs %zu bytes of split-K scratch; the no-allocation entry point "
                    "holds at most %zu (use hx_decode_attention with a caller workspace)",
                    need, kNoAllocScratchBytes);
    if (need && !c->noalloc_scratch)
        return fail(HX_ERR_CUDA, "the decode scratch of this device was not set up");
    return run_decode(c, p, c->noalloc_scratch, (cudaStream_t)stream);
}
