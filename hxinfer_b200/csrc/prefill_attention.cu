// prefill_attention.cu — K3: causal prefill attention on the 5th-generation
// tensor cores (tcgen05.mma, accumulators in tensor memory).
//
// The reference has no prefill kernel: it runs one token per forward call
// (hxinfer demos/bench_1024.cpp:62-70), i.e. the decode step of
// attention_score_cuda.cu:17-83 once per prompt position.  Here one launch
// computes, for query rows i in [0, n) at positions start + i,
//     out[i] = softmax(q_i . K[0 .. start+i]^T * scale) V
// over the paged cache (the rows' own K/V must already be appended).
//
// One CTA per (128-row query tile, q head); 320 threads:
//   warp 8  TMA producers: lane 0 the Q tile once (2 boxes 128x64, 128-byte
//           swizzle) then a 3-stage ring of 128-position K tiles (two cache
//           blocks each); lane 1 a 3-stage ring of V tiles; block-table rows
//           are read one tile ahead; no multicast.
//   warp 9  TMEM allocator (512 columns) and, lane 0, the MMA issuer:
//           S_j = Q K_j^T  (M=128, N=128, K=16 x 8, fp16 -> fp32) into TMEM
//           buffer j & 1, then for each key half w: O_w += P_j[:, w] V_j[w]
//           (K = 16 x 4, P read from the S buffer, V as an MN-major
//           operand, O_0 and O_1 in columns 256 and 384); order S_0, S_1,
//           then PV_j (both halves), S_{j+2} for each j, so S_{j+1} runs
//           during softmax j and S_{j+2} overwrites P_j only after PV_j (this
//           thread's MMAs execute in order); completion via tcgen05.commit.
//   warps 0-7  softmax in two warpgroups: warpgroup w takes key columns
//           64 w .. 64 w + 63 of every tile, thread t (mod 128) query row t;
//           reads its S columns with tcgen05.ld, applies the causal mask,
//           keeps its own running max (moved only when it rises by more than
//           2^8, then O_w is rescaled) and sum, and writes its P half as fp16
//           over its own S columns with tcgen05.st.  The halves never wait
//           for each other; the epilogue combines
//           O = (a_0 O_0 + a_1 O_1) / (a_0 l_0 + a_1 l_1), staged through an
//           idle K stage for coalesced stores.
// Key tiles above the diagonal are never loaded.  Every mbarrier wait is
// bounded; TMEM is always released before exit.
#include "hx_common.cuh"

namespace hx {

constexpr int kPfSoftmaxWarps = 8;             // two warpgroups: key halves of every tile
constexpr int kPfProducerWarp = kPfSoftmaxWarps;  // TMA
constexpr int kPfMmaWarp = kPfSoftmaxWarps + 1;   // TMEM allocation and the MMA issuer
constexpr int kPfThreads = 32 * (kPfSoftmaxWarps + 2);
constexpr int kRegionBytes = 128 * 128;  // 128 rows x 64 fp16 (one 128-byte swizzled region)
constexpr int kPfKStages = 3, kPfVStages = 3;  // K and V tile rings

struct PrefillParams {
    KVView view;
    int seq, start, n, hq, group, n_qtiles;
    float scale_log2;
    void* out;
    int out_f32;
    int* status;
};

struct PrefillSmem {
    uint8_t q[2][kRegionBytes];                // [d half]
    uint8_t k[kPfKStages][2][kRegionBytes];    // [stage][d half]
    uint8_t v[kPfVStages][2][kRegionBytes];    // [stage][d half]
    uint64_t q_full;
    uint64_t k_full[kPfKStages], k_empty[kPfKStages];
    uint64_t v_full[kPfVStages], v_empty[kPfVStages];
    uint64_t s_full[2];                        // per TMEM S/P buffer
    uint64_t p_full[2][2], pv_done[2][2];      // [key half][TMEM S/P buffer]
    uint64_t mma_idle;
    uint32_t tmem_base;
    int abort_flag;
};

// ------------------------------------------------------------ tcgen05 helpers

// Shared-memory matrix descriptor: start, leading / stride byte offsets,
// version 1, 128-byte swizzle.
__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo)
{
    return (uint64_t)((saddr >> 4) & 0x3FFF) | ((uint64_t)((lbo >> 4) & 0x3FFF) << 16) |
           ((uint64_t)((sbo >> 4) & 0x3FFF) << 32) | (1ull << 46) | (2ull << 61);
}

// Instruction descriptor, kind::f16: fp32 accumulate, fp16 A and B,
// M = 128, N = 128; b_mn selects an MN-major B operand.
__device__ __forceinline__ uint32_t umma_idesc(bool b_mn)
{
    return (1u << 4) | ((b_mn ? 1u : 0u) << 16) | ((128u >> 3) << 17) | ((128u >> 4) << 24);
}

__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                         uint32_t idesc, uint32_t accumulate)
{
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// The same MMA with the A operand (M = 128 rows x K = 16 fp16) read from
// tensor memory: row i in lane i, two K elements per 32-bit column.
__device__ __forceinline__ void umma_f16_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc,
                                            uint32_t idesc, uint32_t accumulate)
{
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem_d),
        "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ void umma_commit(uint64_t* bar)
{
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// 32 consecutive fp32 columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float* v)
{
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, "
        "%12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, "
        "%30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
          "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
          "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
          "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float* v)
{
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
        "%11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, "
        "%29, %30, %31, %32};" ::"r"(taddr),
        "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
        "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
        "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
        "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
        "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
        "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])),
        "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])), "r"(__float_as_uint(v[20])),
        "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
        "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])),
        "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])),
        "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
        : "memory");
}

__device__ __forceinline__ void tmem_st32u(uint32_t taddr, const uint32_t* v)
{
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
        "%11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, "
        "%29, %30, %31, %32};" ::"r"(taddr),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
        "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]),
        "r"(v[15]), "r"(v[16]), "r"(v[17]), "r"(v[18]), "r"(v[19]), "r"(v[20]), "r"(v[21]),
        "r"(v[22]), "r"(v[23]), "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]), "r"(v[28]),
        "r"(v[29]), "r"(v[30]), "r"(v[31])
        : "memory");
}

__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// A bounded wait that also gives up when another role has aborted.
__device__ __forceinline__ bool pf_wait(PrefillSmem& sm, uint64_t* bar, uint32_t parity, int* status)
{
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    while (true) {
#pragma unroll 1
        for (int i = 0; i < 64; ++i)
            if (mbar_try_wait(bar, parity)) return true;
        if (*reinterpret_cast<volatile int*>(&sm.abort_flag)) return false;
        if (globaltimer_ns() - t0 > kWaitTimeoutNs) {
            record_status(status, HX_ERR_TIMEOUT);
            atomicExch(&sm.abort_flag, 1);
            return false;
        }
    }
}

__global__ void __launch_bounds__(kPfThreads, 1)
    prefill_attention_kernel(const __grid_constant__ CUtensorMap tm_q,
                             const __grid_constant__ CUtensorMap tm_k,
                             const __grid_constant__ CUtensorMap tm_v, const PrefillParams p)
{
    extern __shared__ uint8_t smem_raw[];
    auto& sm = *reinterpret_cast<PrefillSmem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~uintptr_t(1023));
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // grid (q heads, query tiles): the last query tiles (most key tiles)
    // of every head are issued first
    const int qt = p.n_qtiles - 1 - (int)blockIdx.y;
    const int h = blockIdx.x, kvh = h / p.group;
    const int q0 = qt * 128;
    const int rows_valid = min(128, p.n - q0);
    const int kend = p.start + q0 + rows_valid;  // keys [0, kend) are needed by this tile
    const int nk = (kend + 127) / 128;

    if (threadIdx.x == 0) {
        mbar_init(&sm.q_full, 1);
        for (int i = 0; i < kPfKStages; ++i) {
            mbar_init(&sm.k_full[i], 1);
            mbar_init(&sm.k_empty[i], 1);
        }
        for (int i = 0; i < kPfVStages; ++i) {
            mbar_init(&sm.v_full[i], 1);
            mbar_init(&sm.v_empty[i], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&sm.s_full[i], 1);
            for (int w = 0; w < 2; ++w) {
                mbar_init(&sm.p_full[w][i], 4);  // the four warps of warpgroup w
                mbar_init(&sm.pv_done[w][i], 1);
            }
        }
        mbar_init(&sm.mma_idle, 1);
        sm.abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == kPfMmaWarp) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(
                         smem_u32(&sm.tmem_base))
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = sm.tmem_base;

    if (warp == kPfProducerWarp) {
        // ------------------------------------------------------------ TMA producers
        // lane 0: Q, then the K ring; lane 1: the V ring (V tiles are needed
        // one softmax later than K tiles, so each ring runs at its own pace)
        if (lane < 2) {
            // Q is read by this CTA only; a head's K/V tiles are read again by
            // every later query tile of the head (and by the other q heads of
            // its group), so they are kept in L2
            const uint64_t pol = l2_evict_last_policy();
            const KVView& v = p.view;
            const bool is_k = lane == 0;
            const int stages = is_k ? kPfKStages : kPfVStages;
            if (is_k) {
                const uint64_t qpol = l2_evict_first_policy();
                mbar_arrive_expect_tx(&sm.q_full, 2 * kRegionBytes);
                tma_load_2d(sm.q[0], &tm_q, h * 128, q0, &sm.q_full, qpol);
                tma_load_2d(sm.q[1], &tm_q, h * 128 + 64, q0, &sm.q_full, qpol);
            }
            int issued = 0;
            // Block-table entries of tile j + 1 are read while tile j's ring
            // slot is awaited, so no table load sits between a freed slot and
            // its copy.  -2 marks a block past the keys this tile needs.
            auto table_pair = [&](int j, int64_t* pb) {
                for (int b = 0; b < 2; ++b) {
                    const int blk = 2 * j + b;
                    pb[b] = blk * kBlockTokens < kend ? phys_block(v, p.seq, blk) : -2;
                }
            };
            int64_t next_pb[2];
            table_pair(0, next_pb);
            for (int j = 0; j < nk; ++j) {
                const int s = j % stages;
                uint64_t* full = is_k ? &sm.k_full[s] : &sm.v_full[s];
                uint64_t* empty = is_k ? &sm.k_empty[s] : &sm.v_empty[s];
                const int64_t pb[2] = {next_pb[0], next_pb[1]};
                if (j + 1 < nk) table_pair(j + 1, next_pb);
                if (j >= stages && !pf_wait(sm, empty, ((j / stages) - 1) & 1, p.status)) break;
                int64_t rows[2];
                uint32_t bytes = 0;
                for (int b = 0; b < 2; ++b) {
                    rows[b] = -1;
                    if (pb[b] == -2) continue;
                    if (pb[b] < 0) {
                        record_status(p.status, HX_ERR_CAPACITY);
                        continue;
                    }
                    rows[b] = (pb[b] * v.block_stride + (int64_t)kvh * v.head_stride) / 256;
                    bytes += 2 * (kRegionBytes / 2);
                }
                mbar_arrive_expect_tx(full, bytes);
                uint8_t(*dst)[kRegionBytes] = is_k ? sm.k[s] : sm.v[s];
                const CUtensorMap* tm = is_k ? &tm_k : &tm_v;
                const int64_t row0 = is_k ? v.k_row0 : v.v_row0;
                for (int b = 0; b < 2; ++b) {
                    if (rows[b] < 0) continue;
                    const int r = (int)(row0 + rows[b]);
                    const int off = b * (kRegionBytes / 2);
                    tma_load_2d(dst[0] + off, tm, 0, r, full, pol);
                    tma_load_2d(dst[1] + off, tm, 64, r, full, pol);
                }
                issued = j + 1;
            }
            // Copies still in flight must land before the CTA exits (bounded).
            if (is_k) mbar_wait(&sm.q_full, 0);
            for (int j = issued > stages ? issued - stages : 0; j < issued; ++j)
                mbar_wait(is_k ? &sm.k_full[j % stages] : &sm.v_full[j % stages], (j / stages) & 1);
        }
    } else if (warp == kPfMmaWarp) {
        // ------------------------------------------------------------ MMA issuer
        // Order: S_0, S_1, then for each j: PV_j (two halves), S_{j+2}.  S_j
        // lands in TMEM buffer j & 1 (columns 128 (j & 1) ..); each softmax
        // warpgroup writes its half of P_j (keys 64 w .. 64 w + 63) over the
        // first 32 of its own 64 S columns, and the PV half
        // w = P_j[:, half w] V_j[half w]
        // accumulates into O_w (columns 256 + 128 w), so the two warpgroups
        // never wait for each other; S_{j+2} (same buffer) is issued after
        // both PV halves of j, and this thread's MMAs execute in order.
        // The shared-memory descriptors are built once: an operand's start
        // address sits in the low 14 bits as address / 16, and every address
        // here is below 256 KB, so moving to another K slice, region or ring
        // stage adds a constant (bytes / 16) without a carry out of the
        // field.  Each MMA then costs this thread one add, not a rebuild
        // (this warp shares its issue slots with two softmax warps).
        if (lane == 0) {
            const uint32_t id_qk = umma_idesc(false), id_pv = umma_idesc(true);
            const uint64_t q_desc = umma_desc(smem_u32(sm.q[0]), 16, 1024);
            const uint64_t k_desc = umma_desc(smem_u32(sm.k[0][0]), 16, 1024);
            const uint64_t v_desc = umma_desc(smem_u32(sm.v[0][0]), kRegionBytes, 1024);
            constexpr uint64_t kStageStep = (2 * kRegionBytes) >> 4;  // one ring stage
            bool ok = pf_wait(sm, &sm.q_full, 0, p.status);
            auto issue_s = [&](int j) {
                const int ks = j % kPfKStages;
                if (!pf_wait(sm, &sm.k_full[ks], (j / kPfKStages) & 1, p.status)) return false;
                tc_fence_after();
                const uint64_t kd = k_desc + (uint64_t)ks * kStageStep;
#pragma unroll
                for (int kk = 0; kk < 8; ++kk) {
                    // K slice kk: region kk / 4, 32 bytes (16 fp16) apart within it
                    const uint64_t off = (uint64_t)(((kk >> 2) * kRegionBytes + (kk & 3) * 32) >> 4);
                    umma_f16(tmem + 128 * (j & 1), q_desc + off, kd + off, id_qk, kk > 0);
                }
                umma_commit(&sm.s_full[j & 1]);
                umma_commit(&sm.k_empty[ks]);
                return true;
            };
            if (ok && nk > 0) ok = issue_s(0);
            if (ok && nk > 1) ok = issue_s(1);
            for (int j = 0; ok && j < nk; ++j) {
                const int vs = j % kPfVStages;
                if (!pf_wait(sm, &sm.v_full[vs], (j / kPfVStages) & 1, p.status)) break;
                for (int w = 0; w < 2 && ok; ++w) {
                    if (!pf_wait(sm, &sm.p_full[w][j & 1], (j >> 1) & 1, p.status)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint64_t vd = v_desc + (uint64_t)vs * kStageStep;
#pragma unroll
                    for (int kk = 4 * w; kk < 4 * w + 4; ++kk) {
                        const uint64_t bd = vd + (uint64_t)((kk * 2048) >> 4);  // 16 keys = 2048 bytes
                        // P half w sits in the first 32 of its own 64 S columns
                        umma_f16_ts(tmem + 256 + 128 * w, tmem + 128 * (j & 1) + 32 * w + 8 * kk, bd,
                                    id_pv, (j > 0 || kk > 4 * w) ? 1u : 0u);
                    }
                    umma_commit(&sm.pv_done[w][j & 1]);
                }
                if (!ok) break;
                umma_commit(&sm.v_empty[vs]);
                if (j + 2 < nk) ok = issue_s(j + 2);
            }
            // Every MMA this thread issued must finish before TMEM is freed.
            umma_commit(&sm.mma_idle);
            if (!mbar_wait(&sm.mma_idle, 0)) record_status(p.status, HX_ERR_TIMEOUT);
        }
    } else {
        // ------------------------------------------------------------ softmax warps
        // Warpgroup w (warps 4w .. 4w + 3) takes key columns 64 w .. 64 w + 63
        // of every tile for the query rows t = threadIdx.x % 128, with its own
        // running max m_w, sum l_w and accumulator O_w; the two halves are
        // combined once, in the epilogue.
        const int t = threadIdx.x & 127;  // query row within the tile
        const int wg = threadIdx.x >> 7;  // key half
        const int row_pos = p.start + q0 + t;
        const uint32_t lane_base = tmem + ((uint32_t)((warp & 3) * 32) << 16);
        const uint32_t o_col = 256 + 128 * wg;
        const float sc = p.scale_log2;
        float m_run = -INFINITY, l = 0.f;  // running max (scaled, log2 domain) and sum of this half
        bool ok = true;
        for (int j = 0; j < nk; ++j) {
            const int b = j & 1;
            // tcgen05.ld/st are warp-collective (.sync.aligned): every branch
            // around them is made warp-uniform, wait outcomes included
            if (!__all_sync(0xffffffffu, pf_wait(sm, &sm.s_full[b], (j >> 1) & 1, p.status))) {
                ok = false;
                break;
            }
            tc_fence_after();
            float sv[64];
            tmem_ld32(lane_base + 128 * b + 64 * wg, sv);
            tmem_ld32(lane_base + 128 * b + 64 * wg + 32, sv + 32);
            tmem_ld_wait();
            const int k0 = 128 * j + 64 * wg;
            const int lim = row_pos - k0;  // keys c <= lim of this half are visible to this row
            if (lim < 63) {
#pragma unroll
                for (int c = 0; c < 64; ++c) sv[c] = c <= lim ? sv[c] : -INFINITY;
            }
            float mx8[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) mx8[e] = sv[e];
#pragma unroll
            for (int c = 8; c < 64; c += 8)
#pragma unroll
                for (int e = 0; e < 8; ++e) mx8[e] = fmaxf(mx8[e], sv[c + e]);
#pragma unroll
            for (int w = 4; w; w >>= 1)
#pragma unroll
                for (int e = 0; e < w; ++e) mx8[e] = fmaxf(mx8[e], mx8[e + w]);
            const float mt = mx8[0] * sc;  // the scale is positive: the max commutes with it
            // Lazy rescale: a row moves its reference max only when the max
            // grew by more than 2^8.  The decision is per row, the O update
            // per warp: when any row of the warp rescales, the whole warp
            // loads and stores its O rows, the others with alpha = 1 (exact).
            const bool grow = mt > m_run + 8.f;
            const float alpha = grow ? fast_exp2(m_run - mt) : 1.f;  // 0 when m_run = -inf
            if (j >= 1 && __any_sync(0xffffffffu, alpha < 1.f)) {
                // O_w must be stable: this half's P_{j-1} V_{j-1} has finished
                if (!__all_sync(0xffffffffu, pf_wait(sm, &sm.pv_done[wg][(j - 1) & 1],
                                                     ((j - 1) >> 1) & 1, p.status))) {
                    ok = false;
                    break;
                }
                tc_fence_after();
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    float ov[32];
                    tmem_ld32(lane_base + o_col + 32 * c, ov);
                    tmem_ld_wait();
#pragma unroll
                    for (int e = 0; e < 32; ++e) ov[e] *= alpha;
                    tmem_st32(lane_base + o_col + 32 * c, ov);
                }
                tmem_st_wait();
            }
            if (grow) {
                l *= alpha;
                m_run = mt;
            }
            // P = 2^(s * scale - m) as fp16 pairs over this half's own S
            // columns (the other warpgroup may still be reading its columns):
            // column 64 w + c of this lane holds keys 64 w + 2c (low half) and
            // 64 w + 2c + 1.  A half with no visible key yet (m_run still
            // -inf) writes zeros.
            const float nm = m_run == -INFINITY ? 0.f : -m_run;
            uint32_t pw[32];
            float l8[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};  // eight partial sums
#pragma unroll
            for (int c = 0; c < 32; ++c) {
                const float p0 = fast_exp2(fmaf(sv[2 * c], sc, nm));
                const float p1 = fast_exp2(fmaf(sv[2 * c + 1], sc, nm));
                l8[c & 7] += p0 + p1;
                pw[c] = pack_half2(p0, p1);
            }
            l += ((l8[0] + l8[1]) + (l8[2] + l8[3])) + ((l8[4] + l8[5]) + (l8[6] + l8[7]));
            tmem_st32u(lane_base + 128 * b + 64 * wg, pw);
            tmem_st_wait();
            if (128 * j + 128 > kend) {
                // V rows (keys) of this half past the last needed key may hold
                // stale bytes: zero them so 0 * garbage cannot reach O_w
                // (two threads per key row, one 128-byte head-dim half each).
                const int vs = j % kPfVStages;
                if (!__all_sync(0xffffffffu, pf_wait(sm, &sm.v_full[vs], (j / kPfVStages) & 1, p.status))) {
                    ok = false;
                    break;
                }
                const int key = 64 * wg + (t & 63), dh = t >> 6;
                if (128 * j + key >= kend) {
#pragma unroll
                    for (int ch = 0; ch < 8; ++ch)
                        *reinterpret_cast<uint4*>(sm.v[vs][dh] + key * 128 + ch * 16) = make_uint4(0, 0, 0, 0);
                }
                fence_proxy_async_smem();
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&sm.p_full[wg][b]);
        }
        // Both halves' last PV must have completed: each warpgroup combines
        // O_0 and O_1 for its half of the head dims.
        const bool have_o = __all_sync(
            0xffffffffu, ok && nk > 0 &&
                             pf_wait(sm, &sm.pv_done[0][(nk - 1) & 1], ((nk - 1) >> 1) & 1, p.status) &&
                             pf_wait(sm, &sm.pv_done[1][(nk - 1) & 1], ((nk - 1) >> 1) & 1, p.status));
        // Epilogue: the K ring is idle once the last PV has completed (every
        // S MMA completed before it).  Each row's (m_w, l_w) go through K
        // stage 2; O = (a_0 O_0 + a_1 O_1) / (a_0 l_0 + a_1 l_1) with
        // a_w = 2^(m_w - max(m_0, m_1)) is staged through stages 0-1 (row t at
        // t * row_bytes, 16-byte chunks permuted chunk ^ (t & mask) to spread
        // banks) so the global stores are coalesced.
        float2* ml = reinterpret_cast<float2*>(&sm.k[2][0][0]);  // [2][128]
        ml[wg * 128 + t] = make_float2(m_run, l);
        asm volatile("bar.sync 1, 256;" ::: "memory");  // the eight softmax warps
        const int row_bytes = p.out_f32 ? 512 : 256;
        const int chunks = row_bytes / 16, cmask = chunks - 1;
        uint8_t* stage = &sm.k[0][0][0];
        if (have_o) {
            tc_fence_after();
            const float2 ml0 = ml[t], ml1 = ml[128 + t];
            const float m = fmaxf(ml0.x, ml1.x);
            const float a0 = ml0.x == -INFINITY ? 0.f : fast_exp2(ml0.x - m);
            const float a1 = ml1.x == -INFINITY ? 0.f : fast_exp2(ml1.x - m);
            const float inv = 1.f / (a0 * ml0.y + a1 * ml1.y);
            const float c0 = a0 * inv, c1 = a1 * inv;
            uint8_t* srow = stage + t * row_bytes;
            float o0[64], o1[64];  // dims 64 wg .. 64 wg + 63 of O_0 and O_1
            tmem_ld32(lane_base + 256 + 64 * wg, o0);
            tmem_ld32(lane_base + 256 + 64 * wg + 32, o0 + 32);
            tmem_ld32(lane_base + 384 + 64 * wg, o1);
            tmem_ld32(lane_base + 384 + 64 * wg + 32, o1 + 32);
            tmem_ld_wait();
            if (p.out_f32) {
#pragma unroll
                for (int e = 0; e < 16; ++e) {
                    const int ch = 16 * wg + e;  // 16-byte chunk of the row
                    *reinterpret_cast<float4*>(srow + 16 * (ch ^ (t & cmask))) =
                        make_float4(o0[4 * e] * c0 + o1[4 * e] * c1, o0[4 * e + 1] * c0 + o1[4 * e + 1] * c1,
                                    o0[4 * e + 2] * c0 + o1[4 * e + 2] * c1, o0[4 * e + 3] * c0 + o1[4 * e + 3] * c1);
                }
            } else {
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    const int ch = 8 * wg + e;
                    float x[8];
#pragma unroll
                    for (int u = 0; u < 8; ++u) x[u] = o0[8 * e + u] * c0 + o1[8 * e + u] * c1;
                    *reinterpret_cast<uint4*>(srow + 16 * (ch ^ (t & cmask))) =
                        make_uint4(pack_half2(x[0], x[1]), pack_half2(x[2], x[3]),
                                   pack_half2(x[4], x[5]), pack_half2(x[6], x[7]));
                }
            }
        }
        asm volatile("bar.sync 1, 256;" ::: "memory");
        if (have_o) {
            uint8_t* out = static_cast<uint8_t*>(p.out);
            for (int u = threadIdx.x; u < rows_valid * chunks; u += 256) {
                const int r = u / chunks, ch = u % chunks;
                const uint4 val = *reinterpret_cast<const uint4*>(stage + r * row_bytes + 16 * (ch ^ (r & cmask)));
                *reinterpret_cast<uint4*>(out + ((int64_t)(q0 + r) * p.hq + h) * row_bytes + 16 * ch) = val;
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == kPfMmaWarp) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem) : "memory");
    }
}

typedef CUresult (*EncodeTiledFnPf)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                    const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                    const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                    CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// Q viewed as [n][hq*128] fp16 with 64x128 boxes, 128-byte swizzle.
static int encode_q_map(CUtensorMap* tm, const void* q, int hq, int n)
{
    static EncodeTiledFnPf fn = nullptr;
    if (!fn) {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult r;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &r) !=
                cudaSuccess ||
            r != cudaDriverEntryPointSuccess)
            return fail(HX_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
        fn = reinterpret_cast<EncodeTiledFnPf>(f);
    }
    cuuint64_t gdim[2] = {(cuuint64_t)hq * 128, (cuuint64_t)n};
    cuuint64_t gstride[1] = {(cuuint64_t)hq * 256};
    cuuint32_t box[2] = {64, 128};
    cuuint32_t es[2] = {1, 1};
    CUresult r = fn(tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(q), gdim, gstride, box,
                    es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(HX_ERR_CUDA, "q tensor map (%d)", (int)r);
    return HX_OK;
}

}  // namespace hx

using namespace hx;

extern "C" int hx_prefill_attention(const hx_kv_cache* c, int layer, const void* q, int seq,
                                    int start, int n, int num_q_heads, float scale, void* out,
                                    int out_dtype, hx_stream_t stream)
{
    HX_NVTX_RANGE("hx_prefill_attention");
    if (!c) return fail(HX_ERR_INVALID, "null cache");
    if (layer < 0 || layer >= c->cfg.num_layers) return fail(HX_ERR_INVALID, "layer %d out of range", layer);
    if (!q || !out) return fail(HX_ERR_INVALID, "null q/out");
    if (seq < 0 || seq >= c->cfg.max_seqs) return fail(HX_ERR_INVALID, "seq %d out of range", seq);
    if (start < 0 || n < 0) return fail(HX_ERR_INVALID, "start/n must be >= 0");
    if ((int64_t)start + n > (int64_t)c->n_mapped[seq] * kBlockTokens ||
        (int64_t)start + n > c->cfg.max_tokens_per_seq)
        return fail(HX_ERR_CAPACITY, "positions [0, %d) not reserved for seq %d", start + n, seq);
    const int hkv = c->cfg.num_kv_heads;
    if (num_q_heads < hkv || num_q_heads % hkv)
        return fail(HX_ERR_INVALID, "num_q_heads %d must be a multiple of kv heads %d", num_q_heads, hkv);
    if (c->cfg.head_dim != 128 || !c->has_tmap)
        return fail(HX_ERR_UNSUPPORTED, "prefill attention needs head_dim 128 (got %d)", c->cfg.head_dim);
    if (out_dtype != HX_FP16 && out_dtype != HX_FP32) return fail(HX_ERR_INVALID, "out dtype");
    if (reinterpret_cast<uintptr_t>(q) & 15 || reinterpret_cast<uintptr_t>(out) & 15)
        return fail(HX_ERR_INVALID, "q/out must be 16-byte aligned");
    if (n == 0) return HX_OK;
    if (int rc = check_device(c->device, "the cache")) return rc;
    CUtensorMap tm_q;
    if (int rc = encode_q_map(&tm_q, q, num_q_heads, n)) return rc;
    PrefillParams p{};
    p.view = make_view(c, layer);
    p.seq = seq;
    p.start = start;
    p.n = n;
    p.hq = num_q_heads;
    p.group = num_q_heads / hkv;
    p.n_qtiles = (n + 127) / 128;
    p.scale_log2 = scale * 1.4426950408889634f;
    p.out = out;
    p.out_f32 = out_dtype == HX_FP32;
    p.status = status_word();
    const size_t smem = sizeof(PrefillSmem) + 1024;
    static std::atomic<bool> attr_set[64];  // per device; set again on ordinals past 63
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64 || !attr_set[dev].load(std::memory_order_acquire)) {
        HX_CUDA_TRY(cudaFuncSetAttribute(prefill_attention_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        if (dev >= 0 && dev < 64) attr_set[dev].store(true, std::memory_order_release);
    }
    dim3 grid(num_q_heads, p.n_qtiles);
    prefill_attention_kernel<<<grid, kPfThreads, smem, (cudaStream_t)stream>>>(tm_q, c->tm_k, c->tm_v, p);
    return check_launch("prefill_attention_kernel");
}
