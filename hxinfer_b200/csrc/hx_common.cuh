// hx_common.cuh — device helpers shared by the sm_100a kernels of libhxkv.
//
// Inline-PTX wrappers for mbarriers (every wait is bounded by a wall-clock
// deadline, after which the caller records HX_ERR_TIMEOUT and unwinds),
// TMA tile loads (no multicast), ldmatrix, mma.sync and ex2.approx.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <utility>

#include "hx_internal.h"

namespace hx {

// A bounded wait gives up after this many nanoseconds of %globaltimer.
constexpr uint64_t kWaitTimeoutNs = 4ull * 1000 * 1000 * 1000;

__device__ __forceinline__ uint32_t smem_u32(const void* p)
{
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer_ns()
{
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Records the first failure of any kernel in the device status word.
__device__ __forceinline__ void record_status(int* status, int code)
{
    if (status) atomicCAS(status, 0, code);
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count)
{
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
                 : "memory");
}

__device__ __forceinline__ void fence_mbar_init()
{
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes)
{
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar)
{
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity)
{
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Waits for the phase with the given parity to complete.  Returns false if
// the deadline passed first (the caller must then stop using the barrier).
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity)
{
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    while (true) {
#pragma unroll 1
        for (int i = 0; i < 128; ++i)
            if (mbar_try_wait(bar, parity)) return true;
        if (globaltimer_ns() - t0 > kWaitTimeoutNs) return false;
    }
}

// GPU-scope acquire-release fence: after a CTA barrier, orders the CTA's
// earlier global writes before this thread's next atomic (release side), or
// an atomic's result before the CTA's later reads (acquire side).
__device__ __forceinline__ void fence_acq_rel_gpu()
{
    asm volatile("fence.acq_rel.gpu;" ::: "memory");
}

// Orders this thread's generic-proxy shared-memory writes before later
// async-proxy (TMA) accesses to the same bytes.
__device__ __forceinline__ void fence_proxy_async_smem()
{
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Orders this thread's earlier generic-proxy global writes before later
// async-proxy (TMA) reads of the same memory.
__device__ __forceinline__ void fence_proxy_async_global()
{
    asm volatile("fence.proxy.async.global;" ::: "memory");
}

__device__ __forceinline__ uint64_t l2_evict_first_policy()
{
    uint64_t policy;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(policy));
    return policy;
}

__device__ __forceinline__ uint64_t l2_evict_last_policy()
{
    uint64_t policy;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(policy));
    return policy;
}

// 2-D TMA tile load global -> shared, completing on `bar` (no multicast).
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* tm, int x, int y,
                                            uint64_t* bar, uint64_t policy)
{
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_u32(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(tm)), "r"(x), "r"(y), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap* tm)
{
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(tm)) : "memory");
}

__device__ __forceinline__ void ldmatrix_x4(uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3,
                                            uint32_t addr)
{
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}

__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                                  uint32_t& r3, uint32_t addr)
{
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}

// Transposes an 8x8 matrix of 16-bit values held one 32-bit pair per lane
// (lane 4r + c holds row r, columns 2c and 2c+1).
__device__ __forceinline__ uint32_t movmatrix_trans(uint32_t x)
{
    uint32_t y;
    asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
    return y;
}

// D = A(16x16 fp16, row) * B(16x8 fp16, col) + D (fp32)
__device__ __forceinline__ void mma_16816(float* d, const uint32_t* a, uint32_t b0, uint32_t b1)
{
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
        "{%8, %9}, {%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// 2^x by the hardware ex2.approx instruction (flush-to-zero).
__device__ __forceinline__ float fast_exp2(float x)
{
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// ---- K1 numerics (rope_append.cu and the append-and-decode path) ----
// The bias add rounds like the reference (fp16 __hadd, bias_add.cu:6-11, or
// an fp32 add); the NeoX rotation of a pair (x1, x2) = (x[d], x[d + hd/2])
// evaluates x1*c - x2*s and x2*c + x1*s with separately rounded multiplies
// and adds, the order of rope_cpu.cpp:29-30 without FMA contraction.
template <typename T>
__device__ __forceinline__ float ld(const T* p)
{
    return (float)*p;
}
template <>
__device__ __forceinline__ float ld<__half>(const __half* p)
{
    return __half2float(*p);
}

// x + b with the reference's rounding: fp16 __hadd (bias_add.cu:6-11) or fp32 add.
template <typename T>
__device__ __forceinline__ float ld_bias(const T* x, const T* b)
{
    return b ? __fadd_rn(*x, *b) : (float)*x;
}
template <>
__device__ __forceinline__ float ld_bias<__half>(const __half* x, const __half* b)
{
    return b ? __half2float(__hadd(*x, *b)) : __half2float(*x);
}

template <typename T>
__device__ __forceinline__ void st(T* p, float v)
{
    *p = v;
}
template <>
__device__ __forceinline__ void st<__half>(__half* p, float v)
{
    *p = __float2half_rn(v);
}

__device__ __forceinline__ void rotate(float x1, float x2, float2 cs, float& o1, float& o2)
{
    o1 = __fsub_rn(__fmul_rn(x1, cs.x), __fmul_rn(x2, cs.y));
    o2 = __fadd_rn(__fmul_rn(x2, cs.x), __fmul_rn(x1, cs.y));
}

__device__ __forceinline__ uint32_t pack_half2(float lo, float hi)
{
    __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
}

// Programmatic dependent launch: let the next kernel on the stream start /
// wait until the previous kernel on the stream has finished (both are no-ops
// for a kernel launched without the programmatic attribute).
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Launches `kernel`, as a programmatic dependent of the previous kernel on
// the stream when `overlap` is set.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_kernel(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                                 cudaStream_t stream, bool overlap, Args&&... args)
{
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = overlap ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// Physical block of logical block `blk` of sequence `seq`, or -1 when the
// block is unmapped or (seq, blk) lies outside the block table.
__device__ __forceinline__ int64_t phys_block(const KVView& v, int seq, int blk)
{
    if (seq < 0 || seq >= v.max_seqs || blk < 0 || blk >= v.mbps) return -1;
    if (v.table) return v.table[(int64_t)seq * v.mbps + blk];
    return (int64_t)seq * v.mbps + blk;
}

// Byte offset of position `pos` of kv head `h` in sequence `seq`, or -1 if
// the block is unmapped.
__device__ __forceinline__ int64_t token_offset(const KVView& v, int seq, int h, int pos)
{
    int64_t pb = phys_block(v, seq, pos / kBlockTokens);
    if (pb < 0) return -1;
    return pb * v.block_stride + (int64_t)h * v.head_stride +
           (int64_t)(pos % kBlockTokens) * v.hd * 2;
}

}  // namespace hx
