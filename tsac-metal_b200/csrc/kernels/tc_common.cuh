// tcgen05 / TMA building blocks shared by this library's tensor-core kernels
// (tc_conv.cu: 3xTF32 convolution; qlinear_tc.cu: int8 GEMM): mbarriers with
// bounded waits, 2D/3D TMA loads, the K-major 128-byte-swizzle shared-memory
// descriptor, tcgen05 commit / fences / TMEM loads, and the host lookup of
// cuTensorMapEncodeTiled.
//
// Every wait is bounded (about one second of global time) and returns false
// when it gives up or when another role raised the kernel's abort flag, so a
// kernel can record the failure and leave instead of hanging the GPU.
#pragma once
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <mutex>

namespace tsacb::dev::tc
{
constexpr unsigned long long WAIT_NS = 1000000000ull;

__device__ __forceinline__ uint32_t smem_u32(const void* p)
{
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ unsigned long long global_ns()
{
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void bar_init(uint32_t bar, uint32_t count)
{
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count));
}

__device__ __forceinline__ bool bar_try(uint32_t bar, uint32_t parity)
{
    uint32_t ok;
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
                 "selp.u32 %0, 1, 0, p;\n\t}"
                 : "=r"(ok)
                 : "r"(bar), "r"(parity)
                 : "memory");
    return ok != 0;
}

// Bounded wait for the phase of `parity` to complete.  Returns false after
// about WAIT_NS of global time, or early when another role has aborted.
__device__ __forceinline__ bool bar_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag)
{
    if (bar_try(bar, parity))
        return true;
    const unsigned long long start = global_ns();
    for (unsigned iter = 1;; ++iter)
    {
        if (bar_try(bar, parity))
            return true;
        if ((iter & 63u) == 0)
        {
            if (*abort_flag)
                return false;
            if (global_ns() - start > WAIT_NS)
                return false;
        }
    }
}

__device__ __forceinline__ void bar_expect_tx(uint32_t bar, uint32_t bytes)
{
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void bar_arrive(uint32_t bar)
{
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void tma_2d(uint32_t dst, const CUtensorMap* map, int c0, int c1,
                                       uint32_t bar)
{
    asm volatile("cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
                 " [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
                 "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(bar)
                 : "memory");
}

__device__ __forceinline__ void tma_3d(uint32_t dst, const CUtensorMap* map, int c0, int c1, int c2,
                                       uint32_t bar)
{
    asm volatile("cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
                 " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(dst),
                 "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(bar)
                 : "memory");
}

// Shared-memory matrix descriptor: K-major operand, 128-byte swizzle, rows of
// 128 bytes in 8-row (1024-byte) atoms stacked along M/N.  The swizzle follows
// the shared-memory address bits, as the TMA writes it, so an operand may start
// at any 128-byte row of a 1024-byte-aligned tile or window (base offset 0;
// measured: setting the descriptor's base-offset field to the row phase gave
// wrong products).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr)
{
    uint64_t d = static_cast<uint64_t>((saddr & 0x3ffffu) >> 4);
    d |= static_cast<uint64_t>(1) << 16;           // leading byte offset (unused here)
    d |= static_cast<uint64_t>(1024 >> 4) << 32;   // stride byte offset: 8 rows x 128 B
    d |= static_cast<uint64_t>(1) << 46;           // descriptor version
    d |= static_cast<uint64_t>(2) << 61;           // 128-byte swizzle
    return d;
}

__device__ __forceinline__ void mma_commit(uint32_t bar)
{
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     bar)
                 : "memory");
}

__device__ __forceinline__ void tc_fence_before()
{
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after()
{
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// 16 consecutive TMEM columns of this thread's lane; the values are valid
// after tmem_wait_loads().
__device__ __forceinline__ void tmem_load16(uint32_t taddr, uint32_t (&r)[16])
{
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x16.b32"
                 " {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),
                   "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]),
                   "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
                 : "r"(taddr));
}

__device__ __forceinline__ void tmem_wait_loads()
{
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// ------------------------------------------------------------ host side --
inline PFN_cuTensorMapEncodeTiled_v12000 encode_fn()
{
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once,
                   []
                   {
                       void* p = nullptr;
                       cudaDriverEntryPointQueryResult q{};
                       if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000,
                                                            cudaEnableDefault, &q) == cudaSuccess &&
                           q == cudaDriverEntryPointSuccess)
                           fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
                   });
    return fn;
}

inline int sm_count()
{
    int device = 0, count = 148;
    if (cudaGetDevice(&device) == cudaSuccess)
        cudaDeviceGetAttribute(&count, cudaDevAttrMultiProcessorCount, device);
    return count;
}
} // namespace tsacb::dev::tc
