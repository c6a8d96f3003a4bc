// Asynchronous global -> shared copies (cp.async), for kernels that stage
// operands without holding them in registers: the copies of a thread are all
// in flight at once, and cp_async_wait_all() waits for that thread's copies
// (a barrier afterwards makes them visible to the other threads).
#pragma once
#include <cuda_runtime.h>

namespace tsacb::dev
{
// 4-byte copy; both addresses 4-byte aligned.
__device__ __forceinline__ void cp_async_4(void* smem, const void* gmem)
{
    const unsigned address = static_cast<unsigned>(__cvta_generic_to_shared(smem));
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(address), "l"(gmem) : "memory");
}

__device__ __forceinline__ void cp_async_wait_all()
{
    asm volatile("cp.async.wait_all;" ::: "memory");
}
} // namespace tsacb::dev
