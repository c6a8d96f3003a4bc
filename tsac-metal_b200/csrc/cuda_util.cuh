// CUDA runtime error mapping for the C ABI.
#pragma once
#include "host/abi_util.hpp"

#include <cuda_runtime.h>
#include <string>

namespace tsacb
{
inline void cuda_check(cudaError_t status, const char* what)
{
    if (status != cudaSuccess)
    {
        throw DeviceError(std::string(what) + ": " + cudaGetErrorString(status));
    }
}

inline void require_device()
{
    int count = 0;
    const auto status = cudaGetDeviceCount(&count);
    if (status != cudaSuccess || count == 0)
    {
        throw DeviceError("no CUDA device available (this library has no CPU fallback)");
    }
}

inline bool aligned16(const void* p)
{
    return (reinterpret_cast<std::uintptr_t>(p) & 15u) == 0;
}
} // namespace tsacb
