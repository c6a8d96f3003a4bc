// Status mapping shared by every C-ABI translation unit.
#pragma once
#include "common.hpp"
#include "tsac_cuda.h"

#include <cstdlib>
#include <cstring>
#include <string>

namespace tsacb
{
extern thread_local std::string last_error_message;

// CUDA runtime failure (or no device): mapped to TSAC_CUDA_ERROR_DEVICE.
struct DeviceError : Error
{
    using Error::Error;
};

// Device error word reported a nonfinite value: TSAC_CUDA_ERROR_NUMERIC.
struct NumericError : Error
{
    using Error::Error;
};

template <class F> int guarded(F&& f)
{
    try
    {
        f();
        last_error_message.clear();
        return TSAC_CUDA_OK;
    }
    catch (const DeviceError& e)
    {
        last_error_message = e.what();
        return TSAC_CUDA_ERROR_DEVICE;
    }
    catch (const NumericError& e)
    {
        last_error_message = e.what();
        return TSAC_CUDA_ERROR_NUMERIC;
    }
    catch (const std::exception& e)
    {
        last_error_message = e.what();
        return TSAC_CUDA_ERROR;
    }
}

template <class T> T* malloc_copy(const T* data, std::size_t count)
{
    auto* p = static_cast<T*>(std::malloc(count * sizeof(T) + 1));
    if (!p)
    {
        throw Error("out of host memory");
    }
    if (count)
    {
        std::memcpy(p, data, count * sizeof(T));
    }
    return p;
}
} // namespace tsacb
