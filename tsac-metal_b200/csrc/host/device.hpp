// Device memory plumbing for the host orchestration: RAII buffers and a
// grow-only named workspace (device scratch is reused across calls).
#pragma once
#include "abi_util.hpp"

#include <cuda_runtime.h>
#include <map>
#include <string>
#include <vector>

namespace tsacb
{
inline void cuda_ok(cudaError_t status, const char* what)
{
    if (status != cudaSuccess)
    {
        throw DeviceError(std::string(what) + ": " + cudaGetErrorString(status));
    }
}

class DeviceBuffer
{
public:
    DeviceBuffer() = default;
    explicit DeviceBuffer(std::size_t bytes)
    {
        resize(bytes);
    }
    ~DeviceBuffer()
    {
        if (ptr_)
        {
            cudaFree(ptr_);
        }
    }
    DeviceBuffer(const DeviceBuffer&) = delete;
    DeviceBuffer& operator=(const DeviceBuffer&) = delete;
    DeviceBuffer(DeviceBuffer&& o) noexcept : ptr_(o.ptr_), bytes_(o.bytes_)
    {
        o.ptr_ = nullptr;
        o.bytes_ = 0;
    }
    DeviceBuffer& operator=(DeviceBuffer&& o) noexcept
    {
        std::swap(ptr_, o.ptr_);
        std::swap(bytes_, o.bytes_);
        return *this;
    }
    void resize(std::size_t bytes)
    {
        if (bytes <= bytes_)
        {
            return;
        }
        if (ptr_)
        {
            cudaFree(ptr_);
            ptr_ = nullptr;
            bytes_ = 0;
        }
        cuda_ok(cudaMalloc(&ptr_, bytes ? bytes : 1), "cudaMalloc");
        bytes_ = bytes;
    }
    template <class T> T* as() const
    {
        return static_cast<T*>(ptr_);
    }
    std::size_t bytes() const
    {
        return bytes_;
    }

private:
    void* ptr_ = nullptr;
    std::size_t bytes_ = 0;
};

template <class T> DeviceBuffer upload(const std::vector<T>& host, cudaStream_t stream)
{
    DeviceBuffer b(host.size() * sizeof(T));
    if (!host.empty())
    {
        cuda_ok(cudaMemcpyAsync(b.as<void>(), host.data(), host.size() * sizeof(T),
                                cudaMemcpyHostToDevice, stream),
                "upload");
    }
    return b;
}

// Named scratch buffers that only grow; valid until the next get() of the same name.
class Workspace
{
public:
    template <class T> T* get(const std::string& name, std::size_t count)
    {
        auto& b = buffers_[name];
        b.resize(count * sizeof(T) + 256);
        return b.as<T>();
    }

private:
    std::map<std::string, DeviceBuffer> buffers_;
};
} // namespace tsacb
