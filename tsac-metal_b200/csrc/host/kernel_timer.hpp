// Opt-in per-kernel-family timing with CUDA events (tsac_cuda_kernel_timing).
//
// When enabled, launch sites wrap their kernels in a Scope that records a
// start/end event pair on the launching stream plus the algorithmic work of the
// launch (FLOPs or bytes).  Events are resolved only when statistics are read,
// so timing adds no synchronisation to the timed region.
#pragma once
#include "device.hpp"

#include <mutex>
#include <string>
#include <vector>

namespace tsacb
{
class KernelTimer
{
public:
    static KernelTimer& instance();
    bool enabled() const
    {
        return enabled_;
    }
    void enable(bool on);
    void reset();
    // JSON object {name: {"launches": n, "ms": total, "work": total}}.
    std::string stats();

    class Scope
    {
    public:
        Scope(const char* name, cudaStream_t stream, double work);
        ~Scope();

    private:
        const char* name_;
        cudaStream_t stream_;
        double work_;
        cudaEvent_t start_ = nullptr;
    };

private:
    struct Record
    {
        std::string name;
        cudaEvent_t start, end;
        double work;
    };
    bool enabled_ = false;
    std::mutex mutex_;
    std::vector<Record> records_;
    std::vector<cudaEvent_t> pool_;
    cudaEvent_t take();
    friend class Scope;
};
} // namespace tsacb
