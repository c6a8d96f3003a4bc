#include "kernel_timer.hpp"

#include "abi_util.hpp"
#include "kernels/launch_count.hpp"

#include <atomic>
#include <map>
#include <sstream>

namespace tsacb
{
KernelTimer& KernelTimer::instance()
{
    static KernelTimer timer;
    return timer;
}

void KernelTimer::enable(bool on)
{
    std::lock_guard lock(mutex_);
    enabled_ = on;
}

cudaEvent_t KernelTimer::take()
{
    if (!pool_.empty())
    {
        auto e = pool_.back();
        pool_.pop_back();
        return e;
    }
    cudaEvent_t e = nullptr;
    cuda_ok(cudaEventCreate(&e), "cudaEventCreate");
    return e;
}

void KernelTimer::reset()
{
    std::lock_guard lock(mutex_);
    for (auto& r : records_)
    {
        pool_.push_back(r.start);
        pool_.push_back(r.end);
    }
    records_.clear();
}

std::string KernelTimer::stats()
{
    std::lock_guard lock(mutex_);
    struct Sum
    {
        std::size_t launches = 0;
        double ms = 0, work = 0;
    };
    std::map<std::string, Sum> sums;
    for (auto& r : records_)
    {
        cuda_ok(cudaEventSynchronize(r.end), "kernel timing");
        float ms = 0;
        cuda_ok(cudaEventElapsedTime(&ms, r.start, r.end), "kernel timing");
        auto& s = sums[r.name];
        ++s.launches;
        s.ms += ms;
        s.work += r.work;
    }
    std::ostringstream out;
    out.precision(9);
    out << '{';
    bool first = true;
    for (const auto& [name, s] : sums)
    {
        out << (first ? "" : ",") << '"' << name << "\":{\"launches\":" << s.launches
            << ",\"ms\":" << s.ms << ",\"work\":" << s.work << '}';
        first = false;
    }
    out << '}';
    return out.str();
}

KernelTimer::Scope::Scope(const char* name, cudaStream_t stream, double work)
    : name_(name), stream_(stream), work_(work)
{
    auto& t = instance();
    if (!t.enabled_)
    {
        return;
    }
    // Launches recorded into a CUDA graph are timed as a whole by their caller.
    cudaStreamCaptureStatus capture = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(stream_, &capture) != cudaSuccess ||
        capture != cudaStreamCaptureStatusNone)
    {
        return;
    }
    std::lock_guard lock(t.mutex_);
    start_ = t.take();
    cudaEventRecord(start_, stream_);
}

KernelTimer::Scope::~Scope()
{
    if (!start_)
    {
        return;
    }
    auto& t = instance();
    std::lock_guard lock(t.mutex_);
    auto end = t.take();
    cudaEventRecord(end, stream_);
    t.records_.push_back({name_, start_, end, work_});
}
} // namespace tsacb

namespace tsacb::dev
{
namespace
{
std::atomic<unsigned long long> launches{0};
thread_local CaptureTally* capturing = nullptr;
} // namespace

void note_launch(unsigned long long kernels)
{
    if (capturing)
        capturing->kernels_ += kernels;
    else
        launches.fetch_add(kernels, std::memory_order_relaxed);
}

unsigned long long launch_count()
{
    return launches.load(std::memory_order_relaxed);
}

CaptureTally::CaptureTally() : outer_(capturing)
{
    capturing = this;
}

CaptureTally::~CaptureTally()
{
    capturing = outer_;
}

unsigned long long CaptureTally::kernels() const
{
    return kernels_;
}
} // namespace tsacb::dev

extern "C"
{
uint64_t tsac_cuda_launch_count(void)
{
    return tsacb::dev::launch_count();
}

int tsac_cuda_kernel_timing(int enable)
{
    return tsacb::guarded(
        [&]
        {
            tsacb::KernelTimer::instance().enable(enable != 0);
            tsacb::KernelTimer::instance().reset();
        });
}

int tsac_cuda_kernel_stats(char** json)
{
    return tsacb::guarded(
        [&]
        {
            tsacb::require(json != nullptr, "null argument");
            const auto s = tsacb::KernelTimer::instance().stats();
            *json = tsacb::malloc_copy(s.c_str(), s.size() + 1);
        });
}
}
