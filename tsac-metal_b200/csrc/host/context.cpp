#include "context.hpp"

#include "dac_engine.hpp"
#include "kernels/qlinear.cuh"

namespace tsacb
{
namespace
{
void ensure_device(int device)
{
    int count = 0;
    if (cudaGetDeviceCount(&count) != cudaSuccess || count == 0)
    {
        throw DeviceError("no CUDA device available (this library has no CPU fallback)");
    }
    require(device >= 0 && device < count, "CUDA device index out of range");
}
} // namespace

Context::Context(const std::string& package, int device, const Limits& limits)
    : package_(package, limits), device_(device), limits_(limits)
{
    ensure_device(device);
    cuda_ok(cudaSetDevice(device), "cudaSetDevice");
    cuda_ok(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking), "cudaStreamCreate");
    dev::qlinear_init();
}

Context::~Context()
{
    cudaSetDevice(device_);
    for (auto& e : engines_)
        e.reset();
    for (auto& a : analysis_)
        a.reset();
    for (auto& s : synthesis_)
        s.reset();
    for (auto& r : rvq_)
        r.reset();
    for (auto& t : transformers_)
        t.reset();
    if (stream_)
    {
        cudaStreamSynchronize(stream_);
        cudaStreamDestroy(stream_);
    }
    if (pinned_)
        cudaFreeHost(pinned_);
}

void Context::bind() const
{
    cuda_ok(cudaSetDevice(device_), "cudaSetDevice");
}

TransformerEngine& Context::transformer(unsigned channels)
{
    require(channels == 1 || channels == 2, "invalid model variant");
    auto& e = engines_[channels - 1];
    if (!e)
    {
        const unsigned books = channels == 1 ? 9 : 12;
        transformers_[channels - 1] = std::make_shared<DeviceTransformer>(
            prepare_transformer(package_, channels, books), stream_);
        e = std::make_unique<TransformerEngine>(transformers_[channels - 1], stream_);
    }
    return *e;
}

DacEngine& Context::analysis(unsigned channels)
{
    require(channels == 1 || channels == 2, "invalid model variant");
    auto& e = analysis_[channels - 1];
    if (!e)
        e = std::make_unique<DacEngine>(prepare_dac(package_, channels, false, limits_), stream_);
    return *e;
}

DacEngine& Context::synthesis(unsigned channels)
{
    require(channels == 1 || channels == 2, "invalid model variant");
    auto& e = synthesis_[channels - 1];
    if (!e)
    {
        e = std::make_unique<DacEngine>(prepare_dac(package_, channels, true, limits_), stream_);
        e->set_exact_synthesis(exact_synthesis_);
    }
    return *e;
}

void Context::set_exact_synthesis(bool exact)
{
    exact_synthesis_ = exact;
    for (auto& e : synthesis_)
        if (e)
            e->set_exact_synthesis(exact);
}

float* Context::pinned_staging(std::size_t floats_per_half)
{
    if (pinned_floats_ < 2 * floats_per_half)
    {
        if (pinned_)
        {
            cuda_ok(cudaStreamSynchronize(stream_), "pinned staging");
            cudaFreeHost(pinned_);
            pinned_ = nullptr;
            pinned_floats_ = 0;
        }
        void* p = nullptr;
        cuda_ok(cudaMallocHost(&p, 2 * floats_per_half * sizeof(float)), "cudaMallocHost");
        pinned_ = static_cast<float*>(p);
        pinned_floats_ = 2 * floats_per_half;
    }
    return pinned_;
}

void Context::set_host_threads(unsigned threads)
{
    require(threads <= 256, "CPU thread count exceeds supported limit (256)");
    host_threads_ = threads;
}

void Context::set_fast_analysis(float margin)
{
    require(margin >= 0.0f && margin <= 2.0f, "fast analysis margin must be in [0, 2]");
    fast_margin_ = margin;
}

RvqEngine& Context::rvq(unsigned channels)
{
    require(channels == 1 || channels == 2, "invalid model variant");
    auto& e = rvq_[channels - 1];
    if (!e)
        e = std::make_unique<RvqEngine>(prepare_rvq(package_, channels, channels == 1 ? 9 : 12),
                                        stream_);
    return *e;
}
} // namespace tsacb
