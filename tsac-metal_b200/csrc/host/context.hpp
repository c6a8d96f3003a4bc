// One analyzer instance: a model package bound to one CUDA device and stream.
// Mirrors the reference analyzers' ownership (ModelDirectory + Limits,
// include/tsac/scalar_analyzer.hpp:8-19): prepared device models are created
// on first use per variant and reused by later calls on the same context.
#pragma once
#include "models.hpp"
#include "transformer_engine.hpp"

#include <memory>
#include <mutex>

namespace tsacb
{
class DacEngine;
class RvqEngine;

class Context
{
public:
    Context(const std::string& package, int device, const Limits& limits);
    ~Context();
    Context(const Context&) = delete;
    Context& operator=(const Context&) = delete;

    const Limits& limits() const
    {
        return limits_;
    }
    void set_limits(const Limits& limits)
    {
        limits_ = limits;
    }
    cudaStream_t stream() const
    {
        return stream_;
    }
    void bind() const; // makes the context's device current on this thread
    TransformerEngine& transformer(unsigned channels);
    DacEngine& analysis(unsigned channels);
    DacEngine& synthesis(unsigned channels);
    // Exact synthesis (bit-identical PCM, serial CUDA-core convolutions) or
    // the default tensor-core synthesis (PCM within tolerance).
    void set_exact_synthesis(bool exact);
    // Host worker budget for range coding (the -T thread count of the
    // reference CLI, AppleArmAnalyzer's 1-256 bound,
    // src/apple-arm/audio_analyzer.cpp:93); 0: automatic.
    void set_host_threads(unsigned threads);
    // Certified fast analysis: 0 (default) runs the exact analysis; a positive
    // margin runs fused multiply-add convolutions and recomputes exactly every
    // frame whose RVQ decision margin is below it.
    void set_fast_analysis(float margin);
    float fast_analysis_margin() const
    {
        return fast_margin_;
    }
    // Cumulative counts of the fast analysis: central frames analysed,
    // frames flagged uncertain, frames the exact recomputation evaluated.
    void note_fast_analysis(std::uint64_t frames, std::uint64_t flagged, std::uint64_t recomputed)
    {
        fast_frames_ += frames;
        fast_flagged_ += flagged;
        fast_recomputed_ += recomputed;
    }
    void fast_analysis_stats(std::uint64_t* frames, std::uint64_t* flagged, std::uint64_t* recomputed) const
    {
        *frames = fast_frames_;
        *flagged = fast_flagged_;
        *recomputed = fast_recomputed_;
    }
    unsigned host_threads() const
    {
        return host_threads_;
    }
    RvqEngine& rvq(unsigned channels);
    const Package& package() const
    {
        return package_;
    }
    // Grow-only device buffers of the codec's staging (PCM, window tokens,
    // latents, PCM windows), kept across calls so a call allocates nothing
    // once warm.  Valid until the next get() of the same name.
    Workspace& workspace()
    {
        return workspace_;
    }
    // Pinned host staging for large device -> host results: two halves of
    // `floats_per_half` floats each, allocated on first use and kept.
    float* pinned_staging(std::size_t floats_per_half);

private:
    Package package_;
    int device_;
    unsigned host_threads_ = 0;
    float fast_margin_ = 0.0f;
    std::uint64_t fast_frames_ = 0, fast_flagged_ = 0, fast_recomputed_ = 0;
    Limits limits_;
    cudaStream_t stream_ = nullptr;
    std::shared_ptr<DeviceTransformer> transformers_[2];
    std::unique_ptr<TransformerEngine> engines_[2];
    std::unique_ptr<DacEngine> analysis_[2], synthesis_[2];
    bool exact_synthesis_ = false;
    std::unique_ptr<RvqEngine> rvq_[2];
    Workspace workspace_;
    float* pinned_ = nullptr;
    std::size_t pinned_floats_ = 0;
};
} // namespace tsacb
