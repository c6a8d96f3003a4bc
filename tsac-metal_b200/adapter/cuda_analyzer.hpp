// tsac::CudaAnalyzer — the B200 backend behind the reference's analyzer seam.
//
// A drop-in peer of ScalarAnalyzer (include/tsac/scalar_analyzer.hpp:8-19)
// and MetalAnalyzer (include/tsac/metal_analyzer.hpp:7-22): it implements
// tsac::AudioAnalyzer (include/tsac/audio_analyzer.hpp:30-37) over the C ABI of
// libtsac_cuda (include/tsac_cuda.h).  The contract it keeps
// (include/tsac/audio_analyzer.hpp:24-29, AUDIO_API.md:81-118):
//  - encode/decode are synchronous: the GPU work is complete on return;
//  - input views are borrowed for the call, returned Bytes / PcmAudio own
//    their storage;
//  - Limits are checked before allocation;
//  - observers run synchronously in entropy order after the work completes,
//    and an exception one throws propagates without leaving the analyzer
//    unusable;
//  - errors are tsac::Error, and nothing falls back to another backend;
//  - calls on one instance are serialised by the instance (concurrent callers
//    wait), separate instances run independently.
#pragma once
#include "tsac/audio_analyzer.hpp"
#include "tsac/model_directory.hpp"

#include <mutex>

struct tsac_cuda_context;

namespace tsac
{
class CudaAnalyzer final : public AudioAnalyzer
{
public:
    // device: CUDA device ordinal; host_threads: host range-coding workers
    // (the CLI's -T, 1..256; 0 = automatic); exact_synthesis: decode with the
    // reference's serial arithmetic (bit-identical PCM) instead of the
    // tensor-core decoder (PCM within 1e-4 (1 + max |x|)).
    explicit CudaAnalyzer(ModelDirectory directory, const Limits& limits = {}, int device = 0,
                          unsigned host_threads = 0, bool exact_synthesis = false);
    ~CudaAnalyzer() override;
    CudaAnalyzer(const CudaAnalyzer&) = delete;
    CudaAnalyzer& operator=(const CudaAnalyzer&) = delete;

    Bytes encode(PcmView audio, const EncodeOptions& options = {},
                 const EntropyObserver& observer = {}) override;
    PcmAudio decode(ByteView stream, const EntropyObserver& observer = {}) override;

private:
    ModelDirectory directory_;
    Limits limits_;
    tsac_cuda_context* context_ = nullptr;
    std::mutex call_;
};
} // namespace tsac
