// Whole-recording encode/decode on the device: the CudaAnalyzer contract of
// tsac::AudioAnalyzer (include/tsac/audio_analyzer.hpp:30-37), restating the
// shared pipeline glue of the reference (src/common/audio_analyzer.cpp:79-209,
// src/common/audio_pipeline.hpp:36-83, src/scalar/audio_analyzer.cpp:14-63).
#pragma once
#include "context.hpp"
#include "format.hpp"

namespace tsacb
{
struct EncodeOptions
{
    int method = 1;            // 0 fast, 1 normal
    unsigned codebooks = 0;    // 0: model maximum
    bool separate_channels = false;
    int entropy_batch = 0;     // 0: automatic
};

// Borrowed PCM view [channel, frame] with positive strides (in floats).
struct PcmInput
{
    const float* data = nullptr;
    std::size_t channels = 0, samples = 0;
    std::ptrdiff_t channel_stride = 1, sample_stride = 1;
};

struct DecodedAudio
{
    std::vector<float> samples; // interleaved [sample][channel]
    unsigned channels = 1;
};

Header audio_header(const PcmInput& pcm, const EncodeOptions& options, const Limits& limits);

// Batched entry points (one call = many independent recordings).
std::vector<Bytes> encode_batch(Context& ctx, const std::vector<PcmInput>& pcm,
                                const EncodeOptions& options, std::vector<std::size_t>* bits);
std::vector<DecodedAudio> decode_batch(Context& ctx, const std::vector<ByteView>& streams);

// pack_normal (src/format/entropy.cpp:57-123) for known tokens with the GPU
// predictor: header.method must be 1; returns the framed normal stream.
Bytes pack_normal(Context& ctx, Header header, std::span<const std::uint16_t> tokens,
                  std::size_t* bits);

// Pipeline stages, exposed for parity tests.
std::vector<std::uint16_t> analyze_tokens(Context& ctx, const PcmInput& pcm,
                                          const EncodeOptions& options, Header* header_out);
} // namespace tsacb
