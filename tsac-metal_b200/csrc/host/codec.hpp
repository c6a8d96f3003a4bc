// Whole-recording encode/decode on the device: the CudaAnalyzer contract of
// tsac::AudioAnalyzer (include/tsac/audio_analyzer.hpp:30-37), restating the
// shared pipeline glue of the reference (src/common/audio_analyzer.cpp:79-209,
// src/common/audio_pipeline.hpp:36-83, src/scalar/audio_analyzer.cpp:14-63).
//
// Data stay in HBM from PCM to latents to tokens: padded PCM is built by a
// device kernel, analysis windows are addressed in place, decoded windows are
// scattered straight into the output PCM.  Only tokens (encode) and the
// range coder's per-symbol inputs cross to the host.
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

// Borrowed PCM view [channel, frame] with positive strides (in floats), in
// host memory or (device = true) in this context's GPU memory.
struct PcmInput
{
    const float* data = nullptr;
    std::size_t channels = 0, samples = 0;
    std::ptrdiff_t channel_stride = 1, sample_stride = 1;
    bool device = false;
};

struct DecodedAudio
{
    std::vector<float> samples; // interleaved [sample][channel] (host results only)
    unsigned channels = 1;
    std::size_t frames = 0;     // samples per channel
};

Header audio_header(const PcmInput& pcm, const EncodeOptions& options, const Limits& limits);

// Batched entry points (one call = many independent recordings).
// bits: each stream's payload bit position before termination; book_bits:
// per-codebook sums and symbol_bits: per-symbol bits in entropy order, the
// values an EntropyObserver's after_symbol receives (empty for fast streams).
std::vector<Bytes> encode_batch(Context& ctx, const std::vector<PcmInput>& pcm,
                                const EncodeOptions& options, std::vector<std::size_t>* bits,
                                std::vector<std::vector<std::size_t>>* book_bits = nullptr,
                                std::vector<std::vector<std::uint32_t>>* symbol_bits = nullptr);
// With device_out, recording i is written to device_out[i] (interleaved,
// channels x padded samples floats) and DecodedAudio::samples stays empty.
// With host_out, recording i is copied from the device straight into the
// caller's host buffer host_out[i] (channels x samples floats) and
// DecodedAudio::samples stays empty.
std::vector<DecodedAudio> decode_batch(Context& ctx, const std::vector<ByteView>& streams,
                                       float* const* device_out = nullptr, float* const* host_out = nullptr);

// pack_normal (src/format/entropy.cpp:57-123) for known tokens with the GPU
// predictor: header.method must be 1; returns the framed normal stream.
Bytes pack_normal(Context& ctx, Header header, std::span<const std::uint16_t> tokens,
                  std::size_t* bits);

// Pipeline stages, exposed for parity tests.
std::vector<std::uint16_t> analyze_tokens(Context& ctx, const PcmInput& pcm,
                                          const EncodeOptions& options, Header* header_out);
} // namespace tsacb
