#include "cuda_analyzer.hpp"

#include "format/container.hpp" // parse_header (src/format/container.hpp:26)
#include "format/entropy.hpp"   // visit_entropy_positions (src/format/entropy.hpp:29-31)
#include "tsac_cuda.h"

#include <memory>

namespace tsac
{
namespace
{
void check(int status)
{
    if (status != TSAC_CUDA_OK)
    {
        throw Error(tsac_cuda_last_error());
    }
}

struct FreeBuffer
{
    void operator()(void* p) const
    {
        tsac_cuda_free(p);
    }
};

bool observing(const EntropyObserver& observer)
{
    return observer.before_symbol || observer.after_symbol;
}

// The observer callbacks of a finished call, in entropy order: before_symbol
// then after_symbol per symbol, as the reference's completed_symbols wrapper
// delivers them (src/common/audio_analyzer.cpp:54-72); `bits` holds each
// symbol's coded bits for an encode and is null for a decode (0 bits,
// src/format/entropy.cpp:150-153).  Fast streams have no entropy symbols.
void replay_observer(const EntropyObserver& observer, ByteView stream, const std::uint32_t* bits,
                     const Limits& limits)
{
    const Header header = parse_header(stream, limits);
    if (header.method != 1)
    {
        return;
    }
    std::size_t symbol = 0;
    visit_entropy_positions(
        header,
        [&](const EntropyPosition& position)
        {
            if (observer.before_symbol)
            {
                observer.before_symbol(position);
            }
            if (observer.after_symbol)
            {
                observer.after_symbol(position, bits ? bits[symbol] : 0);
            }
            ++symbol;
        },
        limits);
}
} // namespace

CudaAnalyzer::CudaAnalyzer(ModelDirectory directory, const Limits& limits, int device, unsigned host_threads,
                           bool exact_synthesis)
    : directory_(std::move(directory)), limits_(limits)
{
    if (host_threads > 256)
    {
        throw Error("CPU thread count exceeds supported limit (256)");
    }
    check(tsac_cuda_context_create(directory_.path().c_str(), device, &context_));
    const tsac_cuda_limits l{limits.file_bytes,      limits.symbols, limits.pcm_bytes,      limits.cache_bytes,
                             limits.tensor_elements, limits.tensors, limits.metadata_bytes, limits.name_bytes};
    try
    {
        check(tsac_cuda_set_limits(context_, &l));
        check(tsac_cuda_set_host_threads(context_, host_threads));
        check(tsac_cuda_set_exact_synthesis(context_, exact_synthesis ? 1 : 0));
    }
    catch (...)
    {
        tsac_cuda_context_destroy(context_);
        throw;
    }
}

CudaAnalyzer::~CudaAnalyzer()
{
    tsac_cuda_context_destroy(context_);
}

Bytes CudaAnalyzer::encode(PcmView audio, const EncodeOptions& options, const EntropyObserver& observer)
{
    // audio_header's batch rule (src/common/audio_analyzer.cpp:99): a batch
    // that is present must be positive; the C ABI reads 0 as "automatic".
    if (options.entropy_batch && *options.entropy_batch == 0)
    {
        throw Error("zero entropy batch size");
    }
    const tsac_cuda_encode_options o{options.method == CodingMethod::normal ? 1 : 0, options.codebooks,
                                     options.separate_channels ? 1 : 0,
                                     options.entropy_batch ? int(*options.entropy_batch) : 0};
    // PcmView is [channel, frame]: extent(0) channels, extent(1) samples, and
    // the strides in floats in the same order.
    const auto channel_stride = static_cast<std::ptrdiff_t>(audio.stride(0));
    const auto sample_stride = static_cast<std::ptrdiff_t>(audio.stride(1));
    std::uint8_t* out = nullptr;
    std::uint32_t* bits = nullptr;
    std::size_t bytes = 0, symbols = 0;
    {
        std::lock_guard lock(call_);
        if (observing(observer))
        {
            check(tsac_cuda_encode_symbol_bits(context_, audio.data_handle(), audio.extent(0), audio.extent(1),
                                               channel_stride, sample_stride, &o, &out, &bytes, &bits, &symbols));
        }
        else
        {
            check(tsac_cuda_encode(context_, audio.data_handle(), audio.extent(0), audio.extent(1), channel_stride,
                                   sample_stride, &o, &out, &bytes, nullptr));
        }
    }
    const std::unique_ptr<std::uint8_t, FreeBuffer> owned(out);
    const std::unique_ptr<std::uint32_t, FreeBuffer> owned_bits(bits);
    Bytes stream(out, out + bytes);
    if (observing(observer))
    {
        replay_observer(observer, stream, bits, limits_);
    }
    return stream;
}

PcmAudio CudaAnalyzer::decode(ByteView stream, const EntropyObserver& observer)
{
    float* out = nullptr;
    std::size_t samples = 0;
    unsigned channels = 0;
    {
        std::lock_guard lock(call_);
        check(tsac_cuda_decode(context_, stream.data(), stream.size(), &out, &samples, &channels));
    }
    const std::unique_ptr<float, FreeBuffer> owned(out);
    PcmAudio audio{std::vector<float>(out, out + samples), channels};
    if (observing(observer))
    {
        replay_observer(observer, stream, nullptr, limits_);
    }
    return audio;
}
} // namespace tsac
