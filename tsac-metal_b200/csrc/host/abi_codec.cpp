// C ABI: analyzer contexts, whole-recording encode/decode and the stage entry
// points used by the parity tests.
#include "abi_util.hpp"
#include "codec.hpp"
#include "dac_engine.hpp"

struct tsac_cuda_context
{
    tsacb::Context impl;
    tsac_cuda_context(const char* package, int device) : impl(package, device, tsacb::Limits{})
    {
    }
};

namespace
{
tsacb::EncodeOptions options(const tsac_cuda_encode_options* o)
{
    tsacb::EncodeOptions r;
    if (o)
    {
        r.method = o->method;
        r.codebooks = o->codebooks;
        r.separate_channels = o->separate_channels != 0;
        r.entropy_batch = o->entropy_batch;
    }
    return r;
}

tsacb::PcmInput pcm_input(const float* pcm, size_t channels, size_t samples,
                          ptrdiff_t channel_stride, ptrdiff_t sample_stride)
{
    tsacb::PcmInput p;
    p.data = pcm;
    p.channels = channels;
    p.samples = samples;
    p.channel_stride = channel_stride;
    p.sample_stride = sample_stride;
    return p;
}

template <class T> tsacb::DeviceBuffer to_device(const T* data, std::size_t count, cudaStream_t s)
{
    tsacb::DeviceBuffer b(count * sizeof(T));
    tsacb::cuda_ok(cudaMemcpyAsync(b.as<void>(), data, count * sizeof(T), cudaMemcpyHostToDevice, s),
                   "H2D");
    return b;
}
} // namespace

extern "C"
{
int tsac_cuda_context_create(const char* package, int device, tsac_cuda_context** out)
{
    return tsacb::guarded(
        [&]
        {
            tsacb::require(package && out, "null argument");
            *out = new tsac_cuda_context(package, device);
        });
}

void tsac_cuda_context_destroy(tsac_cuda_context* ctx)
{
    delete ctx;
}

int tsac_cuda_encode(tsac_cuda_context* ctx, const float* pcm, size_t channels, size_t samples,
                     ptrdiff_t channel_stride, ptrdiff_t sample_stride,
                     const tsac_cuda_encode_options* opts, uint8_t** out, size_t* out_bytes,
                     size_t* symbol_bits)
{
    return tsacb::guarded(
        [&]
        {
            tsacb::require(ctx && out && out_bytes, "null argument");
            std::vector<std::size_t> bits;
            auto r = tsacb::encode_batch(ctx->impl,
                                         {pcm_input(pcm, channels, samples, channel_stride, sample_stride)},
                                         options(opts), &bits);
            *out = tsacb::malloc_copy(r[0].data(), r[0].size());
            *out_bytes = r[0].size();
            if (symbol_bits)
                *symbol_bits = bits[0];
        });
}

int tsac_cuda_encode_observed(tsac_cuda_context* ctx, const float* pcm, size_t channels,
                              size_t samples, ptrdiff_t channel_stride, ptrdiff_t sample_stride,
                              const tsac_cuda_encode_options* opts, uint8_t** out,
                              size_t* out_bytes, uint64_t* codebook_bits, size_t codebooks)
{
    return tsacb::guarded(
        [&]
        {
            tsacb::require(ctx && out && out_bytes && (codebook_bits || codebooks == 0),
                           "null argument");
            std::vector<std::size_t> bits;
            std::vector<std::vector<std::size_t>> book_bits;
            auto r = tsacb::encode_batch(ctx->impl,
                                         {pcm_input(pcm, channels, samples, channel_stride, sample_stride)},
                                         options(opts), &bits, &book_bits);
            for (size_t b = 0; b < codebooks; ++b)
                codebook_bits[b] = b < book_bits[0].size() ? book_bits[0][b] : 0;
            *out = tsacb::malloc_copy(r[0].data(), r[0].size());
            *out_bytes = r[0].size();
        });
}

int tsac_cuda_encode_symbol_bits(tsac_cuda_context* ctx, const float* pcm, size_t channels,
                                 size_t samples, ptrdiff_t channel_stride, ptrdiff_t sample_stride,
                                 const tsac_cuda_encode_options* opts, uint8_t** out, size_t* out_bytes,
                                 uint32_t** symbol_bits, size_t* symbols)
{
    return tsacb::guarded(
        [&]
        {
            tsacb::require(ctx && out && out_bytes && symbol_bits && symbols, "null argument");
            std::vector<std::size_t> bits;
            std::vector<std::vector<std::uint32_t>> per_symbol;
            auto r = tsacb::encode_batch(ctx->impl,
                                         {pcm_input(pcm, channels, samples, channel_stride, sample_stride)},
                                         options(opts), &bits, nullptr, &per_symbol);
            *symbol_bits = per_symbol[0].empty() ? nullptr
                                                 : tsacb::malloc_copy(per_symbol[0].data(), per_symbol[0].size());
            *symbols = per_symbol[0].size();
            *out = tsacb::malloc_copy(r[0].data(), r[0].size());
            *out_bytes = r[0].size();
        });
}

namespace
{
// Host-result decoding: each recording's buffer is allocated (malloc, for
// tsac_cuda_free) once its header has passed the context's limits, and the
// decoder copies the PCM from the device straight into it.
void decode_to_host(tsac_cuda_context& ctx, size_t count, const uint8_t* const* streams, const size_t* bytes,
                    float** out, size_t* samples, unsigned* channels)
{
    std::vector<tsacb::ByteView> views;
    std::vector<float*> buffers(count, nullptr);
    try
    {
        for (size_t i = 0; i < count; ++i)
        {
            views.emplace_back(streams[i], bytes[i]);
            const auto h = tsacb::read_header(views.back(), ctx.impl.limits());
            const auto n = tsacb::checked_mul(h.channels(), h.samples_per_channel());
            tsacb::require(n <= ctx.impl.limits().tensor_elements, "output audio exceeds element limit");
            buffers[i] = static_cast<float*>(std::malloc(n * sizeof(float) + 1));
            if (!buffers[i])
                throw tsacb::Error("out of host memory");
            samples[i] = n;
            channels[i] = static_cast<unsigned>(h.channels());
        }
        tsacb::decode_batch(ctx.impl, views, nullptr, buffers.data());
    }
    catch (...)
    {
        for (auto* b : buffers)
            std::free(b);
        throw;
    }
    for (size_t i = 0; i < count; ++i)
        out[i] = buffers[i];
}
} // namespace

int tsac_cuda_decode(tsac_cuda_context* ctx, const uint8_t* stream, size_t bytes, float** out,
                     size_t* samples, unsigned* channels)
{
    return tsacb::guarded(
        [&]
        {
            tsacb::require(ctx && stream && out && samples && channels, "null argument");
            const uint8_t* const streams[1] = {stream};
            decode_to_host(*ctx, 1, streams, &bytes, out, samples, channels);
        });
}

int tsac_cuda_encode_batch(tsac_cuda_context* ctx, size_t count, const float* const* pcm,
                           const size_t* channels, const size_t* samples,
                           const tsac_cuda_encode_options* opts, uint8_t** out,
                           size_t* out_bytes)
{
    return tsacb::guarded(
        [&]
        {
            tsacb::require(ctx && pcm && channels && samples && out && out_bytes, "null argument");
            std::vector<tsacb::PcmInput> inputs;
            for (size_t i = 0; i < count; ++i)
                inputs.push_back(pcm_input(pcm[i], channels[i], samples[i], 1,
                                           static_cast<ptrdiff_t>(channels[i])));
            auto r = tsacb::encode_batch(ctx->impl, inputs, options(opts), nullptr);
            for (size_t i = 0; i < count; ++i)
            {
                out[i] = tsacb::malloc_copy(r[i].data(), r[i].size());
                out_bytes[i] = r[i].size();
            }
        });
}

int tsac_cuda_decode_batch(tsac_cuda_context* ctx, size_t count, const uint8_t* const* streams,
                           const size_t* bytes, float** out, size_t* samples,
                           unsigned* channels)
{
    return tsacb::guarded(
        [&]
        {
            tsacb::require(ctx && streams && bytes && out && samples && channels, "null argument");
            decode_to_host(*ctx, count, streams, bytes, out, samples, channels);
        });
}

int tsac_cuda_stream_info(const uint8_t* stream, size_t bytes, unsigned* channels,
                          size_t* samples_per_channel, size_t* symbols)
{
    return tsacb::guarded(
        [&]
        {
            tsacb::require(stream && channels && samples_per_channel, "null argument");
            const auto h = tsacb::read_header(tsacb::ByteView(stream, bytes));
            *channels = static_cast<unsigned>(h.channels());
            *samples_per_channel = h.samples_per_channel();
            if (symbols)
                *symbols = h.symbol_count();
        });
}

int tsac_cuda_stream_header_info(const uint8_t* stream, size_t bytes, tsac_cuda_stream_header* out)
{
    return tsacb::guarded(
        [&]
        {
            tsacb::require(stream && out, "null argument");
            const auto h = tsacb::read_header(tsacb::ByteView(stream, bytes));
            out->method = h.method;
            out->model_channels = h.model_channels;
            out->groups = h.groups;
            out->codebooks = h.codebooks;
            out->frames = h.frames;
            out->batch = h.batch;
        });
}

int tsac_cuda_unpack_fast(const uint8_t* stream, size_t bytes, uint16_t** tokens, size_t* count)
{
    return tsacb::guarded(
        [&]
        {
            tsacb::require(stream && tokens && count, "null argument");
            const auto values = tsacb::fast_tokens(tsacb::ByteView(stream, bytes));
            *tokens = tsacb::malloc_copy(values.data(), values.size());
            *count = values.size();
        });
}

int tsac_cuda_range_encode_tree(const float* masses, const uint16_t* symbols, size_t count, uint8_t** out,
                                size_t* out_bytes)
{
    return tsacb::guarded(
        [&]
        {
            tsacb::require(out && out_bytes && (count == 0 || (masses && symbols)), "null argument");
            tsacb::RangeWriter encoder;
            for (size_t i = 0; i < count; ++i)
            {
                tsacb::require(symbols[i] < 1024, "symbol exceeds alphabet");
                tsacb::write_symbol(encoder, masses + i * 1023, symbols[i]);
            }
            const auto bytes = encoder.finish();
            *out = tsacb::malloc_copy(bytes.data(), bytes.size());
            *out_bytes = bytes.size();
        });
}

int tsac_cuda_range_decode_tree(const uint8_t* bytes, size_t size, const float* masses, size_t count,
                                uint16_t* symbols)
{
    return tsacb::guarded(
        [&]
        {
            tsacb::require((bytes || size == 0) && (count == 0 || (masses && symbols)), "null argument");
            tsacb::RangeReader decoder(tsacb::ByteView(bytes, size));
            for (size_t i = 0; i < count; ++i)
                symbols[i] = decoder.symbol(masses + i * 1023);
        });
}

uint32_t tsac_cuda_token_crc32(const uint16_t* tokens, size_t count)
{
    return tsacb::token_crc32(std::span<const std::uint16_t>(tokens, tokens ? count : 0));
}

int tsac_cuda_encode_batch_device(tsac_cuda_context* ctx, size_t count,
                                  const float* const* pcm_device, const size_t* channels,
                                  const size_t* samples, const tsac_cuda_encode_options* opts,
                                  uint8_t** out, size_t* out_bytes)
{
    return tsacb::guarded(
        [&]
        {
            tsacb::require(ctx && pcm_device && channels && samples && out && out_bytes,
                           "null argument");
            std::vector<tsacb::PcmInput> inputs;
            for (size_t i = 0; i < count; ++i)
            {
                auto p = pcm_input(pcm_device[i], channels[i], samples[i], 1,
                                   static_cast<ptrdiff_t>(channels[i]));
                p.device = true;
                inputs.push_back(p);
            }
            auto r = tsacb::encode_batch(ctx->impl, inputs, options(opts), nullptr);
            for (size_t i = 0; i < count; ++i)
            {
                out[i] = tsacb::malloc_copy(r[i].data(), r[i].size());
                out_bytes[i] = r[i].size();
            }
        });
}

int tsac_cuda_decode_batch_device(tsac_cuda_context* ctx, size_t count,
                                  const uint8_t* const* streams, const size_t* bytes,
                                  float* const* pcm_device)
{
    return tsacb::guarded(
        [&]
        {
            tsacb::require(ctx && streams && bytes && pcm_device, "null argument");
            std::vector<tsacb::ByteView> views;
            for (size_t i = 0; i < count; ++i)
                views.emplace_back(streams[i], bytes[i]);
            tsacb::decode_batch(ctx->impl, views, pcm_device);
        });
}

int tsac_cuda_analyze_tokens(tsac_cuda_context* ctx, const float* pcm, size_t channels,
                             size_t samples, const tsac_cuda_encode_options* opts,
                             uint16_t** tokens, size_t* count)
{
    return tsacb::guarded(
        [&]
        {
            tsacb::require(ctx && tokens && count, "null argument");
            auto t = tsacb::analyze_tokens(ctx->impl,
                                           pcm_input(pcm, channels, samples, 1,
                                                     static_cast<ptrdiff_t>(channels)),
                                           options(opts), nullptr);
            *tokens = tsacb::malloc_copy(t.data(), t.size());
            *count = t.size();
        });
}

int tsac_cuda_transformer_probabilities(tsac_cuda_context* ctx, unsigned channels,
                                        unsigned groups, unsigned books, size_t frames,
                                        unsigned batch, const uint16_t* tokens,
                                        float* probabilities, uint16_t* q15)
{
    return tsacb::guarded(
        [&]
        {
            tsacb::require(ctx && tokens, "null argument");
            ctx->impl.bind();
            tsacb::Header h;
            h.method = 1;
            h.model_channels = static_cast<std::uint8_t>(channels);
            h.groups = static_cast<std::uint8_t>(groups);
            h.codebooks = static_cast<std::uint8_t>(books);
            h.frames = frames;
            h.batch = static_cast<std::uint16_t>(batch);
            tsacb::check_header(h);
            std::vector<std::uint16_t> q(h.symbol_count() * 10);
            ctx->impl.transformer(channels).predict_known(
                h, std::span<const std::uint16_t>(tokens, h.symbol_count()), q.data(),
                probabilities);
            if (q15)
                std::copy(q.begin(), q.end(), q15);
        });
}

int tsac_cuda_pack_normal(tsac_cuda_context* ctx, unsigned channels, unsigned groups,
                          unsigned books, size_t frames, unsigned batch, const uint16_t* tokens,
                          uint8_t** out, size_t* out_bytes)
{
    return tsacb::guarded(
        [&]
        {
            tsacb::require(ctx && tokens && out && out_bytes, "null argument");
            tsacb::Header h;
            h.method = 1;
            h.model_channels = static_cast<std::uint8_t>(channels);
            h.groups = static_cast<std::uint8_t>(groups);
            h.codebooks = static_cast<std::uint8_t>(books);
            h.frames = frames;
            h.batch = static_cast<std::uint16_t>(batch);
            const auto bytes = tsacb::pack_normal(
                ctx->impl, h, std::span<const std::uint16_t>(tokens, h.symbol_count()), nullptr);
            *out = tsacb::malloc_copy(bytes.data(), bytes.size());
            *out_bytes = bytes.size();
        });
}

int tsac_cuda_dac_analysis(tsac_cuda_context* ctx, unsigned channels, const float* pcm,
                           size_t pcm_frames, float* latent)
{
    return tsacb::guarded(
        [&]
        {
            tsacb::require(ctx && pcm && latent, "null argument");
            tsacb::require(pcm_frames > 0 && pcm_frames % 512 == 0,
                           "analysis PCM must be a nonempty multiple of 512 samples");
            ctx->impl.bind();
            auto s = ctx->impl.stream();
            auto& dac = ctx->impl.analysis(channels);
            auto d_pcm = to_device(pcm, pcm_frames * channels, s);
            const auto frames = pcm_frames / 512;
            tsacb::DeviceBuffer d_lat(frames * 1024 * 4);
            dac.analyze(d_pcm.as<float>(), {0}, {static_cast<int>(frames)}, d_lat.as<float>(),
                        ctx->impl.fast_analysis_margin() > 0.0f);
            tsacb::cuda_ok(cudaMemcpyAsync(latent, d_lat.as<void>(), frames * 1024 * 4,
                                           cudaMemcpyDeviceToHost, s),
                           "D2H");
            dac.check_errors("analysis");
        });
}

int tsac_cuda_set_exact_synthesis(tsac_cuda_context* ctx, int exact)
{
    return tsacb::guarded(
        [&]
        {
            tsacb::require(ctx != nullptr, "null argument");
            ctx->impl.set_exact_synthesis(exact != 0);
        });
}

int tsac_cuda_set_limits(tsac_cuda_context* ctx, const tsac_cuda_limits* limits)
{
    return tsacb::guarded(
        [&]
        {
            tsacb::require(ctx && limits, "null argument");
            ctx->impl.set_limits({limits->file_bytes, limits->symbols, limits->pcm_bytes, limits->cache_bytes,
                                  limits->tensor_elements, limits->tensors, limits->metadata_bytes,
                                  limits->name_bytes});
        });
}

int tsac_cuda_set_fast_analysis(tsac_cuda_context* ctx, float margin)
{
    return tsacb::guarded(
        [&]
        {
            tsacb::require(ctx != nullptr, "null argument");
            ctx->impl.set_fast_analysis(margin);
        });
}

int tsac_cuda_fast_analysis_stats(tsac_cuda_context* ctx, uint64_t* frames, uint64_t* uncertain,
                                  uint64_t* recomputed_frames)
{
    return tsacb::guarded(
        [&]
        {
            tsacb::require(ctx && frames && uncertain && recomputed_frames, "null argument");
            std::uint64_t f = 0, u = 0, r = 0;
            ctx->impl.fast_analysis_stats(&f, &u, &r);
            *frames = f;
            *uncertain = u;
            *recomputed_frames = r;
        });
}

int tsac_cuda_set_host_threads(tsac_cuda_context* ctx, unsigned threads)
{
    return tsacb::guarded(
        [&]
        {
            tsacb::require(ctx != nullptr, "null argument");
            ctx->impl.set_host_threads(threads);
        });
}

int tsac_cuda_dac_synthesis(tsac_cuda_context* ctx, unsigned channels, const float* latent,
                            size_t frames, float* pcm)
{
    return tsacb::guarded(
        [&]
        {
            tsacb::require(ctx && pcm && latent && frames > 0, "null argument");
            ctx->impl.bind();
            auto s = ctx->impl.stream();
            auto& dac = ctx->impl.synthesis(channels);
            auto d_lat = to_device(latent, frames * 1024, s);
            tsacb::DeviceBuffer d_pcm(frames * 512 * channels * 4);
            dac.synthesize(d_lat.as<float>(), {static_cast<int>(frames)}, d_pcm.as<float>());
            tsacb::cuda_ok(cudaMemcpyAsync(pcm, d_pcm.as<void>(), frames * 512 * channels * 4,
                                           cudaMemcpyDeviceToHost, s),
                           "D2H");
            dac.check_errors("synthesis");
        });
}

int tsac_cuda_rvq_encode(tsac_cuda_context* ctx, unsigned channels, unsigned books,
                         const float* latent, size_t frames, uint16_t* tokens)
{
    return tsacb::guarded(
        [&]
        {
            tsacb::require(ctx && latent && tokens, "null argument");
            ctx->impl.bind();
            auto s = ctx->impl.stream();
            auto& rvq = ctx->impl.rvq(channels);
            auto d_lat = to_device(latent, frames * 1024, s);
            tsacb::DeviceBuffer d_tok(frames * books * 2 + 2);
            rvq.encode(d_lat.as<float>(), static_cast<int>(frames), static_cast<int>(books),
                       d_tok.as<std::uint16_t>(), static_cast<int>(books));
            tsacb::cuda_ok(cudaMemcpyAsync(tokens, d_tok.as<void>(), frames * books * 2,
                                           cudaMemcpyDeviceToHost, s),
                           "D2H");
            tsacb::cuda_ok(cudaStreamSynchronize(s), "rvq");
        });
}

int tsac_cuda_rvq_decode(tsac_cuda_context* ctx, unsigned channels, unsigned books,
                         const uint16_t* tokens, size_t frames, float* latent)
{
    return tsacb::guarded(
        [&]
        {
            tsacb::require(ctx && latent && tokens, "null argument");
            ctx->impl.bind();
            auto s = ctx->impl.stream();
            auto& rvq = ctx->impl.rvq(channels);
            auto d_tok = to_device(tokens, frames * books, s);
            tsacb::DeviceBuffer d_lat(frames * 1024 * 4);
            rvq.decode(d_tok.as<std::uint16_t>(), static_cast<int>(books), static_cast<int>(frames),
                       static_cast<int>(books), d_lat.as<float>());
            tsacb::cuda_ok(cudaMemcpyAsync(latent, d_lat.as<void>(), frames * 1024 * 4,
                                           cudaMemcpyDeviceToHost, s),
                           "D2H");
            tsacb::cuda_ok(cudaStreamSynchronize(s), "rvq");
        });
}
}
