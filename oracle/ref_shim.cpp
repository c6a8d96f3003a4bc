// C ABI over the reference's own portable scalar path (ORACLE ONLY).
//
// Compiled by oracle/Makefile against the reference sources in place; it is
// test infrastructure: only tests/, __graft_entry__.smoke() and bench.py's CPU
// baseline load it.  Every entry point calls the reference implementation
// unchanged and returns 0 on success or -1 with a message for ref_last_error().
#include "common/audio_pipeline.hpp"
#include "common/numeric/probability.hpp"
#include "common/probability.hpp"
#include "common/rvq.hpp"
#include "format/categorical.hpp"
#include "format/container.hpp"
#include "format/entropy.hpp"
#include "scalar/pipeline.hpp"
#include "tsac/scalar_analyzer.hpp"
#include "weights/normalization.hpp"
#include "weights/preparation.hpp"

#include <cstdlib>
#include <cstring>

namespace tsac
{
std::uint16_t nearest_rvq_index(std::span<const float, 8>, std::span<const float>);
}

namespace
{
thread_local std::string last_error;

template <class F> int guarded(F&& f)
{
    try
    {
        f();
        return 0;
    }
    catch (const std::exception& e)
    {
        last_error = e.what();
        return -1;
    }
}

template <class T> T* copy_out(const std::vector<T>& v)
{
    auto* p = static_cast<T*>(std::malloc(v.size() * sizeof(T) + 1));
    if (!v.empty())
    {
        std::memcpy(p, v.data(), v.size() * sizeof(T));
    }
    return p;
}

tsac::EncodeOptions options(int method, int codebooks, int separate, int batch)
{
    tsac::EncodeOptions o;
    o.method = method ? tsac::CodingMethod::normal : tsac::CodingMethod::fast;
    o.codebooks = static_cast<unsigned>(codebooks);
    o.separate_channels = separate != 0;
    if (batch > 0)
    {
        o.entropy_batch = static_cast<std::uint16_t>(batch);
    }
    return o;
}
} // namespace

extern "C"
{
const char* ref_last_error()
{
    return last_error.c_str();
}

void ref_free(void* p)
{
    std::free(p);
}

// ---- whole codec (ScalarAnalyzer, src/scalar/audio_analyzer.cpp:14-63) ----
int ref_encode(const char* package, const float* interleaved, std::size_t channels,
               std::size_t samples, int method, int codebooks, int separate, int batch,
               std::uint8_t** out, std::size_t* out_bytes, std::size_t* symbol_bits)
{
    return guarded(
        [&]
        {
            tsac::ScalarAnalyzer analyzer{tsac::ModelDirectory(package)};
            const auto pcm = tsac::interleaved_pcm(
                std::span<const float>(interleaved, channels * samples), channels);
            std::vector<std::size_t> bits;
            tsac::EntropyObserver observer{{},
                                           [&](const tsac::EntropyPosition&, std::size_t b)
                                           {
                                               bits.push_back(b);
                                           }};
            const auto bytes = analyzer.encode(pcm, options(method, codebooks, separate, batch),
                                               symbol_bits ? observer : tsac::EntropyObserver{});
            *out = copy_out(bytes);
            *out_bytes = bytes.size();
            if (symbol_bits)
            {
                std::size_t total = 0;
                for (auto b : bits)
                {
                    total += b;
                }
                *symbol_bits = total;
            }
        });
}

int ref_decode(const char* package, const std::uint8_t* stream, std::size_t bytes, float** out,
               std::size_t* out_samples, unsigned* out_channels)
{
    return guarded(
        [&]
        {
            tsac::ScalarAnalyzer analyzer{tsac::ModelDirectory(package)};
            const auto audio = analyzer.decode(std::span<const std::uint8_t>(stream, bytes));
            *out = copy_out(audio.samples);
            *out_samples = audio.samples.size();
            *out_channels = audio.channels;
        });
}

// Tokens of a stream (fast or normal) in [frame][group][book] order.
int ref_stream_tokens(const char* package, const std::uint8_t* stream, std::size_t bytes,
                      std::uint16_t** out, std::size_t* count)
{
    return guarded(
        [&]
        {
            const std::span<const std::uint8_t> view(stream, bytes);
            const auto header = tsac::parse_header(view);
            std::vector<std::uint16_t> tokens;
            if (header.method == 0)
            {
                tokens = tsac::unpack_fast(view);
            }
            else
            {
                auto transformer = tsac::scalar::CpuTransformer::from_model(
                    tsac::TransformerModel(tsac::ModelDirectory(package),
                                           tsac::detail::audio_variant(header), header.codebooks));
                tsac::TransformerPredictor predictor(transformer);
                tokens = tsac::unpack_normal(view, predictor);
            }
            *out = copy_out(tokens);
            *count = tokens.size();
        });
}

// ---- pipeline stages --------------------------------------------------------
// DAC analysis of one padded recording chunk: pcm [frames*512][C] -> [frames][1024].
int ref_dac_analysis(const char* package, unsigned channels, const float* pcm,
                     std::size_t pcm_frames, float* latent)
{
    return guarded(
        [&]
        {
            const auto variant = channels == 1 ? tsac::ModelVariant::mono : tsac::ModelVariant::stereo;
            const auto analysis = tsac::scalar::DacAnalysis::from_model(
                tsac::DacAnalysisModel(tsac::ModelDirectory(package), variant));
            const auto out = analysis.apply(std::span<const float>(pcm, pcm_frames * channels),
                                            {channels, pcm_frames, 1});
            std::memcpy(latent, out.values.data(), out.values.size() * 4);
        });
}

// Full encoder front end (padding, chunking, analysis, RVQ) -> tokens.
int ref_analyze_tokens(const char* package, const float* interleaved, std::size_t channels,
                       std::size_t samples, int codebooks, int separate,
                       std::uint16_t** out, std::size_t* count)
{
    return guarded(
        [&]
        {
            const auto pcm_view = tsac::interleaved_pcm(
                std::span<const float>(interleaved, channels * samples), channels);
            auto o = options(0, codebooks, separate, 0);
            const tsac::Limits limits;
            const auto header = tsac::detail::audio_header(pcm_view, o, limits);
            const auto pcm = tsac::detail::padded_audio(pcm_view, header, limits);
            const auto variant = tsac::detail::audio_variant(header);
            tsac::ModelDirectory dir(package);
            const auto analysis =
                tsac::scalar::DacAnalysis::from_model(tsac::DacAnalysisModel(dir, variant));
            const auto quantizer = tsac::scalar::RvqEncoder::from_model(tsac::RvqEncoderModel(
                dir, variant, tsac::RvqInputLayout::input_major, header.codebooks));
            const auto tokens = tsac::detail::analyze_audio(
                pcm, header, analysis, quantizer, tsac::detail::audio_chunk_frames(400, limits),
                limits);
            *out = copy_out(tokens);
            *count = tokens.size();
        });
}

// RVQ encode of latents [frames][1024] (one group) -> tokens [frames][books].
int ref_rvq_encode(const char* package, unsigned channels, unsigned books, const float* latent,
                   std::size_t frames, std::uint16_t* tokens)
{
    return guarded(
        [&]
        {
            const auto variant = channels == 1 ? tsac::ModelVariant::mono : tsac::ModelVariant::stereo;
            const auto quantizer = tsac::scalar::RvqEncoder::from_model(tsac::RvqEncoderModel(
                tsac::ModelDirectory(package), variant, tsac::RvqInputLayout::input_major, books));
            tsac::Header header;
            header.model_channels = static_cast<std::uint8_t>(channels);
            header.codebooks = static_cast<std::uint8_t>(books);
            header.frames = frames;
            const auto out = quantizer.encode(header, std::span<const float>(latent, frames * 1024));
            std::memcpy(tokens, out.data(), out.size() * 2);
        });
}

int ref_rvq_decode(const char* package, unsigned channels, unsigned books,
                   const std::uint16_t* tokens, std::size_t frames, float* latent)
{
    return guarded(
        [&]
        {
            const auto variant = channels == 1 ? tsac::ModelVariant::mono : tsac::ModelVariant::stereo;
            const auto decoder = tsac::RvqDecoder::from_model(
                tsac::RvqDecoderModel(tsac::ModelDirectory(package), variant, books));
            tsac::Header header;
            header.model_channels = static_cast<std::uint8_t>(channels);
            header.codebooks = static_cast<std::uint8_t>(books);
            header.frames = frames;
            const auto out = decoder.decode(header, std::span<const std::uint16_t>(tokens, frames * books));
            std::memcpy(latent, out.data(), out.size() * 4);
        });
}

// DAC synthesis of latents [frames][1024] -> PCM [frames*512][C] (one chunk).
int ref_dac_synthesis(const char* package, unsigned channels, const float* latent,
                      std::size_t frames, float* pcm)
{
    return guarded(
        [&]
        {
            const auto variant = channels == 1 ? tsac::ModelVariant::mono : tsac::ModelVariant::stereo;
            const auto synthesis = tsac::scalar::DacSynthesis::from_model(
                tsac::DacSynthesisModel(tsac::ModelDirectory(package), variant));
            const auto out =
                synthesis.apply(std::span<const float>(latent, frames * 1024), {1024, frames, 1});
            std::memcpy(pcm, out.values.data(), out.values.size() * 4);
        });
}

// Transformer probabilities for every symbol of a known token array, in entropy
// order: probs [symbol_count][1024] (the floats TransformerPredictor returns).
int ref_transformer_probabilities(const char* package, unsigned channels, unsigned groups,
                                  unsigned books, std::size_t frames, unsigned batch,
                                  const std::uint16_t* tokens, float* probabilities)
{
    return guarded(
        [&]
        {
            tsac::Header header;
            header.method = 1;
            header.model_channels = static_cast<std::uint8_t>(channels);
            header.groups = static_cast<std::uint8_t>(groups);
            header.codebooks = static_cast<std::uint8_t>(books);
            header.frames = frames;
            header.batch = static_cast<std::uint16_t>(batch);
            auto transformer = tsac::scalar::CpuTransformer::from_model(tsac::TransformerModel(
                tsac::ModelDirectory(package),
                channels == 1 ? tsac::ModelVariant::mono : tsac::ModelVariant::stereo, books));
            tsac::TransformerPredictor predictor(transformer);
            predictor.reset(header);
            std::size_t index = 0;
            tsac::visit_entropy_positions(header,
                                          [&](const tsac::EntropyPosition& p)
                                          {
                                              const auto probs = predictor.predict(p);
                                              std::memcpy(probabilities + index * 1024,
                                                          probs.data(), 1024 * 4);
                                              ++index;
                                              predictor.commit(p, tokens[p.token_offset]);
                                          });
        });
}

// ---- kernels ----------------------------------------------------------------
// PackedLinear::apply (src/common/packed_linear.tpp:85-123) on canonical
// [out][in] int8 weights: input bf16 [columns][in] -> output bf16 [columns][out].
int ref_packed_linear(const std::int8_t* weights, const float* scales, const float* bias,
                      std::size_t input, std::size_t output, const std::uint16_t* x,
                      std::size_t columns, std::uint16_t* y)
{
    return guarded(
        [&]
        {
            // R4 tiling is layout-only (src/common/packed_linear.tpp:60-72).
            std::vector<std::int8_t> tiled(input * output);
            for (std::size_t out = 0; out < output; out += 4)
                for (std::size_t b = 0; b < input / 256; ++b)
                    for (std::size_t q = 0; q < 64; ++q)
                        for (std::size_t row = 0; row < 4; ++row)
                            std::memcpy(tiled.data() + out * input + b * 1024 + q * 16 + row * 4,
                                        weights + (out + row) * input + b * 256 + q * 4, 4);
            std::vector<float> expanded(columns * input);
            for (std::size_t i = 0; i < expanded.size(); ++i)
            {
                expanded[i] = tsac::probability_float(x[i]);
            }
            tsac::ProbabilityBf8l q;
            tsac::scalar::bf8l(expanded, q);
            std::vector<float> ascale(q.scales.size());
            for (std::size_t i = 0; i < ascale.size(); ++i)
            {
                ascale[i] = tsac::probability_float(q.scales[i]);
            }
            const auto blocks = input / 256;
            for (std::size_t c = 0; c < columns; ++c)
            {
                tsac::scalar::Kernels::linear_column(
                    tiled, std::span<const float>(scales, blocks * output),
                    std::span<const float>(bias, output), input, output,
                    std::span<const std::int8_t>(q.values).subspan(c * input, input),
                    std::span<const float>(ascale).subspan(c * blocks, blocks),
                    std::span<std::uint16_t>(y + c * output, output));
            }
        });
}

int ref_bf8l(const float* values, std::size_t count, std::int8_t* q, std::uint16_t* scales)
{
    return guarded(
        [&]
        {
            const auto r = tsac::scalar::bf8l(std::span<const float>(values, count));
            std::memcpy(q, r.values.data(), r.values.size());
            std::memcpy(scales, r.scales.data(), r.scales.size() * 2);
        });
}

int ref_attention(const std::uint16_t* query, const std::uint16_t* keys,
                  const std::uint16_t* values, std::size_t heads, std::size_t head_width,
                  std::size_t time, int prefill, std::uint16_t* out)
{
    return guarded(
        [&]
        {
            const auto w = heads * head_width;
            const auto r = tsac::scalar::attention_bf16(
                std::span<const std::uint16_t>(query, w),
                std::span<const std::uint16_t>(keys, time * w),
                std::span<const std::uint16_t>(values, time * w), heads, head_width,
                0.0883883461356163f, prefill != 0, false);
            std::memcpy(out, r.data(), r.size() * 2);
        });
}

int ref_layer_norm(const std::uint16_t* x, const std::uint16_t* gain, const std::uint16_t* bias,
                   std::size_t n, std::uint16_t* out)
{
    return guarded(
        [&]
        {
            const auto r = tsac::probability_layer_norm_bf16(std::span<const std::uint16_t>(x, n),
                                                             std::span<const std::uint16_t>(gain, n),
                                                             std::span<const std::uint16_t>(bias, n));
            std::memcpy(out, r.data(), n * 2);
        });
}

int ref_rotary(const std::uint16_t* x, const std::uint16_t* coefficients, std::size_t n,
               std::uint16_t* out)
{
    return guarded(
        [&]
        {
            const auto r = tsac::probability_rotary_bf16(
                std::span<const std::uint16_t>(x, n), std::span<const std::uint16_t>(coefficients, n));
            std::memcpy(out, r.data(), n * 2);
        });
}

std::uint16_t ref_gelu(std::uint16_t x)
{
    return tsac::probability_gelu_bf16(x);
}

int ref_softmax(const std::uint16_t* x, std::size_t n, std::uint16_t* out)
{
    return guarded(
        [&]
        {
            const auto r = tsac::probability_softmax_bf16(std::span<const std::uint16_t>(x, n));
            std::memcpy(out, r.data(), n * 2);
        });
}

float ref_probability_sum(const float* x, std::size_t n)
{
    return tsac::probability_sum(std::span<const float>(x, n));
}

float ref_original_exp(float x)
{
    return tsac::detail::probability::original_exp(x);
}

std::uint16_t ref_conditional_q15(float left, float mass)
{
    return tsac::conditional_q15(left, mass);
}

// scalar::Conv1d on folded weights in the reference's stored order.
int ref_conv1d(std::size_t input_channels, std::size_t output_channels, std::size_t kernel,
               std::size_t stride, std::size_t padding, std::size_t dilation, int transposed,
               const float* weights, const float* bias, const float* input, std::size_t frames,
               float* out, std::size_t* out_frames)
{
    return guarded(
        [&]
        {
            const tsac::Conv1dConfig config{input_channels, output_channels, kernel, stride,
                                            padding, dilation,
                                            transposed ? tsac::ConvolutionKind::transposed
                                                       : tsac::ConvolutionKind::ordinary};
            tsac::scalar::Conv1d conv(
                config, std::span<const float>(weights, input_channels * output_channels * kernel),
                std::span<const float>(bias, output_channels));
            const auto r = conv.apply(std::span<const float>(input, frames * input_channels),
                                      {input_channels, frames, 1});
            std::memcpy(out, r.values.data(), r.values.size() * 4);
            *out_frames = r.shape.frames;
        });
}

// A RangeEncoder stream of `count` symbols, each coded by encode_categorical
// (src/format/categorical.cpp:91-117) over its 1024 probabilities.
int ref_encode_categorical(const float* probabilities, const std::uint16_t* symbols, std::size_t count,
                           std::uint8_t** out, std::size_t* out_bytes)
{
    return guarded(
        [&]
        {
            tsac::RangeEncoder encoder;
            for (std::size_t i = 0; i < count; ++i)
                tsac::encode_categorical(encoder, std::span<const float>(probabilities + i * 1024, 1024),
                                         symbols[i]);
            const auto bytes = encoder.finish();
            *out = copy_out(bytes);
            *out_bytes = bytes.size();
        });
}

// nearest_rvq_index (src/common/rvq.cpp:126-146) over 1024 search vectors.
std::uint16_t ref_rvq_nearest(const float* projected8, const float* search)
{
    return tsac::nearest_rvq_index(std::span<const float, 8>(projected8, 8),
                                   std::span<const float>(search, 1024 * 8));
}

// project_codebook, fused (src/weights/preparation.cpp:95-114): codebook
// [1024][8], weights [1024][8], bias [1024] -> out [1024].
int ref_rvq_project(std::uint16_t index, const float* codebook, const float* weights, const float* bias,
                    float* out)
{
    return guarded(
        [&]
        {
            tsac::weights::project_codebook(index, std::span<const float>(codebook, 1024 * 8),
                                            std::span<const float>(weights, 1024 * 8),
                                            std::span<const float>(bias, 1024), std::span<float>(out, 1024),
                                            true);
        });
}

int ref_snake(const float* input, std::size_t channels, std::size_t frames, const float* alpha,
              float* out)
{
    return guarded(
        [&]
        {
            const auto r = tsac::scalar::snake_dac(std::span<const float>(input, channels * frames),
                                                   {channels, frames, 1},
                                                   std::span<const float>(alpha, channels));
            std::memcpy(out, r.values.data(), r.values.size() * 4);
        });
}
}

extern "C"
{
// pack_normal with the reference CpuTransformer predictor for known tokens
// [frame][group][book] (src/format/entropy.cpp:57-123).  Also returns, when
// `row_crc` is non-null, one CRC-32 per symbol (token-offset order) of the
// 4096 bytes of that symbol's float probabilities.
int ref_pack_normal(const char* package, unsigned channels, unsigned groups, unsigned books,
                    std::size_t frames, unsigned batch, const std::uint16_t* tokens,
                    std::uint8_t** out, std::size_t* out_bytes, std::uint32_t* row_crc)
{
    return guarded(
        [&]
        {
            tsac::Header header;
            header.method = 1;
            header.model_channels = static_cast<std::uint8_t>(channels);
            header.groups = static_cast<std::uint8_t>(groups);
            header.codebooks = static_cast<std::uint8_t>(books);
            header.frames = frames;
            header.batch = static_cast<std::uint16_t>(batch);
            auto transformer = tsac::scalar::CpuTransformer::from_model(tsac::TransformerModel(
                tsac::ModelDirectory(package),
                channels == 1 ? tsac::ModelVariant::mono : tsac::ModelVariant::stereo, books));
            tsac::TransformerPredictor inner(transformer);
            struct Recording final : tsac::TokenPredictor
            {
                tsac::TokenPredictor& base;
                std::uint32_t* crc;
                explicit Recording(tsac::TokenPredictor& b, std::uint32_t* c) : base(b), crc(c) {}
                void reset(const tsac::Header& h) override { base.reset(h); }
                std::span<const float> predict(const tsac::EntropyPosition& p) override
                {
                    const auto probs = base.predict(p);
                    if (crc)
                    {
                        std::uint32_t c = 0xffffffffu;
                        const auto* bytes = reinterpret_cast<const std::uint8_t*>(probs.data());
                        for (std::size_t i = 0; i < probs.size() * 4; ++i)
                        {
                            c ^= bytes[i];
                            for (int k = 0; k < 8; ++k)
                                c = (c >> 1) ^ (0xedb88320u & (0u - (c & 1u)));
                        }
                        crc[p.token_offset] = ~c;
                    }
                    return probs;
                }
                void commit(const tsac::EntropyPosition& p, std::uint16_t t) override
                {
                    base.commit(p, t);
                }
            } predictor(inner, row_crc);
            const auto bytes = tsac::pack_normal(
                header, std::span<const std::uint16_t>(tokens, header.symbol_count()), predictor);
            *out = copy_out(bytes);
            *out_bytes = bytes.size();
        });
}
}

extern "C"
{
// pack_fast (src/format/container.cpp:105-135): a method-0 stream of tokens
// [frame][group][book], 10 bits each.
int ref_pack_fast(unsigned channels, unsigned groups, unsigned books, std::size_t frames,
                  const std::uint16_t* tokens, std::uint8_t** out, std::size_t* out_bytes)
{
    return guarded(
        [&]
        {
            tsac::Header header;
            header.method = 0;
            header.model_channels = static_cast<std::uint8_t>(channels);
            header.groups = static_cast<std::uint8_t>(groups);
            header.codebooks = static_cast<std::uint8_t>(books);
            header.frames = frames;
            header.batch = 1;
            const auto bytes =
                tsac::pack_fast(header, std::span<const std::uint16_t>(tokens, header.symbol_count()));
            *out = copy_out(bytes);
            *out_bytes = bytes.size();
        });
}
}

namespace
{
// The five prepared models ScalarAnalyzer builds inside every encode/decode
// call (src/scalar/audio_analyzer.cpp:14-63), built once for one (variant,
// codebooks) so that a timing loop measures coding, not model preparation.
struct RefSession
{
    tsac::ModelDirectory directory;
    tsac::ModelVariant variant;
    unsigned books;
    tsac::scalar::DacAnalysis analysis;
    tsac::scalar::RvqEncoder encoder;
    tsac::scalar::CpuTransformer transformer;
    tsac::RvqDecoder decoder;
    tsac::scalar::DacSynthesis synthesis;

    RefSession(const char* package, unsigned channels, unsigned codebooks)
        : directory(package),
          variant(channels == 1 ? tsac::ModelVariant::mono : tsac::ModelVariant::stereo),
          books(codebooks),
          analysis(tsac::scalar::DacAnalysis::from_model(tsac::DacAnalysisModel(directory, variant))),
          encoder(tsac::scalar::RvqEncoder::from_model(tsac::RvqEncoderModel(
              directory, variant, tsac::RvqInputLayout::input_major, codebooks))),
          transformer(tsac::scalar::CpuTransformer::from_model(
              tsac::TransformerModel(directory, variant, codebooks))),
          decoder(tsac::RvqDecoder::from_model(tsac::RvqDecoderModel(directory, variant, codebooks))),
          synthesis(
              tsac::scalar::DacSynthesis::from_model(tsac::DacSynthesisModel(directory, variant)))
    {
    }
};
} // namespace

extern "C"
{
int ref_session_create(const char* package, unsigned channels, unsigned codebooks, void** out)
{
    return guarded([&] { *out = new RefSession(package, channels, codebooks); });
}

void ref_session_destroy(void* session)
{
    delete static_cast<RefSession*>(session);
}

// The body of ScalarAnalyzer::encode (src/scalar/audio_analyzer.cpp:14-39) on
// the session's prepared models; the options must select the session's
// variant and codebook count.
int ref_session_encode(void* handle, const float* interleaved, std::size_t channels,
                       std::size_t samples, int method, int batch, std::uint8_t** out,
                       std::size_t* out_bytes)
{
    return guarded(
        [&]
        {
            auto& s = *static_cast<RefSession*>(handle);
            const tsac::Limits limits{};
            const auto pcm = tsac::interleaved_pcm(
                std::span<const float>(interleaved, channels * samples), channels);
            const auto header =
                tsac::detail::audio_header(pcm, options(method, s.books, 0, batch), limits);
            if (tsac::detail::audio_variant(header) != s.variant || header.codebooks != s.books)
            {
                throw std::runtime_error("options do not match the prepared session");
            }
            const auto padded = tsac::detail::padded_audio(pcm, header, limits);
            const auto tokens = tsac::detail::analyze_audio(
                padded, header, s.analysis, s.encoder, tsac::detail::audio_chunk_frames(400, limits),
                limits);
            tsac::Bytes bytes;
            if (header.method == 0)
            {
                bytes = tsac::pack_fast(header, tokens, limits);
            }
            else
            {
                tsac::TransformerPredictor predictor(s.transformer, limits);
                bytes = tsac::pack_normal(header, tokens, predictor, limits, {});
            }
            *out = copy_out(bytes);
            *out_bytes = bytes.size();
        });
}

// The body of ScalarAnalyzer::decode (src/scalar/audio_analyzer.cpp:41-63).
int ref_session_decode(void* handle, const std::uint8_t* stream, std::size_t bytes, float** out,
                       std::size_t* out_samples, unsigned* out_channels)
{
    return guarded(
        [&]
        {
            auto& s = *static_cast<RefSession*>(handle);
            const tsac::Limits limits{};
            const std::span<const std::uint8_t> view(stream, bytes);
            const auto header = tsac::parse_header(view, limits);
            if (tsac::detail::audio_variant(header) != s.variant || header.codebooks != s.books)
            {
                throw std::runtime_error("stream does not match the prepared session");
            }
            std::vector<std::uint16_t> tokens;
            if (header.method == 0)
            {
                tokens = tsac::unpack_fast(view, limits);
            }
            else
            {
                tsac::TransformerPredictor predictor(s.transformer, limits);
                tokens = tsac::unpack_normal(view, predictor, limits, {});
            }
            const auto audio = tsac::detail::synthesize_audio(
                tokens, header, s.decoder, s.synthesis, tsac::detail::audio_chunk_frames(400, limits),
                limits);
            *out = copy_out(audio.samples);
            *out_samples = audio.samples.size();
            *out_channels = audio.channels;
        });
}
}
