// The reference's analyzer contract, run on tsac::CudaAnalyzer through an
// AudioAnalyzer& (the cases of the reference's tests/audio_analyzer.cpp:148-425
// that apply to a non-Apple backend): session reuse with repeated and
// concurrent calls, PCM views and layouts, channel groups and empty audio,
// failures with reuse after them and policy limits checked before allocation,
// and normal-stream observers (entropy order, a throwing observer, CRC
// rejection, an explicit zero entropy batch).
//
//   cuda_analyzer_contract PACKAGE_DIR   -> prints "contract: ok", exit 0
#include "cuda_analyzer.hpp"

#include "format/container.hpp"
#include "format/entropy.hpp"

#include <algorithm>
#include <array>
#include <cmath>
#include <cstdio>
#include <future>
#include <limits>
#include <memory>
#include <string>

using namespace tsac;

namespace
{
int checks = 0;

void expect(bool condition, const char* what)
{
    ++checks;
    if (!condition)
    {
        throw Error(std::string("contract violated: ") + what);
    }
}

template <class F> void expect_error(F&& action, const char* what)
{
    bool rejected = false;
    try
    {
        action();
    }
    catch (const Error&)
    {
        rejected = true;
    }
    expect(rejected, what);
}

EncodeOptions fast(unsigned codebooks)
{
    EncodeOptions o;
    o.method = CodingMethod::fast;
    o.codebooks = codebooks;
    return o;
}

void repeated_and_concurrent_calls(AudioAnalyzer& analyzer)
{
    const std::vector<float> pcm(1025, 0.125f);
    const auto input = interleaved_pcm(pcm, 1);
    auto options = fast(1);
    const auto expected = analyzer.encode(input, options);
    expect(analyzer.encode(input, options) == expected, "repeated encode changed the stream");
    auto concurrent = std::async(std::launch::async, [&] { return analyzer.encode(input, options); });
    expect(analyzer.encode(input, options) == expected && concurrent.get() == expected,
           "concurrent encodes on one instance changed the stream");
    const auto decoded = analyzer.decode(expected).samples;
    auto other = std::async(std::launch::async, [&] { return analyzer.decode(expected).samples; });
    expect(analyzer.decode(expected).samples == decoded && other.get() == decoded,
           "concurrent decodes on one instance changed the PCM");
    options.codebooks = 2;
    const auto two = analyzer.encode(input, options);
    expect(parse_header(two).codebooks == 2 && analyzer.encode(input, options) == two,
           "codebook coverage changed between calls");
    options.method = CodingMethod::normal;
    options.entropy_batch = 2;
    const auto normal = analyzer.encode(input, options);
    expect(analyzer.encode(input, options) == normal, "normal encode kept token state between calls");
    const auto samples = analyzer.decode(normal).samples;
    expect(analyzer.decode(normal).samples == samples, "normal decode kept token state between calls");
}

PcmView planar_view(const std::vector<float>& samples, std::size_t channels, std::size_t frames)
{
    return PcmView(samples.data(), PcmView::mapping_type(PcmView::extents_type(channels, frames),
                                                         std::array<std::size_t, 2>{frames, 1}));
}

void layouts(AudioAnalyzer& analyzer)
{
    constexpr std::size_t frames = 529;
    std::vector<float> interleaved(frames * 2), planar(frames * 2);
    for (std::size_t t = 0; t < frames; ++t)
    {
        for (std::size_t c = 0; c < 2; ++c)
        {
            const float value = 0.2f * std::sin(float(t) * 0.031f + float(c));
            interleaved[t * 2 + c] = planar[c * frames + t] = value;
        }
    }
    auto options = fast(2);
    const auto input = interleaved_pcm(interleaved, 2);
    const auto stream = analyzer.encode(input, options);
    expect(stream == analyzer.encode(planar_view(planar, 2, frames), options), "PCM layout changed the tokens");
    const auto header = parse_header(stream);
    expect(header.frames == 2 && header.model_channels == 2 && header.groups == 1, "wrong padded stereo framing");
    const auto decoded = analyzer.decode(stream);
    expect(decoded.channels == 2 && decoded.samples.size() == 2048, "wrong decoded PCM size");
    expect(std::all_of(decoded.samples.begin(), decoded.samples.end(), [](float x) { return std::isfinite(x); }),
           "nonfinite decoded PCM");
    expect(decoded.view().extent(1) == 1024, "wrong owning PCM view");
    const auto slice = frame_view(input, 11, 513);
    const auto copied = std::span(interleaved).subspan(22, 1026);
    expect(analyzer.encode(slice, options) == analyzer.encode(interleaved_pcm(copied, 2), options),
           "a frame slice changed the tokens");
    options.separate_channels = true;
    const auto separate = parse_header(analyzer.encode(input, options));
    expect(separate.model_channels == 1 && separate.groups == 2, "separate channel encoding failed");
}

void groups_and_empty(AudioAnalyzer& analyzer)
{
    const auto options = fast(1);
    std::vector<float> samples(std::size_t{513} * 3);
    for (std::size_t i = 0; i < samples.size(); ++i)
    {
        samples[i] = float(int((i * 37 + i % 3 * 53) % 257) - 128) / 1024;
    }
    const auto stream = analyzer.encode(interleaved_pcm(samples, 3), options);
    const auto header = parse_header(stream);
    expect(header.model_channels == 1 && header.groups == 3 && header.frames == 2, "wrong grouped framing");
    const auto decoded = analyzer.decode(stream);
    expect(decoded.channels == 3 && decoded.samples.size() == 3072, "wrong grouped PCM");
    const auto tokens = unpack_fast(stream);
    for (std::size_t channel = 0; channel < 3; ++channel)
    {
        Header mono = header;
        mono.groups = 1;
        const std::vector<std::uint16_t> selected{tokens[channel], tokens[3 + channel]};
        const auto alone = analyzer.decode(pack_fast(mono, selected));
        bool same = true;
        for (std::size_t frame = 0; frame < 1024; ++frame)
        {
            same = same && decoded.samples[frame * 3 + channel] == alone.samples[frame];
        }
        expect(same, "grouped PCM channel order changed");
    }
    const auto empty = analyzer.encode(interleaved_pcm({}, 2), options);
    const auto output = analyzer.decode(empty);
    expect(output.channels == 2 && output.samples.empty(), "empty audio failed");
}

void failures(AudioAnalyzer& analyzer, const ModelDirectory& directory)
{
    std::vector<float> pcm(512, 0.1f);
    const auto options = fast(1);
    const auto input = interleaved_pcm(pcm, 1);
    const auto expected = analyzer.encode(input, options);
    pcm[0] = std::numeric_limits<float>::quiet_NaN();
    expect_error([&] { analyzer.encode(input, options); }, "accepted nonfinite PCM");
    pcm[0] = 0.1f;
    auto invalid = options;
    invalid.codebooks = 10;
    expect_error([&] { analyzer.encode(input, invalid); }, "accepted unsupported codebooks");
    invalid = options;
    invalid.entropy_batch = 1;
    expect_error([&] { analyzer.encode(input, invalid); }, "accepted a fast-mode entropy batch");
    expect_error([&] { analyzer.decode({}); }, "accepted a missing stream");
    expect(analyzer.encode(input, options) == expected, "a failure prevented reuse");
    Limits limits;
    limits.tensor_elements = 511;
    CudaAnalyzer bounded(directory, limits);
    AudioAnalyzer& small = bounded;
    expect_error([&] { small.encode(input, options); }, "ignored the PCM allocation limit");
    expect_error([&] { small.decode(expected); }, "ignored the output allocation limit");
    expect_error([&] { CudaAnalyzer(directory, {}, 0, 257); }, "accepted a thread budget above 256");
}

void normal_streams(AudioAnalyzer& analyzer)
{
    std::vector<float> pcm(std::size_t{513} * 2, 0.1f);
    EncodeOptions options;
    options.codebooks = 2;
    options.entropy_batch = 7; // more lanes than frames
    std::vector<std::size_t> encoded, decoded, before;
    const auto bytes = analyzer.encode(interleaved_pcm(pcm, 2), options,
                                       {[&](const EntropyPosition& p) { before.push_back(p.token_offset); },
                                        [&](const EntropyPosition& p, std::size_t) { encoded.push_back(p.token_offset); }});
    const auto result =
        analyzer.decode(bytes, {{}, [&](const EntropyPosition& p, std::size_t) { decoded.push_back(p.token_offset); }});
    std::vector<std::size_t> expected;
    visit_entropy_positions(parse_header(bytes), [&](const EntropyPosition& p) { expected.push_back(p.token_offset); });
    expect(encoded == expected && decoded == expected && before == expected, "entropy observer order changed");
    expect(result.channels == 2 && result.samples.size() == 2048, "normal decode shape changed");
    auto corrupted = bytes;
    corrupted.back() ^= 1;
    expect_error([&] { analyzer.decode(corrupted); }, "accepted an invalid normal CRC");
    expect_error(
        [&]
        {
            analyzer.encode(interleaved_pcm(pcm, 2), options,
                            {{}, [](const EntropyPosition&, std::size_t) { throw Error("observer failure"); }});
        },
        "lost the observer's exception");
    expect(analyzer.decode(bytes).samples == result.samples, "a normal failure prevented reuse");
    options.entropy_batch = 0;
    expect_error([&] { analyzer.encode(interleaved_pcm(pcm, 2), options); }, "accepted an explicit zero batch");
}
} // namespace

int main(int argc, char** argv)
{
    try
    {
        expect(argc == 2, "usage: cuda_analyzer_contract PACKAGE_DIR");
        const ModelDirectory directory(argv[1]);
        CudaAnalyzer cuda(directory);
        AudioAnalyzer& analyzer = cuda;
        repeated_and_concurrent_calls(analyzer);
        layouts(analyzer);
        groups_and_empty(analyzer);
        failures(analyzer, directory);
        normal_streams(analyzer);
        std::printf("contract: ok (%d checks)\n", checks);
        return 0;
    }
    catch (const std::exception& error)
    {
        std::fprintf(stderr, "contract: %s\n", error.what());
        return 1;
    }
}
