#include "codec.hpp"

#include "dac_engine.hpp"
#include "kernels/dac.cuh"

#include <algorithm>
#include <atomic>
#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <exception>
#include <functional>
#include <future>
#include <thread>
#include <utility>

namespace tsacb
{
namespace
{
struct Chunk // detail::AudioChunk (src/common/audio_analyzer.cpp:154-162)
{
    std::size_t begin, count, left, right;
};

Chunk audio_chunk(std::size_t begin, std::size_t frames, std::size_t size, std::size_t lc,
                  std::size_t rc)
{
    require(size > 0 && begin < frames, "invalid audio chunk");
    const auto count = std::min(size, frames - begin);
    const auto end = begin + count;
    return {begin, count, begin > lc ? begin - lc : 0, end + std::min(rc, frames - end)};
}

std::size_t audio_chunk_frames(std::size_t target, const Limits& limits)
{
    const auto available = limits.tensor_elements / (std::size_t{96} * 512);
    return std::min(target, available > 22 ? available - 22 : std::size_t{1});
}

// Windows per DAC launch group: bounds device scratch (~250 MB per window).
constexpr std::size_t window_group = 48;

// Host worker count: the context's budget, else every hardware thread.
std::size_t host_workers(const Context& ctx)
{
    const std::size_t hw = std::max(1u, std::thread::hardware_concurrency());
    return ctx.host_threads() ? ctx.host_threads() : hw;
}

// Host threads for the pinned PCM copies: memory bandwidth saturates with a
// few, and a piece waits for its slowest thread, so more would only add
// exposure to a busy host.
std::size_t copy_workers(const Context& ctx)
{
    return std::min<std::size_t>(host_workers(ctx), 8);
}

template <class F> void parallel_for(std::size_t n, std::size_t max_workers, F&& f)
{
    const std::size_t workers = std::max<std::size_t>(1, std::min(n, max_workers));
    if (workers <= 1)
    {
        for (std::size_t i = 0; i < n; ++i)
            f(i);
        return;
    }
    std::vector<std::future<void>> jobs;
    std::atomic<std::size_t> next{0};
    for (std::size_t w = 0; w < workers; ++w)
    {
        jobs.push_back(std::async(std::launch::async,
                                  [&]
                                  {
                                      for (std::size_t i; (i = next++) < n;)
                                          f(i);
                                  }));
    }
    for (auto& j : jobs)
        j.get();
}


// Stage timing (TSAC_CUDA_PROFILE=1): synchronises the stream at each mark.
class Profile
{
public:
    Profile(cudaStream_t s, const char* name) : stream_(s), name_(name)
    {
        const char* e = std::getenv("TSAC_CUDA_PROFILE");
        enabled_ = e && *e && *e != '0';
        last_ = std::chrono::steady_clock::now();
    }
    void mark(const char* stage)
    {
        if (!enabled_)
            return;
        cudaStreamSynchronize(stream_);
        const auto now = std::chrono::steady_clock::now();
        std::fprintf(stderr, "tsac_cuda %s %-22s %9.3f ms\n", name_, stage,
                     std::chrono::duration<double, std::milli>(now - last_).count());
        last_ = now;
    }

private:
    cudaStream_t stream_;
    const char* name_;
    bool enabled_ = false;
    std::chrono::steady_clock::time_point last_;
};

struct Window
{
    std::size_t recording, group;
    Chunk chunk;
};

void check_word(cudaStream_t s, unsigned* word, const char* message)
{
    unsigned host = 0;
    cuda_ok(cudaMemcpyAsync(&host, word, 4, cudaMemcpyDeviceToHost, s), "D2H");
    cuda_ok(cudaStreamSynchronize(s), message);
    if (host)
    {
        cuda_ok(cudaMemsetAsync(word, 0, 4, s), "memset");
        throw NumericError(message);
    }
}

// Host PCM -> device in 32 MiB pieces through the context's pinned double
// buffer: the host workers copy piece p into one half while piece p - 1 goes
// by DMA from the other (pageable copies ran at about 8 GB/s).  Returns once
// every piece has reached the device.
void upload_pcm(Context& ctx, const std::vector<const float*>& src, const std::vector<float*>& dst,
                const std::vector<std::size_t>& count)
{
    constexpr std::size_t piece = std::size_t{8} << 20; // floats (32 MiB)
    auto s = ctx.stream();
    struct Piece
    {
        std::size_t job, offset, count;
    };
    std::vector<Piece> pieces;
    std::size_t total = 0;
    for (std::size_t j = 0; j < src.size(); ++j)
    {
        total += count[j];
        for (std::size_t at = 0; at < count[j]; at += piece)
            pieces.push_back({j, at, std::min(piece, count[j] - at)});
    }
    if (pieces.empty())
        return;
    if (total < piece / 4)
    {
        for (std::size_t j = 0; j < src.size(); ++j)
            if (count[j])
                cuda_ok(cudaMemcpyAsync(dst[j], src[j], count[j] * 4, cudaMemcpyHostToDevice, s), "H2D");
        cuda_ok(cudaStreamSynchronize(s), "PCM upload");
        return;
    }
    float* staging = ctx.pinned_staging(piece);
    cudaEvent_t done[2] = {nullptr, nullptr};
    for (auto& e : done)
        cuda_ok(cudaEventCreateWithFlags(&e, cudaEventDisableTiming), "cudaEventCreate");
    const std::size_t workers = copy_workers(ctx);
    try
    {
        for (std::size_t p = 0; p < pieces.size(); ++p)
        {
            // This half last carried piece p - 2: its DMA must be finished.
            if (p >= 2)
                cuda_ok(cudaEventSynchronize(done[p & 1]), "H2D");
            const auto& q = pieces[p];
            const float* from = src[q.job] + q.offset;
            float* half = staging + (p & 1) * piece;
            const std::size_t slice = (q.count + workers - 1) / workers;
            parallel_for(workers, workers,
                         [&](std::size_t w)
                         {
                             const std::size_t b = w * slice;
                             if (b < q.count)
                                 std::memcpy(half + b, from + b, std::min(slice, q.count - b) * sizeof(float));
                         });
            cuda_ok(cudaMemcpyAsync(dst[q.job] + q.offset, half, q.count * 4, cudaMemcpyHostToDevice, s), "H2D");
            cuda_ok(cudaEventRecord(done[p & 1], s), "cudaEventRecord");
        }
        cuda_ok(cudaStreamSynchronize(s), "PCM upload");
    }
    catch (...)
    {
        cudaStreamSynchronize(s);
        for (auto e : done)
            cudaEventDestroy(e);
        throw;
    }
    for (auto e : done)
        cudaEventDestroy(e);
}

// padded_audio on the device for every recording of one variant, laid end to
// end: recording r, group g starts at PCM row base[r] + g * padded_samples.
float* padded_device(Context& ctx, const std::vector<PcmInput>& pcm,
                     const std::vector<Header>& headers, std::vector<long long>& base,
                     unsigned* error_word)
{
    auto s = ctx.stream();
    long long rows = 0;
    base.clear();
    for (const auto& h : headers)
    {
        base.push_back(rows);
        rows += static_cast<long long>(h.groups) * static_cast<long long>(h.samples_per_channel());
    }
    const unsigned mc = headers.empty() ? 1 : headers[0].model_channels;
    float* out = ctx.workspace().get<float>("pcm_padded", static_cast<std::size_t>(rows) * mc + 1);
    // Host views are copied into one staging area (interleaved, contiguous),
    // then regrouped on the device.
    std::size_t staged_floats = 0;
    for (const auto& p : pcm)
        if (!p.device)
            staged_floats += p.samples * p.channels;
    float* staging = staged_floats ? ctx.workspace().get<float>("pcm_staging", staged_floats) : nullptr;
    std::vector<std::vector<float>> packed(pcm.size());
    std::vector<const float*> up_src;
    std::vector<float*> up_dst;
    std::vector<std::size_t> up_count;
    std::vector<const float*> src(pcm.size());
    std::vector<long long> cstride(pcm.size()), sstride(pcm.size());
    std::size_t at = 0;
    for (std::size_t r = 0; r < pcm.size(); ++r)
    {
        const auto& p = pcm[r];
        src[r] = p.data;
        cstride[r] = p.channel_stride;
        sstride[r] = p.sample_stride;
        if (!p.device && p.samples)
        {
            const float* host = p.data;
            if (!(p.channel_stride == 1 && p.sample_stride == static_cast<long long>(p.channels)))
            {
                packed[r].resize(p.samples * p.channels);
                for (std::size_t f = 0; f < p.samples; ++f)
                    for (std::size_t c = 0; c < p.channels; ++c)
                        packed[r][f * p.channels + c] =
                            p.data[static_cast<std::ptrdiff_t>(c) * p.channel_stride +
                                   static_cast<std::ptrdiff_t>(f) * p.sample_stride];
                host = packed[r].data();
            }
            up_src.push_back(host);
            up_dst.push_back(staging + at);
            up_count.push_back(p.samples * p.channels);
            src[r] = staging + at;
            at += p.samples * p.channels;
            cstride[r] = 1;
            sstride[r] = static_cast<long long>(p.channels);
        }
    }
    upload_pcm(ctx, up_src, up_dst, up_count);
    for (std::size_t r = 0; r < pcm.size(); ++r)
    {
        const auto& p = pcm[r];
        const auto& h = headers[r];
        dev::pcm_regroup(src[r], static_cast<long long>(p.samples), cstride[r], sstride[r], h.groups, mc,
                         static_cast<long long>(h.samples_per_channel()), out + base[r] * mc, error_word, s);
    }
    return out;
}

// Receptive-field half-width of one latent frame in the analysis, in frames:
// every intermediate value a latent frame depends on lies within 4,026 PCM
// samples of it (the entry convolution, the three residual units and the
// strided convolution of each stage, and the exit convolution), under 8
// frames of 512 samples.  This is also the chunk context of analysis windows
// (8 frames before, 9 after: src/common/audio_pipeline.hpp:46).
constexpr std::size_t analysis_reach = 8;

// Exact recomputation for the certified fast analysis.  Frame f of a window
// [left, right) whose RVQ margin was too small is recomputed with the exact
// kernels on the sub-window [max(left, f - 8), min(right, f + 9)): each
// output of the exact convolution depends only on its own inputs, the
// sub-window shares the window's edges where it reaches them, and elsewhere
// the padding it introduces reaches at most 8 frames inwards, so f's latent
// is bit-identical to the window's exact latent; the exact RVQ of it gives
// the reference's tokens.  Overlapping sub-windows of a window are merged.
void fast_analysis_recompute(Context& ctx, const float* padded, const std::vector<long long>& base,
                             const std::vector<Header>& headers, const std::vector<Window>& windows,
                             std::size_t w0, std::size_t wn, const std::vector<unsigned char>& uncertain,
                             int books, std::vector<std::uint16_t>& host_tok)
{
    struct Run
    {
        std::size_t window, left, right; // frames [left, right) of the recording
        std::vector<std::size_t> frames; // uncertain frames inside, ascending
    };
    std::vector<Run> runs;
    std::vector<std::size_t> token_rows; // central index of each recomputed frame
    std::size_t cen = 0, flagged = 0;
    for (std::size_t i = 0; i < wn; ++i)
    {
        const auto& c = windows[w0 + i].chunk;
        for (std::size_t k = 0; k < c.count; ++k)
        {
            if (!uncertain[cen + k])
                continue;
            ++flagged;
            const std::size_t f = c.begin + k;
            const std::size_t lo = std::max(c.left, f >= analysis_reach ? f - analysis_reach : 0);
            const std::size_t hi = std::min(c.right, f + analysis_reach + 1);
            if (!runs.empty() && runs.back().window == i && lo <= runs.back().right)
                runs.back().right = std::max(runs.back().right, hi);
            else
                runs.push_back({i, lo, hi, {}});
            runs.back().frames.push_back(f);
            token_rows.push_back(cen + k);
        }
        cen += c.count;
    }
    ctx.note_fast_analysis(cen, flagged, 0);
    if (runs.empty())
        return;
    std::vector<int> frames;
    std::vector<long long> offsets;
    std::size_t total = 0;
    for (const auto& r : runs)
    {
        const auto& w = windows[w0 + r.window];
        const auto& h = headers[w.recording];
        frames.push_back(static_cast<int>(r.right - r.left));
        offsets.push_back(base[w.recording] +
                          static_cast<long long>(w.group * h.samples_per_channel() + r.left * 512));
        total += r.right - r.left;
    }
    ctx.note_fast_analysis(0, 0, total);
    auto s = ctx.stream();
    auto& dac = ctx.analysis(headers[0].model_channels);
    auto& rvq = ctx.rvq(headers[0].model_channels);
    auto& ws = ctx.workspace();
    float* d_latent = ws.get<float>("fix_latent", total * 1024);
    float* d_frames = ws.get<float>("fix_frames", token_rows.size() * 1024);
    auto* d_tok = ws.get<std::uint16_t>("fix_tokens", token_rows.size() * static_cast<std::size_t>(books));
    dac.analyze(padded, offsets, frames, d_latent, false);
    std::size_t at = 0, row = 0;
    for (const auto& r : runs)
    {
        for (const auto f : r.frames)
            cuda_ok(cudaMemcpyAsync(d_frames + (row++) * 1024, d_latent + (at + f - r.left) * 1024, 1024 * 4,
                                    cudaMemcpyDeviceToDevice, s),
                    "D2D");
        at += r.right - r.left;
    }
    rvq.encode(d_frames, static_cast<int>(token_rows.size()), books, d_tok, books);
    std::vector<std::uint16_t> fixed(token_rows.size() * static_cast<std::size_t>(books));
    cuda_ok(cudaMemcpyAsync(fixed.data(), d_tok, fixed.size() * 2, cudaMemcpyDeviceToHost, s), "D2H");
    check_word(s, dac.error_word(), "nonfinite DSP value");
    check_word(s, rvq.error_word(), "nonfinite RVQ residual");
    for (std::size_t j = 0; j < token_rows.size(); ++j)
        std::copy_n(fixed.data() + j * books, books, host_tok.data() + token_rows[j] * books);
}

// DAC analysis + RVQ for every recording of one model variant.
void analyze_recordings(Context& ctx, const std::vector<PcmInput>& pcm,
                        const std::vector<Header>& headers,
                        std::vector<std::vector<std::uint16_t>>& tokens, Profile& profile)
{
    if (headers.empty())
        return;
    const unsigned mc = headers[0].model_channels;
    auto& dac = ctx.analysis(mc);
    auto& rvq = ctx.rvq(mc);
    auto s = ctx.stream();
    std::vector<long long> base;
    auto padded = padded_device(ctx, pcm, headers, base, dac.error_word());
    check_word(s, dac.error_word(), "nonfinite PCM sample");
    profile.mark("pcm upload/pad");
    const auto chunk_frames = audio_chunk_frames(400, ctx.limits());
    std::vector<Window> windows;
    for (std::size_t r = 0; r < headers.size(); ++r)
    {
        tokens[r].assign(headers[r].symbol_count(), 0);
        for (std::size_t g = 0; g < headers[r].groups; ++g)
            for (std::size_t b = 0; b < headers[r].frames;)
            {
                const auto c = audio_chunk(b, headers[r].frames, chunk_frames, 8, 9);
                windows.push_back({r, g, c});
                b += c.count;
            }
    }
    const float margin = ctx.fast_analysis_margin();
    for (std::size_t w0 = 0; w0 < windows.size(); w0 += window_group)
    {
        const auto wn = std::min(window_group, windows.size() - w0);
        std::vector<int> frames;
        std::vector<long long> offsets;
        std::size_t latent_frames = 0, central = 0;
        for (std::size_t i = 0; i < wn; ++i)
        {
            const auto& w = windows[w0 + i];
            const auto& h = headers[w.recording];
            frames.push_back(static_cast<int>(w.chunk.right - w.chunk.left));
            offsets.push_back(base[w.recording] +
                              static_cast<long long>(w.group * h.samples_per_channel() +
                                                     w.chunk.left * 512));
            latent_frames += w.chunk.right - w.chunk.left;
            central += w.chunk.count;
        }
        auto& ws = ctx.workspace();
        float* d_latent = ws.get<float>("enc_latent", latent_frames * 1024);
        float* d_central = ws.get<float>("enc_central", central * 1024);
        const int books = headers[0].codebooks;
        auto* d_tok = ws.get<std::uint16_t>("enc_tokens", central * static_cast<std::size_t>(books));
        std::vector<std::uint16_t> host_tok(central * static_cast<std::size_t>(books));
        // Exact analysis (the reference's arithmetic), or the certified fast
        // analysis: fused multiply-add convolutions, RVQ with the winning
        // margin of every decision, and exact recomputation of every frame
        // whose margin is below `margin` (fast_analysis_recompute).
        bool fast = margin > 0.0f;
        for (int attempt = 0; attempt < 2; ++attempt)
        {
            dac.analyze(padded, offsets, frames, d_latent, fast);
            // Keep each window's central latents (src/common/audio_pipeline.hpp:49-56).
            std::size_t lat = 0, cen = 0;
            for (std::size_t i = 0; i < wn; ++i)
            {
                const auto& c = windows[w0 + i].chunk;
                cuda_ok(cudaMemcpyAsync(d_central + cen * 1024, d_latent + (lat + c.begin - c.left) * 1024,
                                        c.count * 1024 * 4, cudaMemcpyDeviceToDevice, s),
                        "D2D");
                lat += c.right - c.left;
                cen += c.count;
            }
            profile.mark(fast ? "dac analysis (fast)" : "dac analysis");
            std::vector<unsigned char> uncertain;
            if (fast)
            {
                auto* d_flags = ws.get<unsigned char>("enc_uncertain", central);
                rvq.encode_margins(d_central, static_cast<int>(central), books, d_tok, books, margin, d_flags);
                uncertain.resize(central);
                cuda_ok(cudaMemcpyAsync(uncertain.data(), d_flags, central, cudaMemcpyDeviceToHost, s), "D2H");
            }
            else
            {
                rvq.encode(d_central, static_cast<int>(central), books, d_tok, books);
            }
            cuda_ok(cudaMemcpyAsync(host_tok.data(), d_tok, host_tok.size() * 2, cudaMemcpyDeviceToHost, s),
                    "D2H");
            unsigned words[2] = {0, 0};
            cuda_ok(cudaMemcpyAsync(&words[0], dac.error_word(), 4, cudaMemcpyDeviceToHost, s), "D2H");
            cuda_ok(cudaMemcpyAsync(&words[1], rvq.error_word(), 4, cudaMemcpyDeviceToHost, s), "D2H");
            cuda_ok(cudaStreamSynchronize(s), "analysis");
            if (fast && (words[0] || words[1]))
            {
                // A nonfinite value on the fast path: redo the group exactly, so
                // that the outcome (a stream or the reference's error) is the
                // exact path's.
                cuda_ok(cudaMemsetAsync(dac.error_word(), 0, 4, s), "memset");
                cuda_ok(cudaMemsetAsync(rvq.error_word(), 0, 4, s), "memset");
                fast = false;
                continue;
            }
            check_word(s, dac.error_word(), "nonfinite DSP value");
            check_word(s, rvq.error_word(), "nonfinite RVQ residual");
            if (fast)
                fast_analysis_recompute(ctx, padded, base, headers, windows, w0, wn, uncertain, books, host_tok);
            break;
        }
        profile.mark("rvq encode");
        // store_tokens (src/common/audio_analyzer.cpp:164-172).
        std::size_t cen = 0;
        for (std::size_t i = 0; i < wn; ++i)
        {
            const auto& w = windows[w0 + i];
            const auto& h = headers[w.recording];
            for (std::size_t f = 0; f < w.chunk.count; ++f)
                std::copy_n(host_tok.data() + (cen + f) * books, books,
                            tokens[w.recording].data() +
                                ((w.chunk.begin + f) * h.groups + w.group) * h.codebooks);
            cen += w.chunk.count;
        }
    }
}

Bytes range_code(const Header& h, std::span<const std::uint16_t> tok, const std::uint16_t* q,
                 const Limits& limits, std::size_t* bits, std::size_t* book_bits = nullptr,
                 std::uint32_t* symbol_bits = nullptr)
{
    require(limits.file_bytes >= 19, "normal framing exceeds file limit");
    RangeWriter encoder(limits.file_bytes - 18);
    const bool observed = book_bits || symbol_bits;
    std::size_t index = 0;
    for_each_entropy_position(h,
                            [&](const EntropyPosition& p)
                            {
                                // Bits of one symbol: the encoder's bit position
                                // difference (EntropyObserver::after_symbol,
                                // src/format/entropy.cpp:93-98).
                                const auto before = observed ? encoder.bit_position() : 0;
                                const unsigned token = tok[p.token_offset];
                                const auto* path = q + p.token_offset * 10;
                                for (int d = 0; d < 10; ++d)
                                    encoder.put(path[d], (token >> (9 - d)) & 1u);
                                const auto used = observed ? encoder.bit_position() - before : 0;
                                if (book_bits)
                                    book_bits[p.codebook] += used;
                                if (symbol_bits)
                                    symbol_bits[index++] = static_cast<std::uint32_t>(used);
                            });
    if (bits)
        *bits = encoder.bit_position();
    const auto payload = encoder.finish();
    return normal_stream(h, payload);
}
} // namespace

Header audio_header(const PcmInput& pcm, const EncodeOptions& options, const Limits& limits)
{
    const auto channels = pcm.channels, samples = pcm.samples;
    require(channels > 0 && channels <= 127, "invalid PCM channel count");
    require(pcm.channel_stride > 0 && pcm.sample_stride > 0, "invalid PCM strides");
    require(samples == 0 || pcm.data != nullptr, "null PCM data");
    require(checked_mul(samples, channels) <= limits.tensor_elements, "PCM exceeds element limit");
    require(options.method == 0 || options.method == 1, "invalid coding method");
    Header header;
    header.method = static_cast<std::uint8_t>(options.method);
    header.model_channels = channels == 2 && !options.separate_channels ? 2 : 1;
    header.groups = static_cast<std::uint8_t>(channels / header.model_channels);
    const unsigned maximum = header.model_channels == 2 ? 12 : 9;
    require(options.codebooks <= maximum, "invalid number of codebooks for audio model");
    header.codebooks = static_cast<std::uint8_t>(options.codebooks ? options.codebooks : maximum);
    header.frames = checked_add(samples, 511) / 512;
    require(options.entropy_batch >= 0 && options.entropy_batch <= 65535, "invalid entropy batch size");
    require(header.method == 1 || options.entropy_batch == 0, "entropy batch requires normal coding");
    if (header.method == 1)
    {
        header.batch = select_entropy_batch(header.frames, options.entropy_batch);
    }
    check_header(header, limits);
    require(checked_mul(header.samples_per_channel(), channels) <= limits.tensor_elements,
            "padded PCM exceeds element limit");
    return header;
}

std::vector<std::uint16_t> analyze_tokens(Context& ctx, const PcmInput& pcm,
                                          const EncodeOptions& options, Header* header_out)
{
    ctx.bind();
    Profile profile(ctx.stream(), "analyze");
    const auto header = audio_header(pcm, options, ctx.limits());
    std::vector<std::vector<std::uint16_t>> tokens(1);
    analyze_recordings(ctx, {pcm}, {header}, tokens, profile);
    if (header_out)
        *header_out = header;
    return std::move(tokens[0]);
}

Bytes pack_normal(Context& ctx, Header header, std::span<const std::uint16_t> tokens,
                  std::size_t* bits)
{
    ctx.bind();
    header.method = 1;
    check_header(header, ctx.limits());
    require(header.frames <= 0xffffffffu, "normal frame count exceeds uint32");
    require(tokens.size() == header.symbol_count(), "normal token count does not match header");
    header.token_crc = token_crc32(tokens);
    std::vector<std::uint16_t> q(header.symbol_count() * 10);
    ctx.transformer(header.model_channels).predict_known(header, tokens, q.data(), nullptr);
    return range_code(header, tokens, q.data(), ctx.limits(), bits);
}

std::vector<Bytes> encode_batch(Context& ctx, const std::vector<PcmInput>& pcm,
                                const EncodeOptions& options, std::vector<std::size_t>* bits,
                                std::vector<std::vector<std::size_t>>* book_bits,
                                std::vector<std::vector<std::uint32_t>>* symbol_bits)
{
    ctx.bind();
    Profile profile(ctx.stream(), "encode");
    const auto n = pcm.size();
    std::vector<Header> headers(n);
    for (std::size_t i = 0; i < n; ++i)
        headers[i] = audio_header(pcm[i], options, ctx.limits());
    std::vector<std::vector<std::uint16_t>> tokens(n);
    for (unsigned mc : {1u, 2u})
    {
        std::vector<std::size_t> ids;
        std::vector<PcmInput> p;
        std::vector<Header> h;
        for (std::size_t i = 0; i < n; ++i)
            if (headers[i].model_channels == mc)
            {
                ids.push_back(i);
                p.push_back(pcm[i]);
                h.push_back(headers[i]);
            }
        std::vector<std::vector<std::uint16_t>> t(ids.size());
        analyze_recordings(ctx, p, h, t, profile);
        for (std::size_t j = 0; j < ids.size(); ++j)
            tokens[ids[j]] = std::move(t[j]);
    }
    std::vector<Bytes> out(n);
    if (bits)
        bits->assign(n, 0);
    if (book_bits)
    {
        book_bits->assign(n, {});
        for (std::size_t i = 0; i < n; ++i)
            (*book_bits)[i].assign(headers[i].codebooks, 0);
    }
    if (symbol_bits)
    {
        symbol_bits->assign(n, {});
        for (std::size_t i = 0; i < n; ++i)
            if (headers[i].method == 1)
                (*symbol_bits)[i].assign(headers[i].symbol_count(), 0);
    }
    std::vector<std::vector<std::uint16_t>> q15(n);
    for (std::size_t i = 0; i < n; ++i)
    {
        if (headers[i].method == 0)
        {
            out[i] = fast_stream(headers[i], tokens[i], ctx.limits());
            continue;
        }
        headers[i].token_crc = token_crc32(tokens[i]);
        q15[i].resize(headers[i].symbol_count() * 10);
        ctx.transformer(headers[i].model_channels)
            .predict_known(headers[i], tokens[i], q15[i].data(), nullptr);
    }
    profile.mark("transformer (known)");
    // Sequential range coding per recording on host cores (pack_normal,
    // src/format/entropy.cpp:57-123), recordings in parallel.
    parallel_for(n, host_workers(ctx),
                 [&](std::size_t i)
                 {
                     if (headers[i].method == 1)
                         out[i] = range_code(headers[i], tokens[i], q15[i].data(), ctx.limits(),
                                             bits ? &(*bits)[i] : nullptr,
                                             book_bits ? (*book_bits)[i].data() : nullptr,
                                             symbol_bits ? (*symbol_bits)[i].data() : nullptr);
                 });
    profile.mark("range encode");
    return out;
}

namespace
{
// Decoded PCM, device -> host.  Pageable copies into fresh host buffers run
// on one driver thread that also takes every first-touch page fault (about
// 2 GB/s measured); here 32 MiB pieces go by DMA into one half of a pinned
// double buffer while the host workers move the previous piece into place.
void download_pcm(Context& ctx, const std::vector<Header>& headers, const std::vector<float*>& src,
                  const std::vector<float*>& dst)
{
    constexpr std::size_t piece = std::size_t{8} << 20; // floats (32 MiB)
    auto s = ctx.stream();
    struct Piece
    {
        std::size_t recording, offset, count;
    };
    std::vector<Piece> pieces;
    std::size_t total = 0;
    for (std::size_t i = 0; i < headers.size(); ++i)
    {
        const auto count = headers[i].channels() * headers[i].samples_per_channel();
        total += count;
        for (std::size_t at = 0; at < count; at += piece)
            pieces.push_back({i, at, std::min(piece, count - at)});
    }
    if (total < piece / 4)
    {
        for (std::size_t i = 0; i < headers.size(); ++i)
            cuda_ok(cudaMemcpyAsync(dst[i], src[i], headers[i].channels() * headers[i].samples_per_channel() * 4,
                                    cudaMemcpyDeviceToHost, s),
                    "D2H");
        cuda_ok(cudaStreamSynchronize(s), "decode");
        return;
    }
    float* staging = ctx.pinned_staging(piece);
    cudaEvent_t done[2] = {nullptr, nullptr};
    for (auto& e : done)
        cuda_ok(cudaEventCreateWithFlags(&e, cudaEventDisableTiming), "cudaEventCreate");
    const auto issue = [&](std::size_t p)
    {
        const auto& q = pieces[p];
        cuda_ok(cudaMemcpyAsync(staging + (p & 1) * piece, src[q.recording] + q.offset, q.count * 4,
                                cudaMemcpyDeviceToHost, s),
                "D2H");
        cuda_ok(cudaEventRecord(done[p & 1], s), "cudaEventRecord");
    };
    const std::size_t workers = copy_workers(ctx);
    try
    {
        issue(0);
        for (std::size_t p = 0; p < pieces.size(); ++p)
        {
            // The other half held piece p - 1, already moved into place.
            if (p + 1 < pieces.size())
                issue(p + 1);
            cuda_ok(cudaEventSynchronize(done[p & 1]), "D2H");
            const auto& q = pieces[p];
            const float* from = staging + (p & 1) * piece;
            float* to = dst[q.recording] + q.offset;
            const std::size_t slice = (q.count + workers - 1) / workers;
            parallel_for(workers, workers,
                         [&](std::size_t w)
                         {
                             const std::size_t b = w * slice;
                             if (b < q.count)
                                 std::memcpy(to + b, from + b, std::min(slice, q.count - b) * sizeof(float));
                         });
        }
    }
    catch (...)
    {
        cudaStreamSynchronize(s);
        for (auto e : done)
            cudaEventDestroy(e);
        throw;
    }
    for (auto e : done)
        cudaEventDestroy(e);
}
} // namespace

std::vector<DecodedAudio> decode_batch(Context& ctx, const std::vector<ByteView>& streams,
                                       float* const* device_out, float* const* host_out)
{
    ctx.bind();
    Profile profile(ctx.stream(), "decode");
    const auto n = streams.size();
    std::vector<Header> headers(n);
    std::vector<std::vector<std::uint16_t>> tokens(n);
    for (std::size_t i = 0; i < n; ++i)
    {
        headers[i] = read_header(streams[i], ctx.limits());
        // allocate_pcm's limit (src/common/audio_analyzer.cpp), checked
        // before any device work rather than after the token loop.
        require(checked_mul(headers[i].channels(), headers[i].samples_per_channel()) <= ctx.limits().tensor_elements,
                "output audio exceeds element limit");
        if (headers[i].method == 0)
            tokens[i] = fast_tokens(streams[i], ctx.limits());
        else
            tokens[i].assign(headers[i].symbol_count(), 0);
    }
    // Normal streams: the whole token loop (probability model, bisection
    // masses, range decoders) runs on the GPU, one model variant at a time.
    for (unsigned mc : {1u, 2u})
    {
        std::vector<std::size_t> ids;
        std::vector<Header> hs;
        std::vector<ByteView> payloads;
        for (std::size_t i = 0; i < n; ++i)
            if (headers[i].method == 1 && headers[i].model_channels == mc)
            {
                ids.push_back(i);
                hs.push_back(headers[i]);
                payloads.push_back(streams[i].subspan(headers[i].payload_offset, headers[i].payload_bytes));
            }
        if (ids.empty())
            continue;
        std::vector<std::vector<std::uint16_t>> decoded;
        ctx.transformer(mc).decode_streams(hs, payloads, decoded);
        for (std::size_t j = 0; j < ids.size(); ++j)
        {
            check_token_crc(headers[ids[j]], decoded[j]);
            tokens[ids[j]] = std::move(decoded[j]);
        }
    }
    profile.mark("transformer + range");
    // RVQ reconstruction + DAC synthesis over chunk windows
    // (src/common/audio_pipeline.hpp:63-83, context 11/11).
    std::vector<DecodedAudio> out(n);
    std::vector<float*> dst(n);
    std::size_t host_floats = 0;
    for (std::size_t i = 0; i < n; ++i)
    {
        out[i].channels = static_cast<unsigned>(headers[i].channels());
        out[i].frames = headers[i].samples_per_channel();
        const auto count = headers[i].channels() * headers[i].samples_per_channel();
        require(count <= ctx.limits().tensor_elements, "output audio exceeds element limit");
        host_floats = checked_add(host_floats, align_up(count, 64));
    }
    // Host results are assembled in one device buffer of the context (kept
    // between calls), then copied out.
    float* assembled = device_out ? nullptr : ctx.workspace().get<float>("pcm_out", host_floats);
    for (std::size_t i = 0, at = 0; i < n; ++i)
    {
        if (device_out)
        {
            dst[i] = device_out[i];
        }
        else
        {
            dst[i] = assembled + at;
            at += align_up(headers[i].channels() * headers[i].samples_per_channel(), 64);
        }
    }
    auto s = ctx.stream();
    const auto chunk_frames = audio_chunk_frames(400, ctx.limits());
    for (unsigned mc : {1u, 2u})
    {
        std::vector<Window> windows;
        for (std::size_t i = 0; i < n; ++i)
        {
            if (headers[i].model_channels != mc)
                continue;
            for (std::size_t g = 0; g < headers[i].groups; ++g)
                for (std::size_t b = 0; b < headers[i].frames;)
                {
                    const auto c = audio_chunk(b, headers[i].frames, chunk_frames, 11, 11);
                    windows.push_back({i, g, c});
                    b += c.count;
                }
        }
        if (windows.empty())
            continue;
        auto& rvq = ctx.rvq(mc);
        auto& dac = ctx.synthesis(mc);
        for (std::size_t w0 = 0; w0 < windows.size(); w0 += window_group)
        {
            const auto wn = std::min(window_group, windows.size() - w0);
            std::vector<int> frames;
            std::size_t total = 0;
            int books = 0;
            for (std::size_t i = 0; i < wn; ++i)
            {
                const auto& c = windows[w0 + i].chunk;
                frames.push_back(static_cast<int>(c.right - c.left));
                total += c.right - c.left;
                books = std::max<int>(books, headers[windows[w0 + i].recording].codebooks);
            }
            // Window tokens [frame][books] (chunk_tokens, src/common/audio_analyzer.cpp:174-183).
            std::vector<std::uint16_t> wt(total * static_cast<std::size_t>(books), 0);
            std::size_t at = 0;
            for (std::size_t i = 0; i < wn; ++i)
            {
                const auto& w = windows[w0 + i];
                const auto& h = headers[w.recording];
                for (std::size_t f = w.chunk.left; f < w.chunk.right; ++f, ++at)
                    std::copy_n(tokens[w.recording].data() + (f * h.groups + w.group) * h.codebooks,
                                h.codebooks, wt.data() + at * books);
            }
            auto& ws = ctx.workspace();
            auto* d_tok = ws.get<std::uint16_t>("dec_tokens", wt.size());
            float* d_latent = ws.get<float>("dec_latent", total * 1024);
            float* d_pcm = ws.get<float>("dec_pcm", total * 512 * mc);
            cuda_ok(cudaMemcpyAsync(d_tok, wt.data(), wt.size() * 2,
                                    cudaMemcpyHostToDevice, s),
                    "H2D");
            std::size_t off = 0;
            for (std::size_t i = 0; i < wn;)
            {
                // Runs of windows with the same book count decode in one launch.
                std::size_t j = i, len = 0;
                const int q = headers[windows[w0 + i].recording].codebooks;
                while (j < wn && headers[windows[w0 + j].recording].codebooks == q)
                {
                    len += windows[w0 + j].chunk.right - windows[w0 + j].chunk.left;
                    ++j;
                }
                rvq.decode(d_tok + off * books, books, static_cast<int>(len), q,
                           d_latent + off * 1024);
                off += len;
                i = j;
            }
            profile.mark("rvq decode");
            dac.synthesize(d_latent, frames, d_pcm);
            // store_pcm (src/common/audio_analyzer.cpp:185-199): central samples
            // of each window into the interleaved output, channel g*mc + c.
            off = 0;
            for (std::size_t i = 0; i < wn; ++i)
            {
                const auto& w = windows[w0 + i];
                const auto channels = headers[w.recording].channels();
                cuda_ok(cudaMemcpy2DAsync(dst[w.recording] + w.chunk.begin * 512 * channels + w.group * mc,
                                          channels * 4,
                                          d_pcm + (off + (w.chunk.begin - w.chunk.left) * 512) * mc,
                                          mc * 4, mc * 4, w.chunk.count * 512,
                                          cudaMemcpyDeviceToDevice, s),
                        "D2D");
                off += (w.chunk.right - w.chunk.left) * 512;
            }
            dac.check_errors("synthesis");
            profile.mark("dac synthesis");
        }
    }
    if (!device_out)
    {
        std::vector<float*> targets(n);
        for (std::size_t i = 0; i < n; ++i)
        {
            targets[i] = host_out ? host_out[i] : nullptr;
            if (!targets[i])
            {
                out[i].samples.resize(headers[i].channels() * headers[i].samples_per_channel());
                targets[i] = out[i].samples.data();
            }
        }
        download_pcm(ctx, headers, dst, targets);
        profile.mark("pcm download");
    }
    return out;
}
} // namespace tsacb
