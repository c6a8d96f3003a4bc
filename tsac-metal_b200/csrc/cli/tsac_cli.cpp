// tsac-cuda: the TSAC command line tool on the CUDA library.
//
// Same commands, options, file formats and messages as the reference tool
// (src/main.cpp, src/cli.cpp:6-157, src/codec.cpp:112-246, src/audio.cpp):
//   tsac-cuda [options] c infile outfile   compress (.wav / .sw natively, other formats via FFmpeg)
//   tsac-cuda [options] d infile outfile   decompress to 16-bit WAVE
//   tsac-cuda [options] t infile outfile   compress, then decompress the stream to outfile
// The options keep the reference's spelling and checks; --metal is refused
// (no Metal on this platform).  Additions: --exact (bit-identical decoder PCM),
// --device n, --models DIR (package directory; default: beside the executable,
// or $TSAC_CUDA_MODELS).  The tool links only the C ABI (include/tsac_cuda.h).
#include "tsac_cuda.h"

#include <algorithm>
#include <cerrno>
#include <charconv>
#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <filesystem>
#include <fstream>
#include <iomanip>
#include <iostream>
#include <limits>
#include <spawn.h>
#include <stdexcept>
#include <string>
#include <string_view>
#include <sys/resource.h>
#include <sys/wait.h>
#include <unistd.h>
#include <vector>

extern char** environ;

namespace
{
using Bytes = std::vector<std::uint8_t>;

struct Error : std::runtime_error
{
    using std::runtime_error::runtime_error;
};

void require(bool ok, const std::string& message)
{
    if (!ok)
        throw Error(message);
}

void check(int status)
{
    if (status != TSAC_CUDA_OK)
        throw Error(tsac_cuda_last_error());
}

// ------------------------------------------------------------------ options --
struct Options
{
    bool help = false, fast = false, separate = false, exact = false;
    unsigned verbose = 0;
    int threads = 0, quality = 0, channels = 0, batch = 0, device = 0;
    char command = 0;
    std::string input, output, models;
};

// The reference's parser (src/cli.cpp:6-126): short options group ("-vv"),
// "+n" values, "--" ends options, exactly three positionals.
Options parse_cli(const std::vector<std::string_view>& arguments)
{
    Options options;
    std::vector<std::string_view> positional;
    for (std::size_t i = 0; i < arguments.size(); ++i)
    {
        const auto arg = arguments[i];
        if (arg == "--")
        {
            positional.insert(positional.end(), arguments.begin() + static_cast<std::ptrdiff_t>(i + 1),
                              arguments.end());
            break;
        }
        if (arg.size() <= 1 || arg[0] != '-')
        {
            positional.push_back(arg);
            continue;
        }
        const auto text_value = [&](std::string_view name)
        {
            if (++i == arguments.size())
                throw Error("option '" + std::string(name) + "' must have an argument");
            return std::string(arguments[i]);
        };
        const auto value = [&](std::string_view name)
        {
            if (++i == arguments.size())
                throw Error("option '" + std::string(name) + "' must have an argument");
            auto text = arguments[i];
            if (text.starts_with('+'))
                text.remove_prefix(1);
            int number = 0;
            const auto parsed = std::from_chars(text.data(), text.data() + text.size(), number);
            if (text.empty() || parsed.ec != std::errc{} || parsed.ptr != text.data() + text.size())
            {
                const auto canonical = name == "-q" ? "--n_codebooks" : name == "-c" ? "--channels" : name;
                throw Error("option " + std::string(canonical) + " expects an integer");
            }
            return number;
        };
        const auto flag = [&](std::string_view name)
        {
            if (name == "-h" || name == "--help")
                options.help = true;
            else if (name == "-f" || name == "--fast")
                options.fast = true;
            else if (name == "-s" || name == "--separate_channels")
                options.separate = true;
            else if (name == "-v")
                ++options.verbose;
            else if (name == "-T")
                options.threads = value(name);
            else if (name == "-q" || name == "--n_codebooks")
                options.quality = value(name);
            else if (name == "-c" || name == "--channels")
                options.channels = value(name);
            else if (name == "--batch_size")
                options.batch = value(name);
            else if (name == "--metal")
                throw Error("Metal execution is not available on this platform (this tool runs on CUDA)");
            else if (name == "--exact")
                options.exact = true;
            else if (name == "--device")
                options.device = value(name);
            else if (name == "--models")
                options.models = text_value(name);
            else
                throw Error("unknown option: '" + std::string(name) + "'");
        };
        if (arg.starts_with("--"))
        {
            flag(arg);
        }
        else
        {
            // Validate the whole short-option group before consuming values:
            // -q1 is an unknown -1 option, not an attached value.
            for (const char character : arg.substr(1))
                if (std::string_view("hfsvTqc").find(character) == std::string_view::npos)
                    throw Error("unknown option: '-" + std::string(1, character) + "'");
            for (std::size_t character = 1; character < arg.size(); ++character)
                flag(std::string("-") + arg[character]);
        }
        if (options.help)
            return options;
    }
    if (positional.size() != 3)
    {
        options.help = true;
        return options;
    }
    if (positional[0] != "c" && positional[0] != "d" && positional[0] != "t")
        throw Error("unknown command: " + std::string(positional[0]));
    options.command = positional[0][0];
    options.input = positional[1];
    options.output = positional[2];
    return options;
}

const char* help_text()
{
    return R"(TSAC for NVIDIA Blackwell (CUDA)

Very low bitrate audio compression

usage: tsac-cuda [options] c infile outfile     audio compression
                           d infile outfile     audio decompression
                           t infile outfile     audio compression then decompression to outfile
Uncompressed wave (.wav) and raw audio (.sw) are natively supported as input files.
FFmpeg is invoked to support other audio formats. Decompression outputs WAVE.
Weights load from the package directory beside the executable (or --models DIR,
or $TSAC_CUDA_MODELS).

Available options:
-h --help               show the help
-T n                    number of host threads for range coding (default: automatic)
-q --n_codebooks n      quality (1-12 for joint stereo, 1-9 otherwise; 0=max)
-s --separate_channels  encode stereo as separate channels
-c --channels n         force input channels through FFmpeg
-f --fast               disable the transformer model
--batch_size n          force the entropy batch size (default=auto)
-v                      display statistics
--exact                 decode with the reference's serial arithmetic (bit-identical PCM)
--device n              CUDA device (default 0)
--models DIR            weight package directory
)";
}

// -------------------------------------------------------------------- files --
Bytes read_file(const std::filesystem::path& path)
{
    std::ifstream in(path, std::ios::binary);
    if (!in)
        throw Error(path.string() + ": cannot open file");
    return Bytes(std::istreambuf_iterator<char>(in), std::istreambuf_iterator<char>());
}

void write_file(const std::filesystem::path& path, const Bytes& bytes)
{
    std::ofstream out(path, std::ios::binary);
    if (!out)
        throw Error(path.string() + ": cannot create file");
    out.write(reinterpret_cast<const char*>(bytes.data()), static_cast<std::streamsize>(bytes.size()));
    if (!out)
        throw Error(path.string() + ": write failed");
}

// -------------------------------------------------------------------- audio --
// Interleaved float PCM [frame][channel] padded with zeros to 512 frames.
struct Audio
{
    unsigned channels = 0;
    std::vector<float> samples;
};

std::uint32_t le32(const Bytes& b, std::size_t at)
{
    require(at + 4 <= b.size(), "invalid wav file");
    return std::uint32_t(b[at]) | (std::uint32_t(b[at + 1]) << 8) | (std::uint32_t(b[at + 2]) << 16) |
           (std::uint32_t(b[at + 3]) << 24);
}

// Raw little-endian PCM16 (pcm16_input, src/audio.cpp:19-37): an incomplete
// interleaved frame is discarded; value / 32768.
Audio pcm16_input(const std::uint8_t* data, std::size_t bytes, unsigned channels)
{
    require(channels > 0 && channels <= 127, "unsupported number of channels");
    const std::size_t frames = bytes / (2 * channels);
    const std::size_t padded = (frames + 511) / 512 * 512;
    Audio audio{channels, std::vector<float>(padded * channels, 0.0f)};
    for (std::size_t i = 0; i < frames * channels; ++i)
    {
        const unsigned value = unsigned(data[2 * i]) | (unsigned(data[2 * i + 1]) << 8);
        const int signed_value = value < 32768 ? static_cast<int>(value) : static_cast<int>(value) - 65536;
        audio.samples[i] = static_cast<float>(signed_value) * (1.0f / 32768.0f);
    }
    return audio;
}

// Native RIFF/WAVE reader (wave_input, src/audio.cpp:39-73): PCM16 at
// 44.1 kHz, 1..8 channels, data read to the end of the file.
Audio wave_input(const Bytes& bytes)
{
    const auto tag = [&](std::size_t at, const char* text)
    { return at + 4 <= bytes.size() && std::memcmp(bytes.data() + at, text, 4) == 0; };
    require(tag(0, "RIFF") && tag(8, "WAVE"), "invalid wav file");
    unsigned channels = 0;
    for (std::size_t offset = 12; offset < bytes.size();)
    {
        const std::size_t length = le32(bytes, offset + 4);
        const std::size_t payload = offset + 8;
        if (tag(offset, "fmt "))
        {
            require(length >= 16 && payload + length <= bytes.size(), "invalid wav file");
            const auto* fmt = bytes.data() + payload;
            require(fmt[0] == 1 && fmt[1] == 0 && fmt[14] == 16 && fmt[15] == 0, "invalid wav file");
            channels = unsigned(fmt[2]) | (unsigned(fmt[3]) << 8);
            require(channels > 0 && channels <= 8, "unsupported number of channels");
            require(le32(bytes, payload + 4) == 44100, "the sample rate must be 44100 Hz");
        }
        else if (tag(offset, "data"))
        {
            require(channels > 0, "invalid wav file");
            return pcm16_input(bytes.data() + payload, bytes.size() - std::min(bytes.size(), payload), channels);
        }
        require(payload + length <= bytes.size(), "invalid wav file");
        offset = payload + length;
    }
    throw Error("invalid wav file");
}

// Other formats (and forced channel counts) through FFmpeg, spawned with an
// argument vector, never a shell (read_audio, src/audio.cpp:98-163).
Audio read_audio(const std::filesystem::path& path, int requested_channels)
{
    require(requested_channels >= 0 && requested_channels <= 127, "unsupported number of channels");
    if (path.extension() == ".sw")
    {
        const auto bytes = read_file(path);
        return pcm16_input(bytes.data(), bytes.size(),
                           requested_channels ? static_cast<unsigned>(requested_channels) : 1);
    }
    if (path.extension() == ".wav" && requested_channels == 0)
    {
        try
        {
            return wave_input(read_file(path));
        }
        catch (const Error& error)
        {
            throw Error(path.string() + ": " + error.what());
        }
    }
    char pattern[] = "/tmp/tsac-audio-XXXXXX";
    require(mkdtemp(pattern) != nullptr, "cannot create audio conversion directory");
    const std::filesystem::path directory(pattern);
    const auto converted = directory / "converted.wav";
    std::vector<std::string> arguments{"ffmpeg", "-i", std::filesystem::absolute(path).string(), "-y",
                                       "-loglevel", "error", "-ar", "44100", "-acodec", "pcm_s16le"};
    if (requested_channels)
        arguments.insert(arguments.end(), {"-ac", std::to_string(requested_channels)});
    arguments.push_back(converted.string());
    std::vector<char*> argv;
    for (auto& argument : arguments)
        argv.push_back(argument.data());
    argv.push_back(nullptr);
    pid_t child;
    const int error = posix_spawnp(&child, "ffmpeg", nullptr, nullptr, argv.data(), environ);
    Audio audio;
    bool ok = error == 0;
    if (ok)
    {
        int status = 0;
        pid_t waited;
        do
            waited = waitpid(child, &status, 0);
        while (waited == -1 && errno == EINTR);
        ok = waited != -1 && WIFEXITED(status) && WEXITSTATUS(status) == 0;
        if (ok)
            audio = wave_input(read_file(converted));
    }
    std::error_code ignored;
    std::filesystem::remove_all(directory, ignored);
    if (error)
        throw Error("Error while trying to run FFmpeg: " + std::string(std::strerror(error)));
    require(ok, "Error while trying to run FFmpeg");
    return audio;
}

// 16-bit WAVE writer (pcm16_wave, src/audio.cpp:198-246): samples scaled by
// 32768, clipped, rounded to nearest with ties to even; all padded samples kept.
Bytes pcm16_wave(const std::vector<float>& samples, unsigned channels)
{
    require(channels > 0 && samples.size() % channels == 0, "audio sample shape mismatch");
    const std::size_t block = 2ull * channels, rate = block * 44100, bytes = samples.size() * 2;
    require(block <= 0xffff && rate <= 0xffffffffull && bytes <= 0xffffffffull - 36,
            "audio exceeds RIFF/WAVE dimensions");
    Bytes out;
    out.reserve(bytes + 44);
    const auto word = [&](std::size_t value, unsigned count)
    {
        for (unsigned i = 0; i < count; ++i)
            out.push_back(static_cast<std::uint8_t>((value >> (8 * i)) & 255));
    };
    const auto tag = [&](const char* text) { out.insert(out.end(), text, text + 4); };
    tag("RIFF");
    word(bytes + 36, 4);
    tag("WAVE");
    tag("fmt ");
    word(16, 4);
    word(1, 2);
    word(channels, 2);
    word(44100, 4);
    word(rate, 4);
    word(block, 2);
    word(16, 2);
    tag("data");
    word(bytes, 4);
    for (const float x : samples)
    {
        require(std::isfinite(x), "nonfinite audio sample");
        const double scaled = std::clamp(double(x) * 32768.0, -32768.0, 32767.0);
        const double lower = std::floor(scaled);
        const auto integer = static_cast<std::int32_t>(lower);
        const double fraction = scaled - lower;
        const auto rounded = integer + ((fraction > 0.5 || (fraction == 0.5 && integer % 2 != 0)) ? 1 : 0);
        word(static_cast<std::uint16_t>(rounded), 2);
    }
    return out;
}

// -------------------------------------------------------------------- codec --
std::filesystem::path default_models()
{
    if (const char* env = std::getenv("TSAC_CUDA_MODELS"))
        return env;
    std::error_code error;
    const auto exe = std::filesystem::read_symlink("/proc/self/exe", error);
    require(!error, "cannot locate executable directory");
    return exe.parent_path();
}

double peak_memory_gb()
{
    rusage usage{};
    // Linux reports ru_maxrss in kilobytes.
    return getrusage(RUSAGE_SELF, &usage) == 0 ? double(usage.ru_maxrss) * 1024.0 / 1e9 : 0.0;
}

tsac_cuda_stream_header header_of(const Bytes& stream)
{
    tsac_cuda_stream_header h{};
    check(tsac_cuda_stream_header_info(stream.data(), stream.size(), &h));
    return h;
}

// EntropyProgress (src/codec.cpp:41-110): the header line, the progress
// percentage (the GPU codes a whole recording at once, so it reaches 100%
// in one step) and, at -vv, the average bits per codebook.
void print_header_line(const tsac_cuda_stream_header& h)
{
    const auto block_len = h.frames / h.batch + (h.frames % h.batch != 0);
    std::cout << "batch_size=" << h.batch << " bs=" << h.groups << " n_cb=" << h.codebooks
              << " block_len=" << block_len << '\n';
    std::cout << (h.frames * h.groups * h.codebooks != 0 ? "100%\n" : "\n");
}

struct Context
{
    tsac_cuda_context* ctx = nullptr;
    ~Context()
    {
        if (ctx)
            tsac_cuda_context_destroy(ctx);
    }
};

Bytes compress(Context& c, const Options& options, std::size_t& frames, unsigned& channels)
{
    const auto audio = read_audio(options.input, options.channels);
    require(options.quality >= 0, "invalid number of codebooks");
    tsac_cuda_encode_options encode{};
    encode.method = options.fast ? 0 : 1;
    encode.codebooks = static_cast<unsigned>(options.quality);
    encode.separate_channels = options.separate ? 1 : 0;
    encode.entropy_batch = 0;
    if (!options.fast && options.batch)
    {
        require(options.batch > 0 && options.batch <= 65535, "invalid entropy batch size");
        encode.entropy_batch = static_cast<unsigned>(options.batch);
    }
    std::uint8_t* out = nullptr;
    std::size_t bytes = 0;
    std::uint64_t book_bits[12] = {};
    const std::size_t samples = audio.samples.size() / audio.channels;
    check(tsac_cuda_encode_observed(c.ctx, audio.samples.data(), audio.channels, samples, 1,
                                    static_cast<std::ptrdiff_t>(audio.channels), &encode, &out,
                                    &bytes, book_bits, 12));
    Bytes stream(out, out + bytes);
    tsac_cuda_free(out);
    const auto h = header_of(stream);
    frames = h.frames;
    channels = h.model_channels * h.groups;
    if (options.verbose && h.method == 1)
    {
        print_header_line(h);
        if (options.verbose >= 2)
        {
            std::cout << "CB AVG_BITS\n";
            const auto count = h.frames * h.groups;
            for (unsigned book = 0; book < h.codebooks; ++book)
                std::cout << std::setw(2) << book << ' ' << std::fixed << std::setprecision(3)
                          << std::setw(7) << (count ? double(book_bits[book]) / double(count) : 0.0)
                          << '\n';
        }
    }
    return stream;
}

Bytes decompress(Context& c, const Bytes& stream, const Options& options)
{
    const auto h = header_of(stream);
    if (options.verbose && h.method == 1)
        print_header_line(h);
    float* out = nullptr;
    std::size_t samples = 0;
    unsigned channels = 0;
    check(tsac_cuda_decode(c.ctx, stream.data(), stream.size(), &out, &samples, &channels));
    std::vector<float> pcm(out, out + samples);
    tsac_cuda_free(out);
    return pcm16_wave(pcm, channels);
}

int run(const Options& options)
{
    // The reference's analyzer rejects a thread budget above 256 when it is
    // constructed, before any file is read (src/apple-arm/audio_analyzer.cpp:93).
    if (options.threads > 256)
        throw Error("CPU thread count exceeds supported limit (256)");
    Context c;
    const auto models = options.models.empty() ? default_models() : std::filesystem::path(options.models);
    check(tsac_cuda_context_create(models.c_str(), options.device, &c.ctx));
    if (options.exact)
        check(tsac_cuda_set_exact_synthesis(c.ctx, 1));
    // The reference passes a positive -T to its analyzer and uses the default
    // otherwise (src/codec.cpp:117-120).
    if (options.threads > 0)
        check(tsac_cuda_set_host_threads(c.ctx, static_cast<unsigned>(options.threads)));
    Bytes output;
    if (options.command == 'c' || options.command == 't')
    {
        std::size_t frames = 0;
        unsigned channels = 0;
        output = compress(c, options, frames, channels);
        if (options.verbose)
        {
            const double kbps = frames ? double(output.size()) * 8.0 * 44100.0 / (double(frames) * 512.0 * 1000.0) : 0.0;
            std::cout << std::fixed << std::setprecision(2) << "bitrate=" << kbps
                      << " kb/s, max_memory=" << peak_memory_gb() << " GB\n";
        }
        if (options.command == 't')
            output = decompress(c, output, options);
    }
    else
    {
        output = decompress(c, read_file(options.input), options);
    }
    write_file(options.output, output);
    return 0;
}
} // namespace

int main(int argc, char** argv)
{
    try
    {
        std::vector<std::string_view> arguments;
        for (int i = 1; i < argc; ++i)
            arguments.emplace_back(argv[i]);
        const auto options = parse_cli(arguments);
        if (options.help)
        {
            std::cout << help_text();
            return 1;
        }
        return run(options);
    }
    catch (const std::exception& error)
    {
        std::cerr << "tsac-cuda: " << error.what() << '\n';
        return 1;
    }
}
