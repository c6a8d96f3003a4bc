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
#include <cfenv>
#include <span>
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

// One command line option.  `letter` is its short spelling (0: none), `word`
// its long one ("" for none).  Value options read the following argument; an
// integer may carry a leading '+'.
struct OptionSpec
{
    char letter;
    std::string_view word;
    enum Kind { set_flag, add_one, integer, text, refused } kind;
    bool Options::* flag = nullptr;
    int Options::* number = nullptr;
};

constexpr std::string_view letters = "hfsvTqc";

const std::vector<OptionSpec>& option_table()
{
    static const std::vector<OptionSpec> table{
        {'h', "--help", OptionSpec::set_flag, &Options::help},
        {'f', "--fast", OptionSpec::set_flag, &Options::fast},
        {'s', "--separate_channels", OptionSpec::set_flag, &Options::separate},
        {'v', "", OptionSpec::add_one},
        {'T', "", OptionSpec::integer, nullptr, &Options::threads},
        {'q', "--n_codebooks", OptionSpec::integer, nullptr, &Options::quality},
        {'c', "--channels", OptionSpec::integer, nullptr, &Options::channels},
        {0, "--batch_size", OptionSpec::integer, nullptr, &Options::batch},
        {0, "--metal", OptionSpec::refused},
        {0, "--exact", OptionSpec::set_flag, &Options::exact},
        {0, "--device", OptionSpec::integer, nullptr, &Options::device},
        {0, "--models", OptionSpec::text},
    };
    return table;
}

const OptionSpec* find_option(std::string_view spelled)
{
    for (const auto& spec : option_table())
        if ((spelled.size() == 2 && spec.letter && spelled[1] == spec.letter) ||
            (!spec.word.empty() && spelled == spec.word))
            return &spec;
    return nullptr;
}

// Integer option values: the whole argument, optionally after a '+'.  A bad
// value names the option by its long spelling where it has one.
int integer_value(const OptionSpec& spec, std::string_view spelled, std::string_view text)
{
    const std::string_view digits = text.starts_with('+') ? text.substr(1) : text;
    int number = 0;
    const auto [end, ec] = std::from_chars(digits.data(), digits.data() + digits.size(), number);
    if (digits.empty() || ec != std::errc{} || end != digits.data() + digits.size())
    {
        const bool use_word = spec.letter && !spec.word.empty() && spec.kind == OptionSpec::integer;
        throw Error("option " + std::string(use_word ? spec.word : spelled) + " expects an integer");
    }
    return number;
}

// The reference command line rules (src/cli.cpp:7-130): short options may be
// grouped ("-vv", "-fs"), every letter of a group is checked before any is
// applied (so "-q1" is the unknown option '-1', not an attached value), "--"
// ends the options, "-h" ends parsing, and anything but three positionals
// (command, input, output) prints the help.
Options parse_cli(const std::vector<std::string_view>& arguments)
{
    Options options;
    std::vector<std::string_view> positional;
    std::size_t next = 0;
    const auto take_value = [&](std::string_view spelled) -> std::string_view
    {
        if (next >= arguments.size())
            throw Error("option '" + std::string(spelled) + "' must have an argument");
        return arguments[next++];
    };
    const auto apply = [&](const OptionSpec& spec, std::string_view spelled)
    {
        switch (spec.kind)
        {
        case OptionSpec::set_flag:
            options.*spec.flag = true;
            break;
        case OptionSpec::add_one:
            ++options.verbose;
            break;
        case OptionSpec::integer:
            options.*spec.number = integer_value(spec, spelled, take_value(spelled));
            break;
        case OptionSpec::text:
            options.models = std::string(take_value(spelled));
            break;
        case OptionSpec::refused:
            throw Error("Metal execution is not available on this platform (this tool runs on CUDA)");
        }
    };
    while (next < arguments.size() && !options.help)
    {
        const auto arg = arguments[next++];
        if (arg == "--")
        {
            positional.insert(positional.end(), arguments.begin() + static_cast<std::ptrdiff_t>(next),
                              arguments.end());
            break;
        }
        if (arg.size() < 2 || arg.front() != '-')
        {
            positional.push_back(arg);
        }
        else if (arg.starts_with("--"))
        {
            const auto* spec = find_option(arg);
            if (!spec || spec->word.empty())
                throw Error("unknown option: '" + std::string(arg) + "'");
            apply(*spec, arg);
        }
        else
        {
            const auto group = arg.substr(1);
            if (const auto bad = group.find_first_not_of(letters); bad != std::string_view::npos)
                throw Error("unknown option: '-" + std::string(1, group[bad]) + "'");
            for (const char letter : group)
            {
                const std::string spelled{'-', letter};
                apply(*find_option(spelled), spelled);
            }
        }
    }
    if (options.help)
        return options;
    if (positional.size() != 3)
    {
        options.help = true;
        return options;
    }
    const auto command = positional[0];
    if (command.size() != 1 || std::string_view("cdt").find(command[0]) == std::string_view::npos)
        throw Error("unknown command: " + std::string(command));
    options.command = command[0];
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

// Little-endian unsigned field of `width` bytes; out of range is a bad file.
std::uint32_t le_field(std::span<const std::uint8_t> bytes, std::size_t at, unsigned width)
{
    require(at <= bytes.size() && bytes.size() - at >= width, "invalid wav file");
    std::uint32_t value = 0;
    for (unsigned i = width; i-- > 0;)
        value = (value << 8) | bytes[at + i];
    return value;
}

// Raw little-endian PCM16 (pcm16_input, src/audio.cpp:19-37): whole
// interleaved frames only (a trailing partial frame is dropped), each sample
// value / 32768, zero-padded to a multiple of 512 frames.
Audio pcm16_input(std::span<const std::uint8_t> bytes, unsigned channels)
{
    require(channels > 0 && channels <= 127, "unsupported number of channels");
    const std::size_t frames = bytes.size() / (2 * std::size_t{channels});
    const std::size_t samples = frames * channels;
    Audio audio{channels, std::vector<float>((frames + 511) / 512 * 512 * channels, 0.0f)};
    for (std::size_t i = 0; i < samples; ++i)
    {
        const auto value = static_cast<std::int16_t>(static_cast<std::uint16_t>(le_field(bytes, 2 * i, 2)));
        audio.samples[i] = static_cast<float>(value) * (1.0f / 32768.0f);
    }
    return audio;
}

// RIFF/WAVE input (wave_input, src/audio.cpp:39-73).  Chunks are walked from
// byte 12 by their declared sizes (no pad byte); "fmt " must describe 16-bit
// PCM at 44.1 kHz with 1..8 channels and precede "data", whose samples run to
// the end of the file whatever its declared size.
Audio wave_input(std::span<const std::uint8_t> bytes)
{
    const auto id_is = [&](std::size_t at, std::string_view id)
    { return at <= bytes.size() && bytes.size() - at >= 4 && std::string_view(
                 reinterpret_cast<const char*>(bytes.data() + at), 4) == id; };
    require(id_is(0, "RIFF") && id_is(8, "WAVE"), "invalid wav file");
    unsigned channels = 0;
    std::size_t chunk = 12;
    while (chunk < bytes.size())
    {
        const std::size_t size = le_field(bytes, chunk + 4, 4);
        const std::size_t body = chunk + 8;
        if (id_is(chunk, "data"))
        {
            require(channels > 0, "invalid wav file");
            return pcm16_input(bytes.subspan(body), channels);
        }
        require(bytes.size() - body >= size, "invalid wav file");
        const auto content = bytes.subspan(body, size);
        if (id_is(chunk, "fmt "))
        {
            const bool pcm16 = size >= 16 && le_field(content, 0, 2) == 1 && le_field(content, 14, 2) == 16;
            require(pcm16, "invalid wav file");
            channels = le_field(content, 2, 2);
            require(channels >= 1 && channels <= 8, "unsupported number of channels");
            require(le_field(content, 4, 4) == 44100, "the sample rate must be 44100 Hz");
        }
        chunk = body + size;
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
        return pcm16_input(bytes, requested_channels ? static_cast<unsigned>(requested_channels) : 1);
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

// 16-bit WAVE output (pcm16_wave, src/audio.cpp:184-247): a 44-byte
// canonical header, then every sample (padding included) as
// clamp(x * 32768, -32768, 32767) rounded to nearest, ties to even.
Bytes pcm16_wave(const std::vector<float>& samples, unsigned channels)
{
    require(channels > 0 && samples.size() % channels == 0, "audio sample shape mismatch");
    const std::uint64_t block = 2ull * channels, data_bytes = 2ull * samples.size();
    require(block <= 0xffffu && block * 44100 <= 0xffffffffull && data_bytes <= 0xffffffffull - 36,
            "audio exceeds RIFF/WAVE dimensions");
    require(std::all_of(samples.begin(), samples.end(), [](float x) { return std::isfinite(x); }),
            "nonfinite audio sample");
    struct Field
    {
        std::uint64_t value;
        unsigned width;
    };
    const Field header[] = {{0x46464952u, 4}, {data_bytes + 36, 4}, {0x45564157u, 4}, {0x20746d66u, 4},
                            {16, 4}, {1, 2}, {channels, 2}, {44100, 4}, {block * 44100, 4},
                            {block, 2}, {16, 2}, {0x61746164u, 4}, {data_bytes, 4}};
    Bytes out(44 + data_bytes);
    std::size_t at = 0;
    for (const auto& f : header)
        for (unsigned i = 0; i < f.width; ++i)
            out[at++] = static_cast<std::uint8_t>(f.value >> (8 * i));
    for (const float x : samples)
    {
        // Rounding in double under the default round-to-nearest-even mode.
        const auto value = static_cast<std::int32_t>(std::nearbyint(std::clamp(double(x) * 32768.0, -32768.0, 32767.0)));
        const auto word = static_cast<std::uint16_t>(value);
        out[at++] = static_cast<std::uint8_t>(word);
        out[at++] = static_cast<std::uint8_t>(word >> 8);
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

Bytes compress(Context& c, const Audio& audio, const Options& options, std::size_t& frames,
               unsigned& channels)
{
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
    // Input is read and checked before the device is touched.
    Audio audio;
    Bytes stream;
    if (options.command == 'd')
        stream = read_file(options.input);
    else
        audio = read_audio(options.input, options.channels);
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
        output = compress(c, audio, options, frames, channels);
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
        output = decompress(c, stream, options);
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
