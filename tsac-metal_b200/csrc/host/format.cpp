#include "format.hpp"

#include "range_core.hpp"

#include <algorithm>
#include <array>

namespace tsacb
{
namespace
{
constexpr std::uint32_t stream_magic = 0x4642415au; // "FBAZ"
constexpr unsigned token_field_bits = 10;

// Big-endian field of `width` bytes at `at`; short input is "truncated input".
std::uint32_t field(ByteView bytes, std::size_t at, unsigned width)
{
    require(at <= bytes.size() && bytes.size() - at >= width, "truncated input");
    std::uint32_t value = 0;
    for (unsigned i = 0; i < width; ++i)
    {
        value = (value << 8) | bytes[at + i];
    }
    return value;
}

void append_field(Bytes& out, std::size_t value, unsigned width)
{
    for (unsigned i = width; i-- > 0;)
    {
        out.push_back(static_cast<std::uint8_t>(value >> (8 * i)));
    }
}

std::uint8_t channel_byte(const Header& h)
{
    return static_cast<std::uint8_t>(h.groups | ((h.model_channels - 1) << 7));
}

// The first eight bytes of every stream.
Bytes stream_prefix(const Header& h, std::uint8_t method, std::size_t reserve)
{
    Bytes out;
    out.reserve(reserve);
    append_field(out, stream_magic, 4);
    out.push_back(0); // version
    out.push_back(method);
    out.push_back(channel_byte(h));
    out.push_back(h.codebooks);
    return out;
}

// Fast streams carry no frame count: the payload holds whole frames of
// groups x codebooks 10-bit fields and at most 7 zero bits of padding.
void fast_geometry(Header& h, ByteView stream)
{
    h.payload_bytes = stream.size() - 8;
    const auto frame_bits = checked_mul(checked_mul(h.groups, h.codebooks), token_field_bits);
    const auto payload_bits = checked_mul(h.payload_bytes, 8);
    h.frames = payload_bits / frame_bits;
    const auto slack = static_cast<unsigned>(payload_bits % frame_bits);
    require(slack < 8, "incomplete fast frame or excess padding");
    require(slack == 0 || (stream.back() & ((1u << slack) - 1u)) == 0, "nonzero fast padding");
}

void normal_fields(Header& h, ByteView stream)
{
    require(stream.size() >= 19, "truncated normal stream");
    h.frames = field(stream, 8, 4);
    h.batch = static_cast<std::uint16_t>(field(stream, 12, 2));
    h.payload_offset = 14;
    h.payload_bytes = stream.size() - 18;
    h.token_crc = field(stream, stream.size() - 4, 4);
}

// CRC-32 tables for four bytes at a time: table[k][b] is the register after
// byte b followed by k zero bytes, starting from zero (MSB-first, 0x04c11db7).
using CrcTables = std::array<std::array<std::uint32_t, 256>, 4>;
const CrcTables& crc_tables()
{
    static const CrcTables tables = []
    {
        CrcTables t{};
        for (std::uint32_t b = 0; b < 256; ++b)
        {
            std::uint32_t reg = b << 24;
            for (int i = 0; i < 8; ++i)
            {
                reg = (reg << 1) ^ ((0u - (reg >> 31)) & 0x04c11db7u);
            }
            t[0][b] = reg;
        }
        for (int k = 1; k < 4; ++k)
        {
            for (std::uint32_t b = 0; b < 256; ++b)
            {
                const auto prev = t[k - 1][b];
                t[k][b] = (prev << 8) ^ t[0][prev >> 24];
            }
        }
        return t;
    }();
    return tables;
}

struct HostMath
{
    static std::uint16_t q15(float left, float mass)
    {
        return conditional_q15(left, mass);
    }
    static float sub(float a, float b)
    {
        return ftz_sub(a, b);
    }
};
} // namespace

// ------------------------------------------------------------- container --
void check_header(const Header& h, const Limits& limits)
{
    const unsigned most_books = h.model_channels == 1 ? 9 : 12;
    require(h.method <= 1, "unsupported method");
    require(h.groups >= 1 && h.groups <= 127, "invalid channel groups");
    require(h.model_channels == 1 || h.model_channels == 2, "invalid model channels");
    require(h.codebooks >= 1 && h.codebooks <= most_books, "invalid codebook count");
    require(h.method == 0 || h.batch != 0, "zero entropy batch size");
    require(h.symbol_count() <= limits.symbols, "symbol count exceeds limit");
    require(h.pcm16_bytes() <= limits.pcm_bytes, "decoded PCM size exceeds limit");
}

Header read_header(ByteView stream, const Limits& limits)
{
    require(stream.size() <= limits.file_bytes, "input exceeds file size limit");
    require(field(stream, 0, 4) == stream_magic, "invalid FBAZ magic");
    require(stream.size() >= 8, "truncated input");
    require(stream[4] == 0, "unsupported TSAC version");
    Header h;
    h.method = stream[5];
    h.groups = stream[6] & 0x7f;
    h.model_channels = static_cast<std::uint8_t>((stream[6] >> 7) + 1);
    h.codebooks = stream[7];
    require(h.method <= 1, "unsupported TSAC method");
    require(h.groups != 0 && h.codebooks != 0, "zero groups or codebooks");
    if (h.method == 1)
    {
        normal_fields(h, stream);
    }
    else
    {
        fast_geometry(h, stream);
    }
    check_header(h, limits);
    return h;
}

// Four 10-bit fields are exactly five bytes, so the payload is handled in
// 40-bit words; a final partial word is zero-filled.
std::vector<std::uint16_t> fast_tokens(ByteView stream, const Limits& limits)
{
    const auto h = read_header(stream, limits);
    require(h.method == 0, "normal-mode unpacking requires the probability model");
    const auto count = h.symbol_count();
    require(checked_mul(h.payload_bytes, 8) / token_field_bits == count, "fast symbol count mismatch");
    const auto payload = stream.subspan(8);
    std::vector<std::uint16_t> tokens(count);
    for (std::size_t first = 0; first < count; first += 4)
    {
        const std::size_t at = first / 4 * 5;
        std::uint64_t word = 0;
        for (std::size_t b = 0; b < 5; ++b)
        {
            word = (word << 8) | (at + b < payload.size() ? payload[at + b] : 0u);
        }
        for (std::size_t j = 0; j < 4 && first + j < count; ++j)
        {
            tokens[first + j] = static_cast<std::uint16_t>((word >> (30 - 10 * j)) & 1023u);
        }
    }
    return tokens;
}

Bytes fast_stream(const Header& header, std::span<const std::uint16_t> tokens, const Limits& limits)
{
    check_header(header, limits);
    require(header.method == 0, "pack_fast requires method 0");
    require(tokens.size() == header.symbol_count(), "symbol count does not match header");
    const auto payload = checked_add(checked_mul(tokens.size(), token_field_bits), 7) / 8;
    require(checked_add(payload, 8) <= limits.file_bytes, "output exceeds file size limit");
    require(std::all_of(tokens.begin(), tokens.end(), [](std::uint16_t t) { return t < 1024; }),
            "index outside 10-bit alphabet");
    Bytes out = stream_prefix(header, 0, payload + 8);
    out.resize(payload + 8);
    for (std::size_t first = 0; first < tokens.size(); first += 4)
    {
        std::uint64_t word = 0;
        for (std::size_t j = 0; j < 4; ++j)
        {
            word = (word << 10) | (first + j < tokens.size() ? tokens[first + j] : 0u);
        }
        const std::size_t at = 8 + first / 4 * 5;
        for (std::size_t b = 0; b < 5 && at + b < out.size(); ++b)
        {
            out[at + b] = static_cast<std::uint8_t>(word >> (32 - 8 * b));
        }
    }
    return out;
}

Bytes normal_stream(const Header& header, ByteView payload)
{
    Bytes out = stream_prefix(header, 1, payload.size() + 18);
    append_field(out, header.frames, 4);
    append_field(out, header.batch, 2);
    out.insert(out.end(), payload.begin(), payload.end());
    append_field(out, header.token_crc, 4);
    return out;
}

std::uint32_t token_crc32(std::span<const std::uint16_t> tokens)
{
    const auto& t = crc_tables();
    std::uint32_t reg = 0xffffffffu;
    for (const auto token : tokens)
    {
        require(token < 1024, "index outside 10-bit alphabet");
        // The token's little-endian bytes, first byte in the top position.
        const std::uint32_t x = reg ^ ((std::uint32_t(token & 255u) << 24) | (std::uint32_t(token >> 8) << 16));
        reg = t[3][x >> 24] ^ t[2][(x >> 16) & 255u] ^ t[1][(x >> 8) & 255u] ^ t[0][x & 255u];
    }
    return reg;
}

void check_token_crc(const Header& header, std::span<const std::uint16_t> tokens)
{
    require(header.method == 1 && tokens.size() == header.symbol_count(),
            "CRC requires a normal header and complete indices");
    require(token_crc32(tokens) == header.token_crc, "invalid token CRC32");
}

// ---------------------------------------------------------- entropy order --
std::uint16_t select_entropy_batch(std::size_t frames, int requested)
{
    require(requested >= 0 && requested <= 65535, "invalid entropy batch size");
    if (requested != 0)
    {
        return static_cast<std::uint16_t>(requested);
    }
    std::size_t lanes = frames / 1024 + (frames % 1024 != 0 ? 1 : 0);
    if (lanes > 8)
    {
        lanes = (lanes + 7) / 8 * 8;
    }
    return static_cast<std::uint16_t>(std::clamp<std::size_t>(lanes, 1, 128));
}

LaneSchedule::LaneSchedule(const Header& header)
{
    require(header.batch != 0, "zero entropy batch size");
    lanes = std::min<std::size_t>(header.batch, header.frames);
    short_length = header.frames / header.batch;
    long_lanes = header.frames % header.batch;
    steps = short_length + (long_lanes != 0 ? 1 : 0);
}

void for_each_entropy_position(const Header& header,
                               const std::function<void(const EntropyPosition&)>& symbol,
                               const Limits& limits)
{
    check_header(header, limits);
    require(header.method == 1, "entropy traversal requires method 1");
    const LaneSchedule lanes(header);
    for (std::size_t step = 0; step < lanes.steps; ++step)
    {
        for (std::size_t book = 0; book < header.codebooks; ++book)
        {
            for (std::size_t lane = 0; lane < lanes.lanes; ++lane)
            {
                if (step >= lanes.length(lane))
                {
                    continue;
                }
                const auto frame = lanes.first_frame(lane) + step;
                for (std::size_t group = 0; group < header.groups; ++group)
                {
                    const auto offset = (frame * header.groups + group) * header.codebooks + book;
                    symbol({frame, group, book, lane, step, offset});
                }
            }
        }
    }
}

// ------------------------------------------------------------ range coder --
void RangeWriter::push_top_byte()
{
    require(out_.size() < max_bytes_, "range output exceeds limit");
    out_.push_back(static_cast<std::uint8_t>(low_ >> 16));
    low_ = (low_ & 0xffffu) << 8;
    range_ <<= 8;
}

void RangeWriter::add_carry()
{
    // Bytes of 0xff wrap to 0x00 and pass the carry on to the byte before.
    for (std::size_t i = out_.size(); i-- > 0;)
    {
        if (++out_[i] != 0)
        {
            return;
        }
    }
    require(false, "range carry past the first byte");
}

void RangeWriter::put(std::uint16_t p0, bool bit)
{
    require(!finished_, "range encoder already finished");
    require(p0 > 0 && p0 < 32768, "Q15 probability must be in [1,32767]");
    const auto zero = range::zero_width(range_, p0);
    if (bit)
    {
        low_ += zero;
        range_ -= zero;
        if (low_ >> 24)
        {
            add_carry();
            low_ &= 0xffffffu;
        }
    }
    else
    {
        range_ = zero;
    }
    while (range_ < range::renormalise_below)
    {
        push_top_byte();
    }
}

std::size_t RangeWriter::bit_position() const
{
    require(!finished_, "range encoder already finished");
    return checked_add(checked_mul(out_.size(), 8), static_cast<std::size_t>(24 - std::bit_width(range_)));
}

Bytes RangeWriter::finish()
{
    require(!finished_, "range encoder already finished");
    if (range_ < 0x10000u)
    {
        push_top_byte();
    }
    // The shortest tail: the multiple of the largest power of two not above
    // the range that lies in [low, low + range); its low 16 bits are zero, so
    // only its top byte is written.
    const int top = std::bit_width(range_) - 1;
    require(top >= 16 && top <= 23, "invalid final range");
    const std::uint32_t unit = 1u << top;
    const std::uint32_t end = (low_ + unit - 1) & ~(unit - 1);
    require(end >= low_ && end - low_ < range_, "invalid range termination");
    if (end >> 24)
    {
        add_carry();
    }
    require(out_.size() < max_bytes_, "range output exceeds limit");
    out_.push_back(static_cast<std::uint8_t>(end >> 16));
    finished_ = true;
    return std::move(out_);
}

RangeReader::RangeReader(ByteView payload) : payload_(payload)
{
    for (int i = 0; i < 3; ++i)
    {
        code_ = (code_ << 8) | next_byte();
    }
    range_ = range::initial_range;
    require(code_ < range_, "range code outside initial interval");
}

bool RangeReader::get(std::uint16_t p0)
{
    require(p0 > 0 && p0 < 32768, "Q15 probability must be in [1,32767]");
    range::DecodeWindow w{range_, code_};
    const int bit = range::decide(w, p0, *this);
    require(bit >= 0, "range code outside interval");
    range_ = w.range;
    code_ = w.code;
    return bit != 0;
}

std::uint16_t RangeReader::symbol(const float* left_masses)
{
    struct Step
    {
        RangeReader& reader;
        int node(std::uint32_t p0, int)
        {
            return reader.get(static_cast<std::uint16_t>(p0)) ? 1 : 0;
        }
    } step{*this};
    return static_cast<std::uint16_t>(range::walk_bisection<HostMath>(left_masses, step));
}

void write_symbol(RangeWriter& writer, const float* left_masses, std::uint16_t symbol)
{
    require(symbol < 1024, "symbol outside the 1024-entry alphabet");
    struct Step
    {
        RangeWriter& writer;
        unsigned symbol;
        int node(std::uint32_t p0, int bit_index)
        {
            const bool bit = (symbol >> bit_index) & 1u;
            writer.put(static_cast<std::uint16_t>(p0), bit);
            return bit ? 1 : 0;
        }
    } step{writer, symbol};
    range::walk_bisection<HostMath>(left_masses, step);
}

// ------------------------------------------------------ probability model --
std::uint16_t conditional_q15(float left_mass, float mass)
{
    // round(flush(flush(left * 32768) / mass)) to a 64-bit integer, its low
    // 32 bits as a signed value clamped to [1, 32767]; nonfinite or
    // unrepresentable ratios give 1 (src/format/categorical.cpp:76-89).
    const float value = ftz_div(ftz_mul(left_mass, 32768.0f), mass);
    if (!std::isfinite(value) || value >= 0x1p63f || value < -0x1p63f)
    {
        return 1;
    }
    const auto integer = static_cast<std::int64_t>(std::nearbyint(value));
    const auto low = std::bit_cast<std::int32_t>(static_cast<std::uint32_t>(integer));
    return static_cast<std::uint16_t>(std::clamp(low, 1, 32767));
}

float probability_sum(std::span<const float> values)
{
    // Each block of up to 64 values is summed as a pairwise tree over 64
    // slots (8 slots for inputs of at most 8 values), zero-filled; block sums
    // merge like a binary counter (the running sum of block k carries into
    // the levels that its index's trailing zero bits clear), and the levels
    // left at the end add from the lowest.
    const auto tree = [](std::span<const float> input, std::size_t slots)
    {
        std::array<float, 64> v{};
        std::copy(input.begin(), input.end(), v.begin());
        for (std::size_t width = slots / 2; width >= 1; width /= 2)
        {
            for (std::size_t i = 0; i < width; ++i)
            {
                v[i] = ftz_add(v[2 * i], v[2 * i + 1]);
            }
        }
        return v[0];
    };
    if (values.size() <= 8)
    {
        return tree(values, 8);
    }
    std::array<float, 64> level{};
    std::size_t blocks = 0;
    for (std::size_t at = 0; at < values.size(); at += 64)
    {
        float carry = tree(values.subspan(at, std::min<std::size_t>(64, values.size() - at)), 64);
        ++blocks;
        const auto depth = static_cast<std::size_t>(std::countr_zero(blocks));
        for (std::size_t i = 0; i < depth; ++i)
        {
            carry = ftz_add(carry, level[i]);
            level[i] = 0;
        }
        level[depth] = carry;
    }
    float total = level[0];
    for (std::size_t i = 1; i < static_cast<std::size_t>(std::bit_width(blocks)); ++i)
    {
        total = ftz_add(total, level[i]);
    }
    return total;
}
} // namespace tsacb
