#include "format.hpp"

#include <algorithm>
#include <array>

namespace tsacb
{
void validate_header(const Header& header, const Limits& limits)
{
    require(header.method <= 1, "unsupported method");
    require(header.groups > 0 && header.groups <= 127, "invalid channel groups");
    require(header.model_channels == 1 || header.model_channels == 2, "invalid model channels");
    require(header.codebooks > 0 && header.codebooks <= (header.model_channels == 1 ? 9 : 12),
            "invalid codebook count");
    require(header.method == 0 || header.batch > 0, "zero entropy batch size");
    require(header.symbol_count() <= limits.symbols, "symbol count exceeds limit");
    require(header.pcm16_bytes() <= limits.pcm_bytes, "decoded PCM size exceeds limit");
}

Header parse_header(ByteView bytes, const Limits& limits)
{
    require(bytes.size() <= limits.file_bytes, "input exceeds file size limit");
    require(be32(bytes, 0) == 0x4642415a, "invalid FBAZ magic");
    require(bytes.size() >= 8, "truncated input");
    require(bytes[4] == 0, "unsupported TSAC version");
    Header header;
    header.method = bytes[5];
    header.groups = bytes[6] & 127;
    header.model_channels = static_cast<std::uint8_t>(1 + (bytes[6] >> 7));
    header.codebooks = bytes[7];
    require(header.method <= 1, "unsupported TSAC method");
    require(header.groups && header.codebooks, "zero groups or codebooks");
    if (header.method == 0)
    {
        header.payload_bytes = bytes.size() - 8;
        const auto bits_per_frame = checked_mul(checked_mul(header.groups, header.codebooks), 10);
        const auto bits = checked_mul(header.payload_bytes, 8);
        header.frames = bits / bits_per_frame;
        const auto padding = bits % bits_per_frame;
        require(padding < 8, "incomplete fast frame or excess padding");
        if (padding)
        {
            require((bytes.back() & ((1u << padding) - 1)) == 0, "nonzero fast padding");
        }
    }
    else
    {
        require(bytes.size() >= 19, "truncated normal stream");
        header.frames = be32(bytes, 8);
        header.batch = static_cast<std::uint16_t>((std::uint16_t(bytes[12]) << 8) | bytes[13]);
        header.payload_offset = 14;
        header.payload_bytes = bytes.size() - 18;
        header.token_crc = be32(bytes, bytes.size() - 4);
    }
    validate_header(header, limits);
    return header;
}

std::vector<std::uint16_t> unpack_fast(ByteView bytes, const Limits& limits)
{
    const auto header = parse_header(bytes, limits);
    require(header.method == 0, "normal-mode unpacking requires the probability model");
    std::vector<std::uint16_t> indices;
    indices.reserve(header.symbol_count());
    std::uint32_t buffer = 0;
    unsigned bits = 0;
    for (auto byte : bytes.subspan(8))
    {
        buffer = (buffer << 8) | byte;
        bits += 8;
        while (bits >= 10)
        {
            bits -= 10;
            indices.push_back(static_cast<std::uint16_t>((buffer >> bits) & 1023));
        }
        buffer &= (1u << bits) - 1;
    }
    require(indices.size() == header.symbol_count(), "fast symbol count mismatch");
    return indices;
}

Bytes pack_fast(const Header& header, std::span<const std::uint16_t> indices, const Limits& limits)
{
    validate_header(header, limits);
    require(header.method == 0, "pack_fast requires method 0");
    require(indices.size() == header.symbol_count(), "symbol count does not match header");
    const auto payload = checked_add(checked_mul(indices.size(), 10), 7) / 8;
    require(checked_add(payload, 8) <= limits.file_bytes, "output exceeds file size limit");
    Bytes bytes{'F', 'B', 'A', 'Z', 0, 0,
                static_cast<std::uint8_t>(header.groups | ((header.model_channels - 1) << 7)),
                header.codebooks};
    bytes.reserve(payload + 8);
    std::uint32_t buffer = 0;
    unsigned bits = 0;
    for (auto index : indices)
    {
        require(index < 1024, "index outside 10-bit alphabet");
        buffer = (buffer << 10) | index;
        bits += 10;
        while (bits >= 8)
        {
            bits -= 8;
            bytes.push_back(static_cast<std::uint8_t>(buffer >> bits));
        }
        buffer &= (1u << bits) - 1;
    }
    if (bits)
    {
        bytes.push_back(static_cast<std::uint8_t>(buffer << (8 - bits)));
    }
    return bytes;
}

std::uint32_t token_crc32(std::span<const std::uint16_t> indices)
{
    // CRC-32 (poly 0x04c11db7, MSB first, init ~0, no final xor) over the four
    // little-endian bytes of each token widened to 32 bits; table-driven.
    static const auto table = []
    {
        std::array<std::uint32_t, 256> t{};
        for (std::uint32_t i = 0; i < 256; ++i)
        {
            std::uint32_t c = i << 24;
            for (int b = 0; b < 8; ++b)
            {
                c = (c << 1) ^ ((c & 0x80000000u) ? 0x04c11db7u : 0u);
            }
            t[i] = c;
        }
        return t;
    }();
    std::uint32_t crc = 0xffffffff;
    for (auto index : indices)
    {
        require(index < 1024, "index outside 10-bit alphabet");
        const std::uint32_t v = index;
        for (unsigned shift = 0; shift < 32; shift += 8)
        {
            crc = (crc << 8) ^ table[((crc >> 24) ^ ((v >> shift) & 255u)) & 255u];
        }
    }
    return crc;
}

void verify_token_crc(const Header& header, std::span<const std::uint16_t> indices)
{
    require(header.method == 1 && indices.size() == header.symbol_count(),
            "CRC requires a normal header and complete indices");
    require(token_crc32(indices) == header.token_crc, "invalid token CRC32");
}

std::uint16_t select_entropy_batch(std::size_t frames, int requested)
{
    require(requested >= 0 && requested <= 65535, "invalid entropy batch size");
    if (requested)
    {
        return static_cast<std::uint16_t>(requested);
    }
    auto batch = frames / 1024 + (frames % 1024 != 0);
    if (batch > 8)
    {
        batch = checked_add(batch, 7) & ~std::size_t{7};
    }
    return static_cast<std::uint16_t>(std::clamp<std::size_t>(batch, 1, 128));
}

void visit_entropy_positions(const Header& header,
                             const std::function<void(const EntropyPosition&)>& visit,
                             const Limits& limits)
{
    validate_header(header, limits);
    require(header.method == 1, "entropy traversal requires method 1");
    const auto per_lane = header.frames / header.batch;
    const auto extra = header.frames % header.batch;
    const auto steps = per_lane + (extra != 0);
    const auto lanes = std::min<std::size_t>(header.batch, header.frames);
    for (std::size_t step = 0; step < steps; ++step)
    {
        for (std::size_t book = 0; book < header.codebooks; ++book)
        {
            for (std::size_t lane = 0; lane < lanes; ++lane)
            {
                if (step >= per_lane + (lane < extra))
                {
                    continue;
                }
                const auto frame = lane * per_lane + std::min(lane, extra) + step;
                for (std::size_t group = 0; group < header.groups; ++group)
                {
                    visit({frame, group, book, lane, step,
                           (frame * header.groups + group) * header.codebooks + book});
                }
            }
        }
    }
}

Bytes frame_normal(const Header& header, ByteView payload)
{
    Bytes bytes{'F', 'B', 'A', 'Z', 0, 1,
                static_cast<std::uint8_t>(header.groups | ((header.model_channels - 1) << 7)),
                header.codebooks};
    const auto be = [&](std::size_t value, unsigned count)
    {
        for (unsigned i = count; i > 0; --i)
        {
            bytes.push_back(static_cast<std::uint8_t>(value >> ((i - 1) * 8)));
        }
    };
    be(header.frames, 4);
    be(header.batch, 2);
    bytes.insert(bytes.end(), payload.begin(), payload.end());
    be(header.token_crc, 4);
    return bytes;
}

// ------------------------------------------------------------ range coder --
namespace
{
constexpr std::uint32_t minimum_range = 0xff01;

std::uint32_t split(std::uint32_t range, std::uint16_t p0)
{
    require(p0 > 0 && p0 < 32768, "Q15 probability must be in [1,32767]");
    require(range >= minimum_range, "unnormalized range state");
    return static_cast<std::uint32_t>((std::uint64_t(range) * p0) >> 15);
}
} // namespace

void RangeEncoder::emit(std::uint32_t value)
{
    require(bytes_.size() < max_bytes_, "range output exceeds limit");
    bytes_.push_back(static_cast<std::uint8_t>(value));
}

void RangeEncoder::flush_pending(std::uint32_t value)
{
    const auto carry = (value >> 8) & 255;
    if (pending_count_)
    {
        emit(std::uint32_t(pending_byte_) + carry);
        while (pending_count_ > 1)
        {
            emit(carry - 1);
            --pending_count_;
        }
    }
    pending_byte_ = static_cast<std::uint8_t>(value);
    pending_count_ = 1;
}

void RangeEncoder::shift()
{
    if ((low_ >> 16) == 0xff)
    {
        pending_count_ = checked_add(pending_count_, 1);
        require(pending_count_ <= max_bytes_, "pending range output exceeds limit");
    }
    else
    {
        flush_pending(low_ >> 16);
    }
    low_ = (low_ & 0xffff) << 8;
    range_ <<= 8;
}

void RangeEncoder::put(std::uint16_t probability_zero, bool bit)
{
    require(!finished_, "range encoder already finished");
    const auto range0 = split(range_, probability_zero);
    if (bit)
    {
        low_ += range0;
        range_ -= range0;
    }
    else
    {
        range_ = range0;
    }
    while (range_ < minimum_range)
    {
        shift();
    }
}

std::size_t RangeEncoder::bit_position() const
{
    require(!finished_, "range encoder already finished");
    const auto whole = checked_add(pending_count_, bytes_.size());
    return checked_add(checked_mul(whole, 8),
                       static_cast<std::size_t>(24 - std::bit_width(range_)));
}

Bytes RangeEncoder::finish()
{
    require(!finished_, "range encoder already finished");
    if (range_ < 0x10000)
    {
        shift();
    }
    const auto n = std::bit_width(range_) - 1;
    require(n >= 16 && n <= 23, "invalid final range");
    const std::uint32_t unit = 1u << n;
    const auto val = (low_ & (unit - 1)) == 0 ? low_ : (low_ + unit) & (0u - unit);
    require(val >= low_ && val < low_ + range_, "invalid range termination");
    if ((val >> 16) == 0xff)
    {
        pending_count_ = checked_add(pending_count_, 1);
        require(pending_count_ <= max_bytes_, "pending range output exceeds limit");
    }
    else
    {
        flush_pending(val >> 16);
    }
    if (pending_count_)
    {
        flush_pending(0);
    }
    finished_ = true;
    return std::move(bytes_);
}

std::uint32_t RangeDecoder::read()
{
    return offset_ < bytes_.size() ? bytes_[offset_++] : 0u;
}

RangeDecoder::RangeDecoder(ByteView bytes) : bytes_(bytes)
{
    code_ = read() << 16;
    code_ |= read() << 8;
    code_ |= read();
    require(code_ < range_, "range code outside initial interval");
}

bool RangeDecoder::get(std::uint16_t probability_zero)
{
    const auto range0 = split(range_, probability_zero);
    const bool bit = code_ >= range0;
    if (bit)
    {
        code_ -= range0;
        range_ -= range0;
    }
    else
    {
        range_ = range0;
    }
    while (range_ < minimum_range)
    {
        range_ <<= 8;
        code_ = (code_ << 8) + read();
    }
    require(code_ < range_, "range code outside interval");
    return bit;
}

std::uint16_t conditional_q15(float left_mass, float mass)
{
    const float value = ftz_div(ftz_mul(left_mass, 32768.0f), mass);
    if (!std::isfinite(value) || value >= 0x1p63f || value < -0x1p63f)
    {
        return 1;
    }
    const auto integer = static_cast<std::int64_t>(std::nearbyint(value));
    const auto low = std::bit_cast<std::int32_t>(static_cast<std::uint32_t>(integer));
    return static_cast<std::uint16_t>(std::clamp(low, 1, 32767));
}

void encode_categorical_tree(RangeEncoder& encoder, const float* left_masses, std::uint16_t symbol)
{
    std::size_t node = 0, base = 0, count = 1024;
    float mass = 1;
    while (count > 1)
    {
        const auto half = count / 2;
        const float left = left_masses[node];
        const bool bit = symbol >= base + half;
        encoder.put(conditional_q15(left, mass), bit);
        if (bit)
        {
            base += half;
            count -= half;
            mass = ftz_sub(mass, left);
            node = 2 * node + 2;
        }
        else
        {
            count = half;
            mass = left;
            node = 2 * node + 1;
        }
    }
}

std::uint16_t decode_categorical_tree(RangeDecoder& decoder, const float* left_masses)
{
    std::size_t node = 0, base = 0, count = 1024;
    float mass = 1;
    while (count > 1)
    {
        const auto half = count / 2;
        const float left = left_masses[node];
        if (decoder.get(conditional_q15(left, mass)))
        {
            base += half;
            count -= half;
            mass = ftz_sub(mass, left);
            node = 2 * node + 2;
        }
        else
        {
            count = half;
            mass = left;
            node = 2 * node + 1;
        }
    }
    return static_cast<std::uint16_t>(base);
}

float probability_sum(std::span<const float> values)
{
    const auto pair_sum = [](std::span<const float> input, std::size_t width)
    {
        std::array<float, 64> v{};
        std::copy(input.begin(), input.end(), v.begin());
        while (width > 1)
        {
            width /= 2;
            for (std::size_t i = 0; i < width; ++i)
            {
                v[i] = ftz_add(v[2 * i], v[2 * i + 1]);
            }
        }
        return v[0];
    };
    if (values.size() <= 8)
    {
        return pair_sum(values, 8);
    }
    std::array<float, 64> partial{};
    std::size_t blocks = 0;
    for (std::size_t offset = 0; offset < values.size();)
    {
        const auto count = std::min<std::size_t>(64, values.size() - offset);
        float value = pair_sum(values.subspan(offset, count), 64);
        ++blocks;
        const auto level = static_cast<std::size_t>(std::countr_zero(blocks));
        for (std::size_t i = 0; i < level; ++i)
        {
            value = ftz_add(value, partial[i]);
            partial[i] = 0;
        }
        partial[level] = value;
        offset += count;
    }
    float value = partial[0];
    for (std::size_t i = 1; i < static_cast<std::size_t>(std::bit_width(blocks)); ++i)
    {
        value = ftz_add(value, partial[i]);
    }
    return value;
}
} // namespace tsacb
