// TSAC container format, entropy traversal order and the sequential range
// coder, restated for this library's host side.
//
//   Header / validate / parse / fast pack / CRC   src/format/container.cpp:9-190
//   select_entropy_batch / visit_entropy_positions src/format/entropy.cpp:11-55
//   RangeEncoder / RangeDecoder                     src/format/range.cpp:14-157
//   conditional_q15 / bisection coding             src/format/categorical.cpp:76-142
#pragma once
#include "common.hpp"

#include <functional>

namespace tsacb
{
struct Header
{
    std::uint8_t method = 0;
    std::uint8_t groups = 1;
    std::uint8_t model_channels = 1;
    std::uint8_t codebooks = 1;
    std::size_t frames = 0;
    std::uint16_t batch = 1;
    std::size_t payload_offset = 8;
    std::size_t payload_bytes = 0;
    std::uint32_t token_crc = 0;

    std::size_t symbol_count() const
    {
        return checked_mul(checked_mul(frames, groups), codebooks);
    }
    std::size_t channels() const
    {
        return checked_mul(groups, model_channels);
    }
    std::size_t samples_per_channel() const
    {
        return checked_mul(frames, 512);
    }
    std::size_t pcm16_bytes() const
    {
        return checked_mul(checked_mul(samples_per_channel(), channels()), 2);
    }
    std::size_t lanes() const // entropy lanes x groups
    {
        return (batch < frames ? batch : frames) * groups;
    }
};

struct EntropyPosition
{
    std::size_t frame, group, codebook, lane, step, token_offset;
};

void validate_header(const Header& header, const Limits& limits = {});
Header parse_header(ByteView bytes, const Limits& limits = {});
std::vector<std::uint16_t> unpack_fast(ByteView bytes, const Limits& limits = {});
Bytes pack_fast(const Header& header, std::span<const std::uint16_t> indices,
                const Limits& limits = {});
std::uint32_t token_crc32(std::span<const std::uint16_t> indices);
void verify_token_crc(const Header& header, std::span<const std::uint16_t> indices);
std::uint16_t select_entropy_batch(std::size_t frames, int requested = 0);
// Calls visit in stream order: step, then book, then lane, then group.
void visit_entropy_positions(const Header& header,
                             const std::function<void(const EntropyPosition&)>& visit,
                             const Limits& limits = {});
// Normal-stream framing around a range-coded payload.
Bytes frame_normal(const Header& header, ByteView payload);

class RangeEncoder
{
public:
    explicit RangeEncoder(std::size_t max_bytes = std::size_t{64} * 1024 * 1024)
        : max_bytes_(max_bytes)
    {
    }
    void put(std::uint16_t probability_zero, bool bit);
    std::size_t bit_position() const;
    Bytes finish();

private:
    void emit(std::uint32_t value);
    void flush_pending(std::uint32_t value);
    void shift();
    std::uint32_t range_ = 0xff0000, low_ = 0;
    std::uint8_t pending_byte_ = 0xff;
    std::size_t pending_count_ = 0, max_bytes_;
    bool finished_ = false;
    Bytes bytes_;
};

class RangeDecoder
{
public:
    explicit RangeDecoder(ByteView bytes);
    bool get(std::uint16_t probability_zero);

private:
    std::uint32_t read();
    ByteView bytes_;
    std::size_t offset_ = 0;
    std::uint32_t range_ = 0xff0000, code_ = 0;
};

std::uint16_t conditional_q15(float left_mass, float mass);
// Decodes one symbol of a 1024-entry alphabet from the left-child masses of
// the 1023 internal bisection nodes (heap order: children 2i+1, 2i+2).
std::uint16_t decode_categorical_tree(RangeDecoder& decoder, const float* left_masses);
// The encoding counterpart (encode_categorical, src/format/categorical.cpp:91-117):
// the 10 decisions of `symbol`'s path, each with conditional_q15 of the node's
// left mass and the path mass.
void encode_categorical_tree(RangeEncoder& encoder, const float* left_masses, std::uint16_t symbol);
// Host probability_sum (64-value FTZ pair trees + binary carry).
float probability_sum(std::span<const float> values);
} // namespace tsacb
