// The .tsac stream on the host: container header and framing, the order in
// which a normal stream's symbols are coded, and the sequential range coder
// that writes and reads them.
//
// What the stream fixes, and where the reference defines it:
//   header bytes, fast 10-bit packing, token CRC-32   src/format/container.cpp:9-190
//   entropy lanes and symbol order                    src/format/entropy.cpp:11-55
//   binary range coder                                src/format/range.cpp:14-157
//   bisection coding with conditional_q15             src/format/categorical.cpp:76-142
// The arithmetic shared with the device decoder lives in range_core.hpp.
#pragma once
#include "common.hpp"

#include <functional>

namespace tsacb
{
// Decoded stream header.  Byte layout: "FBAZ", version 0, method, then
// (groups | (model channels - 1) << 7), codebooks; a normal stream follows
// with frames (BE32) and entropy batch (BE16), the range-coded payload and
// the token CRC-32 (BE32); a fast stream with 10-bit token fields.
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
    // Rows the probability model evaluates per step: entropy lanes x groups.
    std::size_t lanes() const
    {
        return (batch < frames ? batch : frames) * groups;
    }
};

// Rejects a header whose dimensions or policy limits are out of range.
void check_header(const Header& header, const Limits& limits = {});
// Decodes and checks the header of a whole stream.
Header read_header(ByteView stream, const Limits& limits = {});
// Tokens [frame][group][book] of a fast (method 0) stream.
std::vector<std::uint16_t> fast_tokens(ByteView stream, const Limits& limits = {});
// A fast stream of tokens [frame][group][book].
Bytes fast_stream(const Header& header, std::span<const std::uint16_t> tokens,
                  const Limits& limits = {});
// A normal stream: header, the range coder's payload, header.token_crc.
Bytes normal_stream(const Header& header, ByteView payload);
// CRC-32 (polynomial 0x04c11db7, MSB first, initial ~0, no final xor) over
// the four little-endian bytes of each token.
std::uint32_t token_crc32(std::span<const std::uint16_t> tokens);
void check_token_crc(const Header& header, std::span<const std::uint16_t> tokens);

// Entropy batch for a recording of `frames` frames: `requested` if nonzero,
// else one lane per started 1024 frames, rounded up to a multiple of 8 past
// 8 lanes, within 1..128.
std::uint16_t select_entropy_batch(std::size_t frames, int requested = 0);

// The frames of a normal stream split into min(batch, frames) lanes of
// consecutive frames; the first frames % batch lanes hold one frame more.
// Step s of lane l is frame first_frame(l) + s.
struct LaneSchedule
{
    std::size_t lanes = 0, steps = 0, short_length = 0, long_lanes = 0;

    explicit LaneSchedule(const Header& header);
    std::size_t length(std::size_t lane) const
    {
        return short_length + (lane < long_lanes ? 1 : 0);
    }
    std::size_t first_frame(std::size_t lane) const
    {
        return lane * short_length + (lane < long_lanes ? lane : long_lanes);
    }
};

struct EntropyPosition
{
    std::size_t frame, group, codebook, lane, step, token_offset;
};
// Calls `symbol` for every symbol of a normal stream in coding order: step,
// then codebook, then lane, then group.
void for_each_entropy_position(const Header& header,
                               const std::function<void(const EntropyPosition&)>& symbol,
                               const Limits& limits = {});

// Writes binary decisions.  Output bytes are appended as soon as they leave
// the 24-bit window; a carry out of the window is added into the bytes
// already written.
class RangeWriter
{
public:
    explicit RangeWriter(std::size_t max_bytes = std::size_t{64} * 1024 * 1024) : max_bytes_(max_bytes) {}
    void put(std::uint16_t p0, bool bit);
    // Bits the stream holds so far (whole bytes written plus the settled
    // high bits of the window).
    std::size_t bit_position() const;
    Bytes finish();

private:
    void add_carry();
    void push_top_byte();
    std::uint32_t low_ = 0, range_ = 0xff0000u;
    std::size_t max_bytes_;
    bool finished_ = false;
    Bytes out_;
};

class RangeReader
{
public:
    explicit RangeReader(ByteView payload);
    bool get(std::uint16_t p0);
    // One symbol of 1024 from its 1023 left-child masses (heap order).
    std::uint16_t symbol(const float* left_masses);

    // The byte source of range::decide: the next payload byte, 0 past the end.
    std::uint32_t next_byte()
    {
        return at_ < payload_.size() ? payload_[at_++] : 0u;
    }

private:
    ByteView payload_;
    std::size_t at_ = 0;
    std::uint32_t range_ = 0, code_ = 0;
};

std::uint16_t conditional_q15(float left_mass, float mass);
// Codes `symbol`'s 10 decisions with the node probabilities of its path.
void write_symbol(RangeWriter& writer, const float* left_masses, std::uint16_t symbol);
// Host probability_sum (64-value FTZ pair trees + binary carry,
// src/format/categorical.cpp:44-74).
float probability_sum(std::span<const float> values);
} // namespace tsacb
