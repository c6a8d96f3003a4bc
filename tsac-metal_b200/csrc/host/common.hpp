// Host-side helpers shared by the TSAC B200 library: error type, checked
// arithmetic, policy limits and the IEEE helpers the codec's bit-exact
// contract is written in.
//
// Every translation unit of this library is compiled with -ffp-contract=off
// (no implicit FMA contraction), matching the reference build
// (CMakeLists.txt:123), so each `a * b + c` below rounds twice.
#pragma once
#include <bit>
#include <cmath>
#include <cstddef>
#include <cstdint>
#include <cstring>
#include <span>
#include <stdexcept>
#include <string>
#include <vector>

namespace tsacb
{
using Bytes = std::vector<std::uint8_t>;
using ByteView = std::span<const std::uint8_t>;

// Mirrors tsac::Error (include/tsac/types.hpp:15-18): every failure is a
// std::runtime_error whose message is surfaced through the C ABI.
struct Error : std::runtime_error
{
    using std::runtime_error::runtime_error;
};

// Same policy fields and defaults as tsac::Limits (include/tsac/types.hpp:20-31).
struct Limits
{
    std::size_t file_bytes = std::size_t{512} * 1024 * 1024;
    std::size_t symbols = std::size_t{64} * 1024 * 1024;
    std::size_t pcm_bytes = std::size_t{1024} * 1024 * 1024;
    std::size_t cache_bytes = std::size_t{1024} * 1024 * 1024;
    std::size_t tensor_elements = std::size_t{128} * 1024 * 1024;
    std::size_t tensors = 10000;
    std::size_t metadata_bytes = std::size_t{1024} * 1024;
    std::size_t name_bytes = 4096;
};

inline void require(bool condition, const char* message)
{
    if (!condition)
    {
        throw Error(message);
    }
}

inline std::size_t checked_add(std::size_t a, std::size_t b)
{
    if (b > SIZE_MAX - a)
    {
        throw Error("size addition overflow");
    }
    return a + b;
}

inline std::size_t checked_mul(std::size_t a, std::size_t b)
{
    if (a && b > SIZE_MAX / a)
    {
        throw Error("size multiplication overflow");
    }
    return a * b;
}

inline std::size_t align_up(std::size_t n, std::size_t a)
{
    return checked_add(n, a - 1) / a * a;
}

// Integer round-to-nearest-even float32 -> bf16 without NaN canonicalisation
// (src/common/numeric/bf16.hpp:9-13).
inline std::uint16_t to_bf16(float value)
{
    const auto bits = std::bit_cast<std::uint32_t>(value);
    return static_cast<std::uint16_t>((bits + 0x7fffu + ((bits >> 16) & 1u)) >> 16);
}

inline float from_bf16(std::uint16_t value)
{
    return std::bit_cast<float>(std::uint32_t(value) << 16);
}

// x86 flush-to-zero of a subnormal operand or result
// (src/common/numeric/float_math.hpp:33-37).
inline float flush(float x)
{
    const auto bits = std::bit_cast<std::uint32_t>(x);
    return (bits & 0x7f800000u) == 0 ? std::bit_cast<float>(bits & 0x80000000u) : x;
}

inline float ftz_add(float x, float y)
{
    volatile float v = flush(x) + flush(y);
    return flush(v);
}

inline float ftz_sub(float x, float y)
{
    volatile float v = flush(x) - flush(y);
    return flush(v);
}

inline float ftz_mul(float x, float y)
{
    volatile float v = flush(x) * flush(y);
    return flush(v);
}

inline float ftz_div(float x, float y)
{
    volatile float v = flush(x) / flush(y);
    return flush(v);
}

// Finite check by unsigned max over |bits| (src/common/numeric.hpp:11-23).
inline void require_finite(std::span<const float> values, const char* message)
{
    std::uint32_t maximum = 0;
    for (float value : values)
    {
        const auto bits = std::bit_cast<std::uint32_t>(value) & 0x7fffffffu;
        maximum = bits > maximum ? bits : maximum;
    }
    require(maximum < 0x7f800000u, message);
}

inline std::uint32_t le32(ByteView data, std::size_t offset)
{
    require(offset <= data.size() && data.size() - offset >= 4, "truncated input");
    return std::uint32_t(data[offset]) | (std::uint32_t(data[offset + 1]) << 8) |
           (std::uint32_t(data[offset + 2]) << 16) | (std::uint32_t(data[offset + 3]) << 24);
}

inline std::uint32_t be32(ByteView data, std::size_t offset)
{
    require(offset <= data.size() && data.size() - offset >= 4, "truncated input");
    return (std::uint32_t(data[offset]) << 24) | (std::uint32_t(data[offset + 1]) << 16) |
           (std::uint32_t(data[offset + 2]) << 8) | std::uint32_t(data[offset + 3]);
}

inline float bf16_at(ByteView data, std::size_t offset)
{
    require(offset <= data.size() && data.size() - offset >= 2, "truncated input");
    return from_bf16(static_cast<std::uint16_t>(data[offset] | (data[offset + 1] << 8)));
}
} // namespace tsacb
