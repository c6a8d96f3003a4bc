// Launch interface of the device range decoder: the host decode loop's
// RangeDecoder + categorical tree walk run on the GPU, one serialized range
// state per stream, as the reference's Metal range_decode kernel does
// (src/metal/probability/range.metal:12-77).
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace tsacb::dev
{
// One stream's decoder between calls (16 bytes): range, code, the next
// payload byte to read, and a status (0 running, 1 the code left its
// interval; the stream then decodes nothing more).
struct RangeCursor
{
    std::uint32_t range, code, offset, status;
};

// Starts the decoders of `streams` payloads: payload s is
// bytes[offsets[s], offsets[s] + sizes[s]) (all device memory).
void range_start(const std::uint8_t* bytes, const std::uint64_t* offsets, const std::uint64_t* sizes,
                 RangeCursor* cursors, int streams, unsigned* error_word, cudaStream_t stream);

// Decodes `count` symbols: row r belongs to stream rows[r], and each stream's
// rows are decoded in increasing r (its stream order).  masses: [count][1023]
// left-child masses in heap order (the softmax_tree output); symbols: [count].
// A stream whose code leaves its interval gets status 1, its remaining rows
// symbol 0, and error_range in error_word.
void range_decode(const std::uint8_t* bytes, const std::uint64_t* offsets, const std::uint64_t* sizes,
                  RangeCursor* cursors, int streams, const int* rows, int count, const float* masses,
                  std::uint16_t* symbols, unsigned* error_word, cudaStream_t stream);
// The decode loop's form: stream s decodes rows [row_begin[s], row_begin[s+1])
// in order (row_begin has streams + 1 entries), and row r's symbol is stored
// to tokens[destination[r]].  Launched with programmatic dependent launch.
void range_decode_rows(const std::uint8_t* bytes, const std::uint64_t* offsets, const std::uint64_t* sizes,
                       RangeCursor* cursors, int streams, const int* row_begin, const float* masses,
                       const int* destination, std::uint16_t* tokens, unsigned* error_word, cudaStream_t stream);
} // namespace tsacb::dev
