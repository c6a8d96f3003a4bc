// Device range decoding of normal-stream symbols, restating (reference
// project paths):
//   RangeDecoder read / start / get   src/format/range.cpp:118-157
//   decode_categorical (tree walk)    src/format/categorical.cpp:119-142,
//                                     with the left-child masses the softmax
//                                     kernel emits (heap order, right mass =
//                                     path mass - left, never re-summed)
//   the Metal serialized decoder      src/metal/probability/range.metal:12-77
//
// B200 mapping: a stream's symbols are one serial chain (each decision's
// renormalisation decides which payload byte the next reads), so a stream is
// one lane; streams (recordings) are independent, one warp each.  The warp
// finds its rows with ballots over the row list, in row order, and lane 0
// walks them.  Every loop is bounded: 10 decisions per symbol and at most
// three renormalising shifts per decision (range >= 1 after any split).
#include "kernels/error_bits.hpp"
#include "kernels/launch_count.hpp"
#include "kernels/numeric.cuh"
#include "kernels/range_decode.cuh"
#include "kernels/row_ops.cuh"

namespace tsacb::dev
{
namespace
{
constexpr std::uint32_t MINIMUM_RANGE = 0xff01u, INITIAL_RANGE = 0xff0000u;

__device__ __forceinline__ std::uint32_t payload_byte(const std::uint8_t* payload, std::uint64_t size,
                                                      RangeCursor& c)
{
    return c.offset < size ? static_cast<std::uint32_t>(payload[c.offset++]) : 0u;
}

__global__ void range_start_kernel(const std::uint8_t* __restrict__ bytes,
                                   const std::uint64_t* __restrict__ offsets,
                                   const std::uint64_t* __restrict__ sizes, RangeCursor* cursors,
                                   int streams, unsigned* error_word)
{
    const int s = blockIdx.x * blockDim.x + threadIdx.x;
    if (s >= streams)
        return;
    const std::uint8_t* payload = bytes + offsets[s];
    const std::uint64_t size = sizes[s];
    RangeCursor c{INITIAL_RANGE, 0u, 0u, 0u};
    c.code = payload_byte(payload, size, c) << 16;
    c.code |= payload_byte(payload, size, c) << 8;
    c.code |= payload_byte(payload, size, c);
    if (c.code >= c.range)
    {
        c.status = 1;
        if (error_word)
            atomicOr(error_word, error_range);
    }
    cursors[s] = c;
}

// One symbol of 1024 from the left-child masses of its bisection heap.
// Returns false (and leaves the cursor's status at 1) when the code leaves
// its interval.
__device__ bool decode_symbol(const std::uint8_t* payload, std::uint64_t size, RangeCursor& c,
                              const float* left_masses, std::uint16_t& symbol)
{
    int node = 0, base = 0, count = 1024;
    float mass = 1.0f;
#pragma unroll 1
    while (count > 1)
    {
        const int half = count / 2;
        const float left = left_masses[node];
        const std::uint32_t p0 = conditional_q15(left, mass);
        const auto range0 = static_cast<std::uint32_t>((static_cast<std::uint64_t>(c.range) * p0) >> 15);
        if (c.code >= range0)
        {
            c.code -= range0;
            c.range -= range0;
            base += half;
            count -= half;
            mass = ftz_sub(mass, left);
            node = 2 * node + 2;
        }
        else
        {
            c.range = range0;
            count = half;
            mass = left;
            node = 2 * node + 1;
        }
#pragma unroll 1
        while (c.range < MINIMUM_RANGE)
        {
            c.range <<= 8;
            c.code = (c.code << 8) + payload_byte(payload, size, c);
        }
        if (c.code >= c.range)
        {
            c.status = 1;
            return false;
        }
    }
    symbol = static_cast<std::uint16_t>(base);
    return true;
}

__global__ void __launch_bounds__(128)
    range_decode_kernel(const std::uint8_t* __restrict__ bytes, const std::uint64_t* __restrict__ offsets,
                        const std::uint64_t* __restrict__ sizes, RangeCursor* cursors, int streams,
                        const int* __restrict__ rows, int count, const float* __restrict__ masses,
                        std::uint16_t* __restrict__ symbols, unsigned* error_word)
{
    const int s = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (s >= streams)
        return;
    const std::uint8_t* payload = bytes + offsets[s];
    const std::uint64_t size = sizes[s];
    RangeCursor c = cursors[s];
    const bool was_running = c.status == 0;
    for (int r0 = 0; r0 < count; r0 += 32)
    {
        const int r = r0 + lane;
        unsigned mine = __ballot_sync(0xffffffffu, r < count && rows[r] == s);
        if (lane == 0)
        {
            while (mine)
            {
                const int row = r0 + __ffs(mine) - 1;
                mine &= mine - 1;
                std::uint16_t symbol = 0;
                if (c.status == 0)
                    decode_symbol(payload, size, c, masses + static_cast<size_t>(row) * 1023, symbol);
                symbols[row] = c.status == 0 ? symbol : 0;
            }
        }
    }
    if (lane == 0)
    {
        cursors[s] = c;
        if (was_running && c.status != 0 && error_word)
            atomicOr(error_word, error_range);
    }
}
} // namespace

void range_start(const std::uint8_t* bytes, const std::uint64_t* offsets, const std::uint64_t* sizes,
                 RangeCursor* cursors, int streams, unsigned* error_word, cudaStream_t stream)
{
    if (streams <= 0)
        return;
    range_start_kernel<<<(streams + 127) / 128, 128, 0, stream>>>(bytes, offsets, sizes, cursors, streams,
                                                                  error_word);
    note_launch();
}

void range_decode(const std::uint8_t* bytes, const std::uint64_t* offsets, const std::uint64_t* sizes,
                  RangeCursor* cursors, int streams, const int* rows, int count, const float* masses,
                  std::uint16_t* symbols, unsigned* error_word, cudaStream_t stream)
{
    if (streams <= 0 || count <= 0)
        return;
    range_decode_kernel<<<(streams + 3) / 4, 128, 0, stream>>>(bytes, offsets, sizes, cursors, streams, rows,
                                                              count, masses, symbols, error_word);
    note_launch();
}
} // namespace tsacb::dev
