// Device range decoding of normal-stream symbols, restating (reference
// project paths):
//   RangeDecoder read / start / get   src/format/range.cpp:118-157
//   decode_categorical (tree walk)    src/format/categorical.cpp:119-142,
//                                     with the left-child masses the softmax
//                                     kernel emits (heap order, right mass =
//                                     path mass - left, never re-summed);
//                                     the decision arithmetic and the walk
//                                     are range_core.hpp's, shared with the
//                                     host decoder
//   the Metal serialized decoder      src/metal/probability/range.metal:12-77
//
// B200 mapping: a stream's symbols are one serial chain (each decision's
// renormalisation decides which payload byte the next reads), so a stream is
// one lane; streams (recordings) are independent, one warp each.  The warp
// finds its rows with ballots over the row list, in row order, and lane 0
// walks them.  Every loop is bounded: 10 decisions per symbol and at most
// three renormalising shifts per decision (range >= 1 after any split).
#include "kernels/async_copy.cuh"
#include "kernels/error_bits.hpp"
#include "kernels/launch_count.hpp"
#include "kernels/numeric.cuh"
#include "kernels/pdl.cuh"
#include "kernels/range_decode.cuh"
#include "kernels/row_ops.cuh"
#include "range_core.hpp"

namespace tsacb::dev
{
namespace
{
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
    RangeCursor c{range::initial_range, 0u, 0u, 0u};
    for (int i = 0; i < 3; ++i)
        c.code = (c.code << 8) | payload_byte(payload, size, c);
    if (c.code >= c.range)
    {
        c.status = 1;
        if (error_word)
            atomicOr(error_word, error_range);
    }
    cursors[s] = c;
}

struct DeviceMath
{
    static __device__ __forceinline__ std::uint16_t q15(float left, float mass)
    {
        return conditional_q15(left, mass);
    }
    static __device__ __forceinline__ float sub(float a, float b)
    {
        return ftz_sub(a, b);
    }
};

// A stream's decoder inside one kernel: its window and payload cursor.
struct StreamDecoder
{
    range::DecodeWindow w;
    const std::uint8_t* payload;
    std::uint64_t size;
    std::uint64_t at;

    __device__ __forceinline__ std::uint32_t next_byte()
    {
        return at < size ? static_cast<std::uint32_t>(payload[at++]) : 0u;
    }
    __device__ __forceinline__ int node(std::uint32_t p0, int)
    {
        return range::decide(w, p0, *this);
    }
};

// One symbol of 1024 from the left-child masses of its bisection heap (the
// walk and the decision arithmetic of range_core.hpp, as the host decoder).
// Returns false (and sets the cursor's status to 1) when the code leaves its
// interval.
__device__ __forceinline__ bool decode_symbol(const std::uint8_t* payload, std::uint64_t size,
                                              RangeCursor& c, const float* left_masses,
                                              std::uint16_t& symbol)
{
    StreamDecoder d{{c.range, c.code}, payload, size, c.offset};
    const int s = range::walk_bisection<DeviceMath>(left_masses, d);
    c.range = d.w.range;
    c.code = d.w.code;
    c.offset = static_cast<std::uint32_t>(d.at);
    if (s < 0)
    {
        c.status = 1;
        return false;
    }
    symbol = static_cast<std::uint16_t>(s);
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
// The decode loop's range decoding: one warp per stream (recording), whose
// rows of this step are rows [row_begin[s], row_begin[s + 1]) in stream
// order.  The warp first stages, with coalesced loads, the next 128 payload
// bytes from its cursor (a step consumes a few bytes per row) and the
// left-child masses of up to four rows; lane 0 then walks the rows' bisection
// heaps from shared memory, reading payload bytes from the staged window
// (global memory only past it).  Each symbol goes to tokens[destination[row]],
// where the next step's embeddings read it.
constexpr int rows_warps = 2, staged_rows = 4, window_bytes = 128;

struct WindowedDecoder
{
    range::DecodeWindow w;
    const std::uint8_t* payload;
    const std::uint8_t* window; // payload bytes [window_start, window_start + window_bytes)
    std::uint64_t size, window_start, at;

    __device__ __forceinline__ std::uint32_t next_byte()
    {
        std::uint32_t byte = 0;
        if (at < size)
            byte = at - window_start < window_bytes ? window[at - window_start] : payload[at];
        ++at;
        return byte;
    }
    __device__ __forceinline__ int node(std::uint32_t p0, int)
    {
        return range::decide(w, p0, *this);
    }
};

__global__ void __launch_bounds__(rows_warps * 32)
    range_decode_rows_kernel(const std::uint8_t* __restrict__ bytes, const std::uint64_t* __restrict__ offsets,
                             const std::uint64_t* __restrict__ sizes, RangeCursor* cursors, int streams,
                             const int* __restrict__ row_begin, const float* __restrict__ masses,
                             const int* __restrict__ destination, std::uint16_t* __restrict__ tokens,
                             unsigned* error_word)
{
    __shared__ float staged[rows_warps][staged_rows * 1023 + 1];
    __shared__ std::uint8_t window[rows_warps][window_bytes];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int s = blockIdx.x * rows_warps + warp;
    // Before the dependency wait: the stream's cursor and payload window.
    // The cursor was last written by this stream's previous decoding (the
    // previous book of the step, or an earlier step), many launches back.
    // Every kernel completes only after its predecessor has, and this
    // kernel's predecessor (softmax_tree_kernel) lets it launch only after
    // passing its own wait, so that write is complete here.
    const bool active = s < streams && row_begin[s] != row_begin[s + 1];
    RangeCursor c{};
    const std::uint8_t* payload = nullptr;
    std::uint64_t size = 0;
    if (active)
    {
        payload = bytes + offsets[s];
        size = sizes[s];
        c = cursors[s];
#pragma unroll
        for (int i = lane; i < window_bytes; i += 32)
            window[warp][i] = c.offset + i < size ? payload[c.offset + i] : 0;
    }
    pdl_prologue();
    if (!active)
        return;
    const int first = row_begin[s], last = row_begin[s + 1];
    const bool was_running = c.status == 0;
    WindowedDecoder d{{c.range, c.code}, payload, window[warp], size, c.offset, c.offset};
    for (int r0 = first; r0 < last; r0 += staged_rows)
    {
        const int n = last - r0 < staged_rows ? last - r0 : staged_rows;
        const float* m = masses + static_cast<size_t>(r0) * 1023;
        // Every lane's copies in flight together, then one wait.
        for (int i = lane; i < n * 1023; i += 32)
            cp_async_4(&staged[warp][i], m + i);
        cp_async_wait_all();
        __syncwarp();
        if (lane == 0)
        {
            for (int j = 0; j < n; ++j)
            {
                int symbol = 0;
                if (c.status == 0)
                {
                    symbol = range::walk_bisection<DeviceMath>(staged[warp] + j * 1023, d);
                    if (symbol < 0)
                    {
                        c.status = 1;
                        symbol = 0;
                    }
                }
                tokens[destination[r0 + j]] = static_cast<std::uint16_t>(symbol);
            }
        }
        __syncwarp();
    }
    if (lane == 0)
    {
        c.range = d.w.range;
        c.code = d.w.code;
        c.offset = static_cast<std::uint32_t>(d.at);
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
void range_decode_rows(const std::uint8_t* bytes, const std::uint64_t* offsets, const std::uint64_t* sizes,
                       RangeCursor* cursors, int streams, const int* row_begin, const float* masses,
                       const int* destination, std::uint16_t* tokens, unsigned* error_word, cudaStream_t stream)
{
    if (streams <= 0)
        return;
    launch_pdl(range_decode_rows_kernel, dim3((streams + rows_warps - 1) / rows_warps), dim3(rows_warps * 32), 0,
               stream, bytes, offsets, sizes, cursors, streams, row_begin, masses, destination, tokens,
               error_word);
    note_launch();
}
} // namespace tsacb::dev
