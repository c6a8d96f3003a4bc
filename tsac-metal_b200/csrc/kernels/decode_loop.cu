// Row inputs of one decode (step, book), computed on the device from the
// step clock (decode_loop.cuh).  What each row reads restates the reference's
// decode bookkeeping (reference project paths):
//   feedback = the previous frame's tokens, zeros before frame 0,
//   context reset + replay of the last 256 frames  src/common/transformer.cpp:26-166
//   codebook input = prefix of the frame's tokens   src/common/cpu_transformer.tpp:356-373
//   replay rows' value sums rounded                 src/scalar/attention.cpp:128
#include "kernels/decode_loop.cuh"
#include "kernels/launch_count.hpp"
#include "kernels/pdl.cuh"

namespace tsacb::dev
{
namespace
{
constexpr int setup_threads = 256;

__global__ void __launch_bounds__(setup_threads)
    decode_setup_kernel(const DecodeLane* __restrict__ lanes, const int* __restrict__ row_lane, int rows,
                        int book, int rows_per_lane, const int* __restrict__ step_position,
                        DecodeClock* clock, int zero_row, DecodeStepRows out)
{
    pdl_prologue();
    __shared__ int step;
    if (threadIdx.x == 0)
    {
        if (book == 0)
        {
            step = clock->next_step;
            clock->step_now = step;
            clock->next_step = step + 1;
        }
        else
        {
            step = clock->step_now;
        }
    }
    __syncthreads();
    for (int j = threadIdx.x; j < rows; j += setup_threads)
    {
        const int lane_index = row_lane[j];
        const DecodeLane lane = lanes[lane_index];
        const int frame = lane.start + step;
        const int frame_tokens = lane.groups * lane.books; // tokens per frame of the recording
        const int base = lane.token_base + (frame * lane.groups + lane.group) * lane.books;
        out.codebook_meta[j] = RowMeta{lane.cslot + book, lane.cslot, book + 1, -1, 0};
        out.codebook_lane[j] = lane_index;
        out.codebook_book[j] = book;
        out.codebook_offsets[j] = base;
        out.codebook_counts[j] = book;
        out.destination[j] = base + book;
        if (book != 0)
            continue;
        out.cond_lane[j] = lane_index;
        out.cond_source[j] = j * rows_per_lane + rows_per_lane - 1;
        if (rows_per_lane == 1)
        {
            const int position = step_position[step];
            out.temporal_meta[j] = RowMeta{lane.tslot + position, lane.tslot, position + 1, position,
                                           position + 1 > 64 ? 1 : 0};
            out.temporal_offsets[j] = step == 0 ? zero_row : base - frame_tokens;
            out.temporal_counts[j] = lane.books;
        }
    }
    if (book != 0 || rows_per_lane == 1)
        return;
    // Replay: row (j, k) re-evaluates frame frame - rows_per_lane + k at position k.
    for (int i = threadIdx.x; i < rows * rows_per_lane; i += setup_threads)
    {
        const int j = i / rows_per_lane, k = i % rows_per_lane;
        const DecodeLane lane = lanes[row_lane[j]];
        const int source = lane.start + step - rows_per_lane + k;
        out.temporal_meta[i] = RowMeta{lane.tslot + k, lane.tslot, k + 1, k, 1};
        out.temporal_offsets[i] = lane.token_base + (source * lane.groups + lane.group) * lane.books;
        out.temporal_counts[i] = lane.books;
    }
}
} // namespace

void decode_setup(const DecodeLane* lanes, const int* row_lane, int rows, int book, int rows_per_lane,
                  const int* step_position, DecodeClock* clock, int zero_row, DecodeStepRows out,
                  cudaStream_t stream)
{
    if (rows <= 0)
        return;
    launch_pdl(decode_setup_kernel, dim3(1), dim3(setup_threads), 0, stream, lanes, row_lane, rows, book,
               rows_per_lane, step_position, clock, zero_row, out);
    note_launch();
}
} // namespace tsacb::dev
