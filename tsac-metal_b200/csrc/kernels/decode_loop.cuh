// Device side of the GPU-resident decode loop.
//
// The decode loop runs the probability model one (step, codebook) at a time
// for every lane of every recording in a batch (TransformerPredictor's decode
// order, src/common/transformer.cpp:26-166, over the entropy order of
// src/format/entropy.cpp:26-55) and range-decodes each row's symbol from its
// left-child masses.  Everything a step needs lives on the device: the
// decoded tokens (the batch token array, in each recording's final
// [frame][group][book] layout), the range decoders' cursors, and a step
// clock.  A step's row inputs (cache slots, positions, which tokens feed the
// embeddings, where the decoded symbol goes) are computed on the device by
// decode_setup from the clock, so one captured graph per (book, active lanes)
// shape serves every step and the host never waits between steps.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

#include "kernels/row_meta.hpp"

namespace tsacb::dev
{
// One entropy lane x channel group of a recording.
struct DecodeLane
{
    int recording;  // index of the recording's range decoder
    int group, groups, books;
    int start;      // first frame of the lane
    int tslot;      // first temporal cache slot (1024 per lane)
    int cslot;      // first codebook cache slot (books per lane)
    int token_base; // batch token index of the recording's token [0][0][0]
};

// step_now: the step of the (step, book) pair being computed; next_step: the
// step the next book-0 launch starts.
struct DecodeClock
{
    int step_now, next_step;
};

// Per-step row inputs, written by decode_setup and read by the step's kernels.
struct DecodeStepRows
{
    // temporal stack (book 0 only): rows_per_lane rows per active lane
    RowMeta* temporal_meta;
    int* temporal_offsets; // batch token index of each row's feedback tokens
    int* temporal_counts;  // books summed into its embedding
    int* cond_source;      // per active lane: its last temporal row
    int* cond_lane;        // per active lane: its lane index
    // codebook stack: one row per active lane
    RowMeta* codebook_meta;
    int* codebook_lane;    // lane index (conditioning row) of each row
    int* codebook_book;    // the book (position row) of each row
    int* codebook_offsets; // batch token index of the frame's book-0 token
    int* codebook_counts;  // prefix books summed into the input embedding
    int* destination;      // batch token index receiving the row's symbol
};

// Fills `out` for the rows of one (step, book): `row_lane` lists the active
// lanes (rows) in stream order.  For book 0 it first advances the clock.
// Temporal rows: one per lane at position step_position[step], or, when
// rows_per_lane == replay (256), the lane's replay of its last 256 frames at
// positions 0..255 (TransformerPredictor's context reset, transformer.cpp:112-125).
// zero_row: batch token index of 12 zero tokens (the feedback before frame 0).
void decode_setup(const DecodeLane* lanes, const int* row_lane, int rows, int book, int rows_per_lane,
                  const int* step_position, DecodeClock* clock, int zero_row, DecodeStepRows out,
                  cudaStream_t stream);
} // namespace tsacb::dev
