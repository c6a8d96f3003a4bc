// Fused codebook step of the Transformer decoder (one launch per step).
//
// A codebook step (every decode step except the first of each frame) runs the
// 3-layer codebook stack, the logits projection and the softmax/bisection
// masses for every active lane; the lanes are independent rows.  Here a
// cluster of 4 CTAs (one per attention head) carries up to 8 rows through
// the whole step: LayerNorm and BF8L are computed per CTA on full rows, each
// linear's outputs are split over the 4 CTAs, head c's attention stays in CTA
// c, and the slices meet through distributed shared memory between cluster
// barriers.  Every element is computed with the same device routines and in
// the same order as the standalone kernels (row_ops.cuh, qlinear.cu), so the
// masses are bit-identical.  Opt-in (TSAC_CUDA_FUSED_CODEBOOK=1): on B200 the
// separate kernels remain faster at the tested batch sizes, because here each
// cluster walks ~30 dependent phases on 4 SMs while they spread every phase
// over the whole GPU.
#pragma once
#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

#include "kernels/row_meta.hpp"

namespace tsacb::dev
{
struct CodebookLinear
{
    const std::int8_t* weights; // [N][K]
    const float* scales;        // [K/256][N]
    const float* bias;          // [N]
};

struct CodebookStepArgs
{
    int rows; // active lanes of the step
    int book; // codebook of the step
    // book 0: h[j] = cond[lane_rows[j]] + positions[books[j]]
    const std::uint16_t* cond;
    const int* lane_rows;
    // book > 0: h[j] = proj61(embed_sum(tokens of the earlier books)) + positions[books[j]]
    const std::uint16_t* embeddings;
    const std::uint16_t* tokens;
    const int* offsets;
    const int* counts;
    CodebookLinear proj61;
    const std::uint16_t* positions;
    const int* books;
    CodebookLinear layer[3][4];          // QKV, attention out, FFN in (GELU), FFN out
    const std::uint16_t* norm_gain[7];   // ln1, ln2 of layers 0..2, then the final norm
    const std::uint16_t* norm_bias[7];
    CodebookLinear proj62;               // logits
    const std::uint16_t* gelu;           // bf16 -> bf16 table
    const RowMeta* meta;                 // per row: slot, base, time (rotary unused: -1)
    std::uint16_t* cache_k;              // [layer][slot][512]
    std::uint16_t* cache_v;
    std::size_t cache_stride;            // elements per layer
    float* tree;                         // [rows][1023] left-child masses
    unsigned* error_word;
};

// Rows one cluster carries, and whether a step fits the fused kernel.
constexpr int CODEBOOK_STEP_ROWS = 8;
void codebook_step(const CodebookStepArgs& args, cudaStream_t stream);
} // namespace tsacb::dev
