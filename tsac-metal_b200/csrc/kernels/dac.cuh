// Launch interface of the DAC (analysis / synthesis) and RVQ kernels.
//
// Activations are [frames][channels] float32 (channels fastest), as in the
// reference's Signal.  A launch covers several independent sequences
// (recording chunks, recordings of a batch) laid end to end; each sequence is
// zero-padded at its own boundaries exactly as a separate reference call.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace tsacb::dev
{
struct Sequence
{
    int in_offset;   // first input frame (row) of the sequence
    int in_frames;   // input frames
    int out_offset;  // first output frame (row)
    int out_frames;  // output frames
};

struct ConvShape
{
    int cin, cout, kernel, stride, padding, dilation;
    bool transposed;
};

// y = x + sin^2(alpha x) / (alpha + eps) per element (captured polynomial).
void snake(const float* x, const float* alpha, int channels, long long frames, float* y,
           unsigned* error_word, cudaStream_t stream);

// Exact-order convolution: per output, sum = sum + x*w over (valid tap, in
// channel) with the product and the add each rounded, then + bias, then
// optionally residual + result.  `tiles` is built by conv_tiles().
// weights: ordinary [out][tap][in]; transposed [in][tap][out].
struct ConvLaunch
{
    unsigned* error_word;
    const float* x;
    const float* weights;
    const float* bias;
    const float* residual; // same shape as y, or null
    float* y;              // raw result, or null when only `act` is wanted
    const Sequence* sequences;
    const int4* tiles; // {sequence, first output frame (per phase for transposed), phase, 0}
    int tile_count;
    ConvShape shape;
    const float* alpha = nullptr; // next layer's Snake alpha [cout], with act
    float* act = nullptr;         // Snake(result) (same shape as y), or null
    // Fused multiply-add chains instead of the exact separately rounded ones
    // (the certified fast analysis; its RVQ decisions are checked).
    bool fast = false;
};
void conv1d(const ConvLaunch& launch, cudaStream_t stream);
// Output channels < 16 (DAC exit to PCM): one serial chain per output.
// `tiles` = sum over sequences of ceil(out_frames / 128): with it (and the
// input window within shared memory) a CTA stages 128 frames' inputs and
// weights once; 0 runs one thread per output reading global memory.
void conv1d_narrow(const float* x, const float* w, const float* bias, float* y,
                   const Sequence* sequences, int sequence_count, const ConvShape& shape,
                   long long total_outputs, unsigned* error_word, cudaStream_t stream,
                   long long tiles = 0);
// Frames per output tile along time (the tile table granularity).
int conv_tile_frames(const ConvShape& shape);

// RVQ encode: latent [frames][1024] -> tokens [frames][books] (row stride
// `token_stride`); the latent is consumed as the residual.
struct RvqBookDevice
{
    const float* input_weights;  // [8][1024]
    const float* input_bias;     // [8]
    const float* search;         // [1024][8]
    const float* codebook;       // [1024][8]
    const float* output_weights; // [1024][8]
    const float* output_bias;    // [1024]
};
void rvq_encode(const float* latent, int frames, const RvqBookDevice* books, int book_count,
                std::uint16_t* tokens, int token_stride, unsigned* error_word,
                cudaStream_t stream);
// rvq_encode that also sets uncertain[frame] = 1 when any book's winning
// similarity leads the runner-up by less than `margin` (0 otherwise).
void rvq_encode_margins(const float* latent, int frames, const RvqBookDevice* books, int book_count,
                        std::uint16_t* tokens, int token_stride, float margin, unsigned char* uncertain,
                        unsigned* error_word, cudaStream_t stream);
// RVQ decode: tokens [frames][books] (row stride token_stride) -> latent [frames][1024].
void rvq_decode(const std::uint16_t* tokens, int token_stride, int frames,
                const RvqBookDevice* books, int book_count, float* latent, cudaStream_t stream);
// Nonfinite scan of a float tensor: sets error bit on any NaN/Inf.
void check_finite(const float* x, long long count, unsigned* error_word, cudaStream_t stream);

// padded_audio (src/common/audio_analyzer.cpp:118-139) on the device:
// dst[(g*padded + f)*mc + c] = src[(g*mc + c)*channel_stride + f*sample_stride]
// for f < samples, zero up to `padded`; nonfinite input sets the error bit.
void pcm_regroup(const float* src, long long samples, long long channel_stride,
                 long long sample_stride, int groups, int model_channels, long long padded,
                 float* dst, unsigned* error_word, cudaStream_t stream);
} // namespace tsacb::dev
