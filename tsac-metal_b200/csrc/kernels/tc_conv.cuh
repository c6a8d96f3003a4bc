// Tensor-core (tcgen05) convolution for DAC synthesis.
//
// Decoded PCM is compared with the reference within a tolerance rather than
// bit for bit, so the decoder's convolutions run as implicit GEMMs on the
// 5th-generation tensor cores instead of the exact serial chains the encoder
// needs.  Precision: each fp32 operand is split into two TF32 values,
// hi = nearest TF32 of x and lo = nearest TF32 of x - hi, and each product is
// formed as hi*hi + hi*lo + lo*hi with fp32 accumulation in TMEM: at most
// about 3 * 2^-22 relative error per product.
//
// Layout ("padded rows"): activations are [row][channel] fp32 with every
// sequence (decoder chunk) followed by zero rows, so a tap that reaches past a
// sequence edge reads zeros and the GEMM needs no per-sequence bounds.  At a
// stage with cumulative upsampling S, padded row o belongs to padded latent
// row o / S, and valid[o / S] says whether it is a real frame; the epilogue
// writes zeros at the other rows, keeping the gaps zero for the next layer.
//
// Geometry of one launch (ordinary and transposed convolutions alike): output
// row out_stride*i + phase receives, for tap t of `taps`,
//   x[i + row_shift[phase] + t*tap_step] . W[phase*taps + t]
// over all input channels; W is [slice][cout][cin] (cin fastest).  An ordinary
// convolution is one phase with row_shift = -padding, tap_step = dilation; a
// transposed convolution of stride s (kernel 2s, padding s/2) is s phases of
// two taps each, tap_step = -1.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace tsacb::dev
{
struct TcConvGeometry
{
    long long rows;    // i range: [0, rows)
    int cin, cout;
    int taps;          // taps per phase
    int phases;        // 1, or the transposed stride
    int out_stride;    // 1, or the transposed stride
    int tap_step;      // input-row step between taps
    int row_shift[8];  // per phase
    long long out_rows;  // rows of the output tensors
    long long in_rows;   // rows of the input tensors
    int out_scale;     // output rows per padded latent row
};

struct TcConvEpilogue
{
    const float* bias;          // [cout] (this and the alpha arrays 16-byte aligned)
    const float* residual;      // [out_rows][cout] or null (may alias raw)
    float* raw;                 // [out_rows][cout] or null: bias + sum (+ residual)
    const float* alpha;         // next Snake's alpha [cout], or null (no Snake)
    const float* alpha_inverse; // 1 / (alpha + eps) [cout] (with alpha)
    float* hi;                  // [out_rows][cout] or null: Snake(raw) head (or full value)
    float* lo;                  // [out_rows][cout] or null: Snake(raw) tail; null = no split
    const unsigned char* valid; // [padded latent rows]
    unsigned* error_word;
};

// Operands: input head/tail [in_rows][cin]; weight head/tail [slices][cout][cin].
struct TcConvOperands
{
    const float* x_hi;
    const float* x_lo;
    const float* w_hi;
    const float* w_lo;
};

// Supported shapes: cin % 32 == 0, cout one of 1536, 768, 384, 192, 96 (or a
// multiple of 128 or 96), taps * phases <= 16, phases <= 8.
bool tc_conv_supported(int cin, int cout);
// Throws a device error (via the returned status) when the tensor maps cannot
// be encoded; launches nothing in that case.
cudaError_t tc_conv(const TcConvOperands& op, const TcConvGeometry& g, const TcConvEpilogue& e,
                    cudaStream_t stream);

// Copies packed rows into the padded layout, split into head and tail (or
// whole into `hi` when lo is null): dst row row_map[r] <- src row r.
void pad_split_rows(const float* src, long long rows, int channels, const long long* row_map,
                    float* hi, float* lo, cudaStream_t stream);
} // namespace tsacb::dev
