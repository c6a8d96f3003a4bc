// Host-side launch interface of the BF8L quantized linear kernels.
#pragma once
#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

#include "kernels/row_meta.hpp"

namespace tsacb::dev
{
// Fused QKV epilogue: rotary on q and k, then q to `query` [row][512] and k,
// v to the caches at the row's slot (the rotary_scatter operations).
struct QkvScatter
{
    const RowMeta* meta = nullptr; // null: plain output to y
    const std::uint16_t* rotations = nullptr;
    std::uint16_t* query = nullptr;
    std::uint16_t* cache_k = nullptr;
    std::uint16_t* cache_v = nullptr;
};

struct QLinearArgs
{
    const std::int8_t* weights = nullptr;     // [n][k] int8
    const float* weight_scales = nullptr;     // [k/256][n]
    const float* bias = nullptr;              // [n]
    const std::int8_t* xq = nullptr;          // [m][k] quantized activations
    const float* xscale = nullptr;            // [m][k/256]
    const std::uint16_t* residual = nullptr;  // [m][residual_stride] bf16, added after rounding
    const std::uint16_t* lut = nullptr;       // bf16 -> bf16 map applied last (GELU)
    std::uint16_t* y = nullptr;               // [m][n] bf16
    int m = 0, n = 0, k = 0;
    int residual_stride = -1;                 // elements per residual row; -1: n, 0: one row for all
    QkvScatter qkv;                           // only where qlinear_qkv_fusable
    unsigned* error_word = nullptr;           // the GEMM's bounded waits report here
};

// True when the decode-shaped kernel can apply the fused QKV epilogue.
bool qlinear_qkv_fusable(int m, int n);

// Bytes of scratch holding the quantized activations of m columns of k inputs.
size_t qlinear_scratch_bytes(size_t m, size_t k);
// BF8L quantization of bf16 activations [m][k] into int8 + per-block scales.
void qlinear_quantize(const std::uint16_t* x, int m, int k, std::int8_t* xq, float* xscale,
                      unsigned* error_word, cudaStream_t stream);
// Exact int8 block dots + ordered FP32 epilogue: int8 mma.sync split-K tiles
// for decode-sized m, the tcgen05 GEMM (qlinear_tc.cu) from 256 rows.
bool qlinear_uses_gemm(int m, int n, int k);
void qlinear_matmul(const QLinearArgs& args, cudaStream_t stream);
// One-time kernel attribute setup (dynamic shared memory limits).
void qlinear_init();
} // namespace tsacb::dev
