// Launch interface of the tcgen05 int8 GEMM for quantized linear layers with
// many rows (qlinear_tc.cu).
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

#include "kernels/qlinear_epilogue.cuh"

namespace tsacb::dev
{
// True when the GEMM handles (m rows, n outputs, k inputs): at least one
// 128-row tile, n a multiple of 128, k a multiple of 256.
bool qlinear_tc_supported(int m, int n, int k);
// y [m][n] = the quantized linear of xq [m][k] (scales xscale [m][k/256]) with
// weights [n][k] (scales weight_scales [k/256][n]); 16-byte aligned operands.
cudaError_t qlinear_tc(const std::int8_t* weights, const float* weight_scales, const std::int8_t* xq,
                       const float* xscale, int m, int n, int k, const Epilogue& e, std::uint16_t* y,
                       unsigned* error_word, cudaStream_t stream);
} // namespace tsacb::dev
