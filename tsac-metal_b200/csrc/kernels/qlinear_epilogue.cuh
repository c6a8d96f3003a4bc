// Output rule of the quantized linear kernels (qlinear.cu, qlinear_tc.cu):
// out = bf16(sum + bias[o]), then the fused passes the reference runs
// separately: + residual with bf16 rounding (probability_add_bf16,
// src/common/probability.cpp:7-12) and a bf16 -> bf16 lookup (GELU).
#pragma once
#include <cstdint>

#include "kernels/numeric.cuh"

namespace tsacb::dev
{
struct Epilogue
{
    const float* bias;
    const std::uint16_t* residual; // [M][residual_stride] or null
    const std::uint16_t* lut;      // 65536-entry bf16 map or null
    int residual_stride;           // 0: one residual row for every column
};

// finish() with the bias and the residual value already loaded.
__device__ __forceinline__ std::uint16_t finish_loaded(float sum, float bias, bool has_residual,
                                                       std::uint16_t residual, const std::uint16_t* lut)
{
    std::uint16_t y = to_bf16(__fadd_rn(sum, bias));
    if (has_residual)
        y = to_bf16(__fadd_rn(from_bf16(residual), from_bf16(y)));
    if (lut)
        y = lut[y];
    return y;
}

// finish() with the bias value already loaded.
__device__ __forceinline__ std::uint16_t finish_with_bias(float sum, float bias, int m, int n, const Epilogue& e)
{
    std::uint16_t y = to_bf16(__fadd_rn(sum, bias));
    if (e.residual)
    {
        y = to_bf16(__fadd_rn(from_bf16(e.residual[static_cast<size_t>(m) * e.residual_stride + n]),
                              from_bf16(y)));
    }
    if (e.lut)
    {
        y = e.lut[y];
    }
    return y;
}

__device__ __forceinline__ std::uint16_t finish(float sum, int m, int n, const Epilogue& e)
{
    std::uint16_t y = to_bf16(__fadd_rn(sum, e.bias[n]));
    if (e.residual)
    {
        y = to_bf16(__fadd_rn(from_bf16(e.residual[static_cast<size_t>(m) * e.residual_stride + n]),
                              from_bf16(y)));
    }
    if (e.lut)
    {
        y = e.lut[y];
    }
    return y;
}

} // namespace tsacb::dev
