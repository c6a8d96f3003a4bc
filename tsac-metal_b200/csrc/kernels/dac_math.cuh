// Elementwise DAC arithmetic shared by the exact kernels and the tensor-core
// synthesis epilogue: the captured sine-squared polynomial and Snake
// (src/scalar/dsp.cpp:55-119; epsilon 0x3089705f, src/weights/normalization.hpp:9).
#pragma once
#include <climits>
#include <cuda_runtime.h>

namespace tsacb::dev
{
// Two-constant reduction of `phase` by its quadrant (the nearest integer to
// phase * 2/pi): x = phase - quadrant * pi/2, |x| <= pi/4.
__device__ __forceinline__ float reduce_quadrant(float phase, float quadrant)
{
    const float x = __fmaf_rn(quadrant, __uint_as_float(0xbfc90000u), phase);
    return __fmaf_rn(quadrant, __uint_as_float(0xb9fdaa22u), x);
}

// sin(x) and cos(x) on the reduced interval (x2 = x * x).
__device__ __forceinline__ float sine_reduced(float x, float x2)
{
    float p = __fmaf_rn(__uint_as_float(0xb94ca1f9u), x2, __uint_as_float(0x3c08839eu));
    p = __fmaf_rn(p, x2, __uint_as_float(0xbe2aaaa3u));
    const float cube = __fmul_rn(x, x2);
    return __fmaf_rn(cube, p, x);
}

__device__ __forceinline__ float cosine_reduced(float x2)
{
    float p = __fmaf_rn(__uint_as_float(0x37ccf5ceu), x2, __uint_as_float(0xbab6061au));
    p = __fmaf_rn(p, x2, __uint_as_float(0x3d2aaaa5u));
    p = __fmaf_rn(p, x2, __uint_as_float(0xbf000000u));
    return __fmaf_rn(p, x2, 1.0f);
}

// sin^2 of `phase` given its quadrant and that quadrant's parity: the odd or
// even polynomial of the reduced argument, squared.
__device__ __forceinline__ float sine_squared_reduced(float phase, float quadrant, bool odd)
{
    const float x = reduce_quadrant(phase, quadrant);
    const float x2 = __fmul_rn(x, x);
    const float value = odd ? cosine_reduced(x2) : sine_reduced(x, x2);
    return __fmul_rn(value, value);
}

__device__ __forceinline__ float sine_squared(float phase)
{
    const float reduced = __fmul_rn(phase, __uint_as_float(0x3f22f983u));
    const float quadrant = rintf(reduced); // ties to even
    const int q = (quadrant >= -2147483648.0f && quadrant < 2147483648.0f)
                      ? static_cast<int>(quadrant)
                      : INT_MIN;
    return sine_squared_reduced(phase, quadrant, (q & 1) != 0);
}

// Snake: v + sin^2(alpha v) / (alpha + eps), each operation rounded.
__device__ __forceinline__ float snake_value(float v, float alpha)
{
    const float eps = __uint_as_float(0x3089705fu);
    const float phase = __fmul_rn(alpha, v);
    return __fadd_rn(v, __fdiv_rn(sine_squared(phase), __fadd_rn(alpha, eps)));
}
} // namespace tsacb::dev
