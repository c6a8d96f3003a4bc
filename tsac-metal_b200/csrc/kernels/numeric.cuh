// Device-side restatement of the codec's captured arithmetic.
//
// TSAC's bitstream is defined by specific float32 rounding boundaries, x86
// flush-to-zero at particular call sites, an integer round-to-nearest-even
// bf16 conversion, a bespoke exp polynomial and fixed reduction trees.  Every
// helper here spells its operations out with the IEEE round-to-nearest
// intrinsics (__fadd_rn, __fmul_rn, __fmaf_rn, __fdiv_rn, __fsqrt_rn), and the
// library is compiled with -fmad=false -ftz=false, so nothing is contracted or
// flushed unless written here.
//
// Sources of each rule (reference project paths):
//   flush/add/subtract/multiply/divide  src/common/numeric/float_math.hpp:33-61
//   bf16 conversion                     src/common/numeric/bf16.hpp:9-18
//   original_exp                        src/common/numeric/probability.hpp:14-33
//   probability_sum / pair_sum          src/format/categorical.cpp:17-74
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

#include "kernels/error_bits.hpp"

namespace tsacb::dev
{
__device__ __forceinline__ float flush(float x)
{
    const unsigned bits = __float_as_uint(x);
    return (bits & 0x7f800000u) == 0 ? __uint_as_float(bits & 0x80000000u) : x;
}

__device__ __forceinline__ float ftz_add(float x, float y)
{
    return flush(__fadd_rn(flush(x), flush(y)));
}

__device__ __forceinline__ float ftz_sub(float x, float y)
{
    return flush(__fsub_rn(flush(x), flush(y)));
}

__device__ __forceinline__ float ftz_mul(float x, float y)
{
    return flush(__fmul_rn(flush(x), flush(y)));
}

__device__ __forceinline__ float ftz_div(float x, float y)
{
    return flush(__fdiv_rn(flush(x), flush(y)));
}

__device__ __forceinline__ std::uint16_t to_bf16(float value)
{
    const unsigned bits = __float_as_uint(value);
    return static_cast<std::uint16_t>((bits + 0x7fffu + ((bits >> 16) & 1u)) >> 16);
}

__device__ __forceinline__ float from_bf16(std::uint16_t value)
{
    return __uint_as_float(static_cast<unsigned>(value) << 16);
}

// exp(z) by range reduction n = rint(z*log2(e)), a two-constant Cody-Waite
// reduction, a degree-6 polynomial in FMA form and an exponent-field add of n.
// Inputs are clamped to [-88, 87]; a NaN input keeps its bits (n is INT_MIN,
// whose shifted value is 0 modulo 2^32).
__device__ __forceinline__ float original_exp(float z)
{
    z = 87.0f < z ? 87.0f : z;
    z = -88.0f > z ? -88.0f : z;
    const float exponent = __fmul_rn(z, 0x1.715476p+0f);
    const int n = isfinite(exponent) ? __float2int_rn(exponent) : INT_MIN;
    const float nf = static_cast<float>(n);
    z = __fmaf_rn(nf, -0x1.630000p-1f, z);
    z = __fmaf_rn(nf, 0x1.bd0106p-13f, z);
    float p = __fmaf_rn(0x1.a01a02p-13f, z, 0x1.6c16c2p-10f);
    p = __fmaf_rn(p, z, 0x1.111112p-7f);
    p = __fmaf_rn(p, z, 0x1.555556p-5f);
    p = __fmaf_rn(p, z, 0x1.555556p-3f);
    const float square = __fmul_rn(z, z);
    p = __fmaf_rn(p, z, 0.5f);
    z = __fmaf_rn(p, square, z);
    const float plus_one = __fadd_rn(z, 1.0f);
    return __uint_as_float(__float_as_uint(plus_one) + (static_cast<unsigned>(n) << 23));
}

// Balanced pair tree over a zero-padded block of `width` (8 or 64) values,
// every add flushed: the leaf reduction of probability_sum.
__device__ __forceinline__ float pair_sum_serial(const float* values, int count, int width)
{
    float v[64];
#pragma unroll 1
    for (int i = 0; i < width; ++i)
    {
        v[i] = i < count ? values[i] : 0.0f;
    }
#pragma unroll 1
    for (int w = width; w > 1;)
    {
        w /= 2;
#pragma unroll 1
        for (int i = 0; i < w; ++i)
        {
            v[i] = ftz_add(v[2 * i], v[2 * i + 1]);
        }
    }
    return v[0];
}

// Same 64-wide pair tree with one warp: lane i holds values 2i and 2i+1 of the
// (zero-padded) block.  Every lane returns the block sum.
__device__ __forceinline__ float warp_pair_sum64(float even, float odd)
{
    const unsigned full = 0xffffffffu;
    const int lane = threadIdx.x & 31;
    float s = ftz_add(even, odd); // level 1: 32 sums
#pragma unroll
    for (int width = 16; width >= 1; width >>= 1)
    {
        const float a = __shfl_sync(full, s, (2 * lane) & 31);
        const float b = __shfl_sync(full, s, (2 * lane + 1) & 31);
        s = ftz_add(a, b); // lanes < width hold the next level
    }
    return __shfl_sync(full, s, 0);
}

// Binary-carry accumulation of consecutive 64-value block sums, in block order,
// followed by the final fold over the carry slots (src/format/categorical.cpp:53-73).
__device__ __forceinline__ float carry_combine(const float* block_sums, int blocks)
{
    float partial[32];
#pragma unroll 1
    for (int i = 0; i < 32; ++i)
    {
        partial[i] = 0.0f;
    }
#pragma unroll 1
    for (int b = 1; b <= blocks; ++b)
    {
        float value = block_sums[b - 1];
        const int level = __ffs(b) - 1;
#pragma unroll 1
        for (int i = 0; i < level; ++i)
        {
            value = ftz_add(value, partial[i]);
            partial[i] = 0.0f;
        }
        partial[level] = value;
    }
    float value = partial[0];
    const int width = 32 - __clz(blocks);
#pragma unroll 1
    for (int i = 1; i < width; ++i)
    {
        value = ftz_add(value, partial[i]);
    }
    return value;
}

// The binary carry over 2^k block sums (k >= 1) leaves the total in slot k and
// zeros below it; the final fold then adds the zero slots and the total to
// partial[0] = 0, which reduces to ftz_add(0, balanced tree of the block sums).
// `tree` is that balanced tree, already flushed by its last ftz_add.
__device__ __forceinline__ float carry_fold_power_of_two(float tree)
{
    return ftz_add(0.0f, tree);
}

// probability_sum of `count` values in shared/global memory, one thread.
__device__ __forceinline__ float probability_sum_serial(const float* values, int count)
{
    if (count <= 8)
    {
        return pair_sum_serial(values, count, 8);
    }
    float sums[32];
    int blocks = 0;
#pragma unroll 1
    for (int offset = 0; offset < count; offset += 64)
    {
        const int n = count - offset < 64 ? count - offset : 64;
        sums[blocks++] = pair_sum_serial(values + offset, n, 64);
    }
    return carry_combine(sums, blocks);
}

// probability_sum of `count` (<= 2048) values in shared memory by one warp:
// block sums with the warp tree, carry combine on every lane.
__device__ __forceinline__ float warp_probability_sum(const float* values, int count)
{
    const int lane = threadIdx.x & 31;
    if (count <= 8)
    {
        float s = 0.0f;
        if (lane == 0)
        {
            s = pair_sum_serial(values, count, 8);
        }
        return __shfl_sync(0xffffffffu, s, 0);
    }
    float sums[32];
    int blocks = 0;
    for (int offset = 0; offset < count; offset += 64)
    {
        const int n = count - offset < 64 ? count - offset : 64;
        const float even = 2 * lane < n ? values[offset + 2 * lane] : 0.0f;
        const float odd = 2 * lane + 1 < n ? values[offset + 2 * lane + 1] : 0.0f;
        sums[blocks++] = warp_pair_sum64(even, odd);
    }
    return carry_combine(sums, blocks);
}

} // namespace tsacb::dev
