// Per-row device routines of the Transformer, shared by its kernels
// (transformer_ops.cu, attention.cu, qlinear.cu) and the device range
// decoder (range_decode.cu: conditional_q15), so every path runs the same
// operations in the same order.
//
// Reference arithmetic restated (reference project paths):
//   probability_layer_norm_bf16_into  src/common/probability.cpp:138-169
//   scalar::bf8l                      src/scalar/probability.cpp:16-40
//   scalar::Attention (one block)     src/scalar/attention.cpp:12-131
//   probability_softmax_bf16_into     src/common/probability.cpp:96-122
//   probability_sum / pair trees      src/format/categorical.cpp:17-74
//   conditional_q15                   src/format/categorical.cpp:76-89
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

#include "kernels/async_copy.cuh"
#include "kernels/numeric.cuh"
#include "kernels/row_meta.hpp"

namespace tsacb::dev
{
// ------------------------------------------------------------- LayerNorm --
// One warp per 512-wide row; lane l owns values [16l, 16l+16).  The 16-value
// lane partials are subtrees of the 64-wide pair tree, lanes 4i..4i+3 form
// 64-block i, and the eight block sums go through the binary carry.
__device__ __forceinline__ float lane_pair16(const float* v)
{
    float s[8];
#pragma unroll
    for (int i = 0; i < 8; ++i)
        s[i] = ftz_add(v[2 * i], v[2 * i + 1]);
#pragma unroll
    for (int i = 0; i < 4; ++i)
        s[i] = ftz_add(s[2 * i], s[2 * i + 1]);
#pragma unroll
    for (int i = 0; i < 2; ++i)
        s[i] = ftz_add(s[2 * i], s[2 * i + 1]);
    return ftz_add(s[0], s[1]);
}

__device__ __forceinline__ float warp_sum512(const float* v)
{
    float s = lane_pair16(v);
    s = ftz_add(s, __shfl_xor_sync(0xffffffffu, s, 1)); // 32-value subtrees
    s = ftz_add(s, __shfl_xor_sync(0xffffffffu, s, 2)); // 64-value block sums (lanes 4b..4b+3)
    // Eight block sums in block order: balanced tree over blocks, then the
    // carry's final fold (numeric.cuh: carry_fold_power_of_two).
    s = ftz_add(s, __shfl_xor_sync(0xffffffffu, s, 4));
    s = ftz_add(s, __shfl_xor_sync(0xffffffffu, s, 8));
    s = ftz_add(s, __shfl_xor_sync(0xffffffffu, s, 16));
    return carry_fold_power_of_two(s);
}

// LayerNorm of one bf16 row by one warp: bf16 output to y (nullable) and/or
// its BF8L quantization to yq / yscale[2] (nullable).  Returns whether every
// output was finite (all lanes agree).
// Gain and bias values of one lane (columns 16 lane .. 16 lane + 15), loaded
// ahead of the row so their latency overlaps the predecessor's completion.
struct NormLane
{
    std::uint16_t gain[16], bias[16];
};

__device__ __forceinline__ NormLane load_norm_lane(const std::uint16_t* gain, const std::uint16_t* bias)
{
    const int lane = threadIdx.x & 31;
    NormLane c;
    *reinterpret_cast<uint4*>(c.gain) = __ldg(reinterpret_cast<const uint4*>(gain + lane * 16));
    *reinterpret_cast<uint4*>(c.gain + 8) = __ldg(reinterpret_cast<const uint4*>(gain + lane * 16 + 8));
    *reinterpret_cast<uint4*>(c.bias) = __ldg(reinterpret_cast<const uint4*>(bias + lane * 16));
    *reinterpret_cast<uint4*>(c.bias + 8) = __ldg(reinterpret_cast<const uint4*>(bias + lane * 16 + 8));
    return c;
}

__device__ __forceinline__ bool layer_norm_values(const std::uint16_t (&h)[16], const NormLane& c,
                                                  std::uint16_t* y, std::int8_t* yq, float* yscale);

__device__ __forceinline__ bool layer_norm_row(const std::uint16_t* x, const NormLane& c, std::uint16_t* y,
                                               std::int8_t* yq, float* yscale)
{
    const int lane = threadIdx.x & 31;
    const std::uint16_t* src = x + lane * 16;
    std::uint16_t h[16];
    *reinterpret_cast<uint4*>(h) = *reinterpret_cast<const uint4*>(src);
    *reinterpret_cast<uint4*>(h + 8) = *reinterpret_cast<const uint4*>(src + 8);
    return layer_norm_values(h, c, y, yq, yscale);
}

__device__ __forceinline__ bool layer_norm_row(const std::uint16_t* x, const std::uint16_t* gain,
                                               const std::uint16_t* bias, std::uint16_t* y,
                                               std::int8_t* yq, float* yscale)
{
    return layer_norm_row(x, load_norm_lane(gain, bias), y, yq, yscale);
}

// The row's 16 values of this lane already in registers.
__device__ __forceinline__ bool layer_norm_values(const std::uint16_t (&h)[16], const NormLane& c,
                                                  std::uint16_t* y, std::int8_t* yq, float* yscale)
{
    const int lane = threadIdx.x & 31;
    float v[16], sq[16];
#pragma unroll
    for (int i = 0; i < 16; ++i)
    {
        v[i] = from_bf16(h[i]);
        sq[i] = __fmul_rn(v[i], v[i]);
    }
    const float reciprocal = 1.0f / 512.0f;
    const float mean = __fmul_rn(warp_sum512(v), reciprocal);
    float variance = __fmaf_rn(warp_sum512(sq), reciprocal, 0.0f);
    variance = __fmaf_rn(mean, -mean, variance);
    variance = __fadd_rn(variance, 1e-5f);
    const float inverse = __fdiv_rn(1.0f, __fsqrt_rn(variance));
    const float offset = __fmul_rn(-mean, inverse);
    std::uint16_t out[16];
    float m = 0.0f;
    bool finite = true;
#pragma unroll
    for (int i = 0; i < 16; ++i)
    {
        const float normalized = __fmaf_rn(v[i], inverse, offset);
        out[i] = to_bf16(__fmaf_rn(normalized, from_bf16(c.gain[i]), from_bf16(c.bias[i])));
        const float o = from_bf16(out[i]);
        finite = finite && isfinite(o);
        m = fmaxf(m, fabsf(flush(o)));
    }
    if (y)
    {
        std::uint16_t* dst = y + lane * 16;
        *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(out);
        *reinterpret_cast<uint4*>(dst + 8) = *reinterpret_cast<const uint4*>(out + 8);
    }
    if (yq)
    {
        // BF8L of the bf16 output: 256-blocks = lanes 0-15 and 16-31.
#pragma unroll
        for (int offset_ = 8; offset_ > 0; offset_ >>= 1)
            m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, offset_));
        float d = ftz_div(m, 127.0f);
        d = d < 1e-35f ? 1e-35f : d;
        const float scale = from_bf16(to_bf16(d));
        const float recip = ftz_div(1.0f, scale);
        unsigned packed[4] = {0, 0, 0, 0};
#pragma unroll
        for (int i = 0; i < 16; ++i)
        {
            float r = rintf(ftz_mul(from_bf16(out[i]), recip));
            r = r < -128.0f ? -128.0f : (r > 127.0f ? 127.0f : r);
            packed[i / 4] |= (static_cast<unsigned>(static_cast<int>(r)) & 0xffu) << (8 * (i % 4));
        }
        *reinterpret_cast<uint4*>(yq + lane * 16) = make_uint4(packed[0], packed[1], packed[2], packed[3]);
        if ((lane & 15) == 0)
            yscale[lane / 16] = scale;
    }
    return __all_sync(0xffffffffu, finite);
}

// ------------------------------------------------------------------- BF8L --
// BF8L quantization of one 256-value block by one warp: lane l holds values
// 8l..8l+7 of the block (a 16-byte load).  Returns the lane's 8 int8 values
// packed in two words and the block scale; nonfinite inputs clear `finite`.
struct Bf8lLane
{
    unsigned packed[2];
    float scale;
};

__device__ __forceinline__ Bf8lLane bf8l_block(uint4 raw, bool& finite)
{
    const std::uint16_t* h = reinterpret_cast<const std::uint16_t*>(&raw);
    float v[8];
    float m = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i)
    {
        v[i] = from_bf16(h[i]);
        finite = finite && isfinite(v[i]);
        m = fmaxf(m, fabsf(flush(v[i])));
    }
#pragma unroll
    for (int offset = 16; offset > 0; offset >>= 1)
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, offset));
    float d = ftz_div(m, 127.0f);
    d = d < 1e-35f ? 1e-35f : d;
    Bf8lLane out;
    out.scale = from_bf16(to_bf16(d));
    const float reciprocal = ftz_div(1.0f, out.scale);
    out.packed[0] = out.packed[1] = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i)
    {
        float r = rintf(ftz_mul(v[i], reciprocal));
        r = r < -128.0f ? -128.0f : (r > 127.0f ? 127.0f : r);
        out.packed[i / 4] |= (static_cast<unsigned>(static_cast<int>(r)) & 0xffu) << (8 * (i % 4));
    }
    return out;
}

// ------------------------------------------------------- categorical Q15 --
// conditional_q15 (src/format/categorical.cpp:76-89): the Q15 probability of
// the left child, round(flush(flush(left * 32768) / mass)) clamped to
// [1, 32767]; nonfinite or out-of-range ratios give 1.
__device__ __forceinline__ std::uint16_t conditional_q15(float left, float mass)
{
    const float value = ftz_div(ftz_mul(left, 32768.0f), mass);
    if (!isfinite(value) || value >= 0x1p63f || value < -0x1p63f)
        return 1;
    const long long integer = __float2ll_rn(value);
    const int low = static_cast<int>(static_cast<unsigned>(static_cast<unsigned long long>(integer)));
    return static_cast<std::uint16_t>(low < 1 ? 1 : (low > 32767 ? 32767 : low));
}

// -------------------------------------------------------------- attention --
constexpr int ATT_HEADS = 4, ATT_HW = 128, ATT_WIDTH = 512, ATT_BLOCK = 64;
constexpr float ATT_SCALE = 0.0883883461356163f;

struct AttArgMax
{
    float value;
    int index;
};

__device__ __forceinline__ AttArgMax att_better(AttArgMax a, AttArgMax b)
{
    return (a.value < b.value || (a.value == b.value && b.index < a.index)) ? b : a;
}

// Shared memory of one 128-thread attention group.
struct AttentionShared
{
    unsigned ks[ATT_BLOCK][65];
    unsigned vs[ATT_BLOCK][65];
    float q[ATT_HW];
    float scores[ATT_BLOCK];
    AttArgMax warp_best[2];
    float block_sum;
};

// Barrier of a 128-thread group: named barrier `id` (0 = the whole block of a
// 128-thread launch).
__device__ __forceinline__ void group_sync(int id)
{
    asm volatile("bar.sync %0, 128;" ::"r"(id) : "memory");
}

struct AttentionBlock
{
    float maximum, block_sum, sum; // sum: this thread's coordinate
};

// Stages keys and values [start, start + count) of `head` for the sequence
// whose position 0 is cache slot `base` (asynchronous copies, all in flight,
// then this thread's wait; the group's next barrier publishes them).
template <class Shared>
__device__ __forceinline__ void attention_stage(int base, int head, const std::uint16_t* cache_k,
                                                const std::uint16_t* cache_v, int start, int count, Shared& sh,
                                                int t)
{
    for (int i = t; i < count * 64; i += 128)
    {
        const int r = i >> 6, w = i & 63;
        const size_t slot = static_cast<size_t>(base + start + r) * ATT_WIDTH + head * ATT_HW;
        cp_async_4(&sh.ks[r][w], reinterpret_cast<const unsigned*>(cache_k + slot) + w);
        cp_async_4(&sh.vs[r][w], reinterpret_cast<const unsigned*>(cache_v + slot) + w);
    }
    cp_async_wait_all();
}

// The block arithmetic of one (row, head) over staged keys and values: serial
// score chains, block max, original_exp weights, pair-tree block sum, serial
// value sums (bf16-rounded when m.round), by a group of 128 threads (thread
// t = coordinate t).  `query` is the head's 128 bf16 values.  The staged
// block may hold more keys than `count`; only the first `count` are used.
template <class Shared>
__device__ __forceinline__ AttentionBlock attention_block_compute(const std::uint16_t* query, const RowMeta& m,
                                                                  int count, Shared& sh, int bar, int t)
{
    sh.q[t] = from_bf16(query[t]);
    group_sync(bar);
    AttArgMax best{-INFINITY, ATT_BLOCK};
    if (t < count)
    {
        float dot = 0.0f;
#pragma unroll 8
        for (int w = 0; w < 64; ++w)
        {
            const unsigned pair = sh.ks[t][w];
            dot = __fmaf_rn(sh.q[2 * w], from_bf16(pair & 0xffffu), dot);
            dot = __fmaf_rn(sh.q[2 * w + 1], from_bf16(pair >> 16), dot);
        }
        const float s = __fmul_rn(dot, ATT_SCALE);
        sh.scores[t] = s;
        best = AttArgMax{s, t};
    }
    if (t < 64)
    {
#pragma unroll
        for (int offset = 16; offset > 0; offset >>= 1)
        {
            AttArgMax other{__shfl_xor_sync(0xffffffffu, best.value, offset),
                            __shfl_xor_sync(0xffffffffu, best.index, offset)};
            best = att_better(best, other);
        }
        if ((t & 31) == 0)
            sh.warp_best[t >> 5] = best;
    }
    group_sync(bar);
    const float maximum = att_better(sh.warp_best[0], sh.warp_best[1]).value;
    if (t < count)
        sh.scores[t] = original_exp(__fsub_rn(sh.scores[t], maximum));
    group_sync(bar);
    if (t < 32)
    {
        float s;
        if (count <= 8)
            s = t == 0 ? pair_sum_serial(sh.scores, count, 8) : 0.0f;
        else
            s = warp_pair_sum64(2 * t < count ? sh.scores[2 * t] : 0.0f,
                                2 * t + 1 < count ? sh.scores[2 * t + 1] : 0.0f);
        if (t == 0)
            sh.block_sum = s;
    }
    // Value sums: thread t owns coordinate t, serial over the block's keys.
    float sum = 0.0f;
    const int w = t >> 1;
    const bool high = t & 1;
#pragma unroll 4
    for (int r = 0; r < count; ++r)
    {
        const unsigned pair = sh.vs[r][w];
        sum = __fmaf_rn(from_bf16(high ? (pair >> 16) : (pair & 0xffffu)), sh.scores[r], sum);
    }
    if (m.round)
        sum = from_bf16(to_bf16(sum));
    group_sync(bar);
    return AttentionBlock{maximum, sh.block_sum, sum};
}

// One 64-key block [start, start + count) of one (row, head): staging, then
// attention_block_compute.  `Shared` is AttentionShared or a smaller struct
// with the same members for blocks of at most as many keys as its arrays hold.
template <class Shared>
__device__ __forceinline__ AttentionBlock attention_block_core(const std::uint16_t* query, const RowMeta& m,
                                                               int head, const std::uint16_t* cache_k,
                                                               const std::uint16_t* cache_v, int start,
                                                               int count, Shared& sh, int bar, int t)
{
    attention_stage(m.base, head, cache_k, cache_v, start, count, sh, t);
    return attention_block_compute(query, m, count, sh, bar, t);
}

// The streaming merge's first (and, for one block, only) step from
// running = -inf, then bf16(numerator / total).
__device__ __forceinline__ std::uint16_t attention_single_output(const AttentionBlock& b)
{
    const float running = -INFINITY;
    const float difference = __fsub_rn(b.maximum, running);
    const float factor = original_exp(-fabsf(difference));
    const float old_scale = running > b.maximum ? 1.0f : factor;
    const float new_scale = running > b.maximum ? factor : 1.0f;
    const float total = __fmaf_rn(b.block_sum, new_scale, __fmul_rn(0.0f, old_scale));
    const float numerator = __fmaf_rn(b.sum, new_scale, __fmul_rn(0.0f, old_scale));
    const float reciprocal = __fdiv_rn(1.0f, total);
    return to_bf16(__fmul_rn(numerator, reciprocal));
}

// ----------------------------------------------------- softmax + masses --
struct SoftmaxShared
{
    AttArgMax warp_best[8];
    float block_sums[16];
    float level_sums[8];
    float total;
};

// Softmax of one 1024-wide bf16 row by 256 threads (thread t owns entries
// [4t, 4t+4)): reference max (first maximal entry), original_exp, the
// 64-block pair trees + carry for the total, bf16 probabilities, and the
// left-child masses of the 1023 internal nodes of the bisection heap (node i's
// children 2i+1, 2i+2; an aligned range of 2^L entries starting at b is heap
// node 2^(10-L) - 1 + b / 2^L; a left child's mass goes to slot (heap - 1) / 2).
// Returns whether every logit was finite.
__device__ __forceinline__ bool softmax_tree_row(const std::uint16_t* logits, std::uint16_t* probs_bf16,
                                                 float* probs_f32, float* tree, SoftmaxShared& sh)
{
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
    const uint2 raw = reinterpret_cast<const uint2*>(logits)[t];
    float x[4] = {from_bf16(raw.x & 0xffffu), from_bf16(raw.x >> 16), from_bf16(raw.y & 0xffffu),
                  from_bf16(raw.y >> 16)};
    const bool finite = __syncthreads_and(isfinite(x[0]) && isfinite(x[1]) && isfinite(x[2]) &&
                                          isfinite(x[3]));
    AttArgMax best{x[0], 4 * t};
#pragma unroll
    for (int i = 1; i < 4; ++i)
        best = att_better(best, AttArgMax{x[i], 4 * t + i});
#pragma unroll
    for (int offset = 16; offset > 0; offset >>= 1)
    {
        AttArgMax other{__shfl_xor_sync(0xffffffffu, best.value, offset),
                        __shfl_xor_sync(0xffffffffu, best.index, offset)};
        best = att_better(best, other);
    }
    if (lane == 0)
        sh.warp_best[warp] = best;
    __syncthreads();
    best = sh.warp_best[0];
#pragma unroll
    for (int w = 1; w < 8; ++w)
        best = att_better(best, sh.warp_best[w]);
    const float maximum = best.value;
    float e[4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
        e[i] = original_exp(__fsub_rn(x[i], maximum));
    // 64-blocks: lanes 16h..16h+15 of a warp hold block 2*warp+h; pair tree.
    float s = ftz_add(ftz_add(e[0], e[1]), ftz_add(e[2], e[3]));
#pragma unroll
    for (int offset = 1; offset < 16; offset <<= 1)
        s = ftz_add(s, __shfl_xor_sync(0xffffffffu, s, offset));
    if ((lane & 15) == 0)
        sh.block_sums[warp * 2 + lane / 16] = s;
    __syncthreads();
    if (t < 8)
    {
        // Sixteen 64-blocks: balanced tree over blocks, then the carry's
        // final fold (numeric.cuh: carry_fold_power_of_two).
        float b = ftz_add(sh.block_sums[2 * t], sh.block_sums[2 * t + 1]);
        b = ftz_add(b, __shfl_xor_sync(0x000000ffu, b, 1));
        b = ftz_add(b, __shfl_xor_sync(0x000000ffu, b, 2));
        b = ftz_add(b, __shfl_xor_sync(0x000000ffu, b, 4));
        if (t == 0)
            sh.total = carry_fold_power_of_two(b);
    }
    __syncthreads();
    const float reciprocal = __fdiv_rn(1.0f, sh.total);
    std::uint16_t p[4];
    float pf[4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
    {
        p[i] = to_bf16(__fmul_rn(e[i], reciprocal));
        pf[i] = from_bf16(p[i]);
    }
    if (probs_bf16)
        reinterpret_cast<uint2*>(probs_bf16)[t] = make_uint2(static_cast<unsigned>(p[0]) | (static_cast<unsigned>(p[1]) << 16),
                                                            static_cast<unsigned>(p[2]) | (static_cast<unsigned>(p[3]) << 16));
    if (probs_f32)
        reinterpret_cast<float4*>(probs_f32)[t] = make_float4(pf[0], pf[1], pf[2], pf[3]);
    if (tree)
    {
        auto emit = [&](int level, int begin, float mass)
        {
            const int heap = ((1 << (10 - level)) - 1) + (begin >> level);
            if (heap & 1)
                tree[(heap - 1) >> 1] = mass;
        };
        const float l0[4] = {flush(pf[0]), flush(pf[1]), flush(pf[2]), flush(pf[3])};
#pragma unroll
        for (int i = 0; i < 4; ++i)
            emit(0, 4 * t + i, l0[i]);
        const float a1 = ftz_add(pf[0], pf[1]), b1 = ftz_add(pf[2], pf[3]);
        emit(1, 4 * t, a1);
        emit(1, 4 * t + 2, b1);
        float m = ftz_add(a1, b1); // level 2, range [4t, 4t+4)
        emit(2, 4 * t, m);
#pragma unroll
        for (int level = 3; level <= 7; ++level)
        {
            const int span = 1 << (level - 2); // lanes per range at this level
            m = ftz_add(m, __shfl_xor_sync(0xffffffffu, m, span >> 1));
            if ((lane & (span - 1)) == 0)
                emit(level, 4 * t, m);
        }
        if (lane == 0)
            sh.level_sums[warp] = m; // 128-wide range [128w, 128w+128)
        __syncthreads();
        if (t == 0)
        {
            const float l8[4] = {ftz_add(sh.level_sums[0], sh.level_sums[1]),
                                 ftz_add(sh.level_sums[2], sh.level_sums[3]),
                                 ftz_add(sh.level_sums[4], sh.level_sums[5]),
                                 ftz_add(sh.level_sums[6], sh.level_sums[7])};
#pragma unroll
            for (int i = 0; i < 4; ++i)
                emit(8, 256 * i, l8[i]);
            emit(9, 0, ftz_add(l8[0], l8[1]));
            emit(9, 512, ftz_add(l8[2], l8[3]));
        }
    }
    __syncthreads();
    return finite;
}
} // namespace tsacb::dev
