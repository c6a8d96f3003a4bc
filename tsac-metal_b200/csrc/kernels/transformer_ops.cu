// Row-wise Transformer kernels: feedback embeddings, LayerNorm (+BF8L), rotary
// + K/V cache scatter, positional adds, softmax with subtree masses, the
// categorical Q15 path and the GELU table.
//
// Reference arithmetic restated here (reference project paths):
//   embed_into / incremental prefix       src/common/cpu_transformer.tpp:171-190, 356-373
//   probability_layer_norm_bf16_into      src/common/probability.cpp:138-169
//   probability_rotary_bf16_into          src/common/probability.cpp:24-43
//   probability_add_bf16                  src/common/probability.cpp:7-12
//   probability_softmax_bf16_into         src/common/probability.cpp:96-122
//   probability_gelu_bf16                 src/common/probability.cpp:45-63
//   encode_categorical / conditional_q15  src/format/categorical.cpp:76-117
#include "kernels/numeric.cuh"
#include "kernels/launch_count.hpp"
#include "kernels/pdl.cuh"
#include "kernels/transformer_ops.cuh"

namespace tsacb::dev
{
namespace
{
__device__ __forceinline__ unsigned pack2(std::uint16_t a, std::uint16_t b)
{
    return static_cast<unsigned>(a) | (static_cast<unsigned>(b) << 16);
}

// ------------------------------------------------------------ embeddings --
// 128 threads x 8 values per 1024-wide row.
__global__ void embed_sum_kernel(const std::uint16_t* __restrict__ table,
                                 const std::uint16_t* __restrict__ tokens,
                                 const int* __restrict__ offsets, const int* __restrict__ counts,
                                 std::uint16_t* __restrict__ out)
{
    pdl_prologue();
    const int row = blockIdx.x;
    const int count = counts[row];
    const int c0 = threadIdx.x * 8;
    std::uint16_t acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int j = 0; j < count; ++j)
    {
        const int token = tokens[offsets[row] + j] & 1023;
        const uint4 raw = *reinterpret_cast<const uint4*>(
            table + (static_cast<size_t>(j) * 1024 + token) * 1024 + c0);
        const std::uint16_t* e = reinterpret_cast<const std::uint16_t*>(&raw);
#pragma unroll
        for (int i = 0; i < 8; ++i)
        {
            acc[i] = j == 0 ? e[i] : to_bf16(__fadd_rn(from_bf16(acc[i]), from_bf16(e[i])));
        }
    }
    *reinterpret_cast<uint4*>(out + static_cast<size_t>(row) * 1024 + c0) =
        make_uint4(pack2(acc[0], acc[1]), pack2(acc[2], acc[3]), pack2(acc[4], acc[5]),
                   pack2(acc[6], acc[7]));
}

// ------------------------------------------------------------ layer norm --
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

__global__ void layer_norm_kernel(const std::uint16_t* __restrict__ x,
                                  const std::uint16_t* __restrict__ gain,
                                  const std::uint16_t* __restrict__ bias, int rows,
                                  std::uint16_t* __restrict__ y, std::int8_t* __restrict__ yq,
                                  float* __restrict__ yscale, unsigned* error_word)
{
    pdl_prologue();
    const int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (row >= rows)
        return;
    const std::uint16_t* src = x + static_cast<size_t>(row) * 512 + lane * 16;
    const uint4 r0 = *reinterpret_cast<const uint4*>(src);
    const uint4 r1 = *reinterpret_cast<const uint4*>(src + 8);
    std::uint16_t h[16];
    *reinterpret_cast<uint4*>(h) = r0;
    *reinterpret_cast<uint4*>(h + 8) = r1;
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
        const int c = lane * 16 + i;
        const float normalized = __fmaf_rn(v[i], inverse, offset);
        out[i] = to_bf16(__fmaf_rn(normalized, from_bf16(gain[c]), from_bf16(bias[c])));
        const float o = from_bf16(out[i]);
        finite = finite && isfinite(o);
        m = fmaxf(m, fabsf(flush(o)));
    }
    if (y)
    {
        std::uint16_t* dst = y + static_cast<size_t>(row) * 512 + lane * 16;
        *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(out);
        *reinterpret_cast<uint4*>(dst + 8) = *reinterpret_cast<const uint4*>(out + 8);
    }
    if (yq)
    {
        // BF8L of the bf16 output: 256-blocks = lanes 0-15 and 16-31.
#pragma unroll
        for (int offset_ = 8; offset_ > 0; offset_ >>= 1)
            m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, offset_));
        if (!__all_sync(0xffffffffu, finite) && lane == 0 && error_word)
            atomicOr(error_word, error_nonfinite);
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
        *reinterpret_cast<uint4*>(yq + static_cast<size_t>(row) * 512 + lane * 16) =
            make_uint4(packed[0], packed[1], packed[2], packed[3]);
        if ((lane & 15) == 0)
            yscale[row * 2 + lane / 16] = scale;
    }
}

// ------------------------------------------------------- rotary + scatter --
// 256 threads per row: thread t owns value pair t of q and of k (t in 0..255)
// and copies value pair t of v.
__global__ void rotary_scatter_kernel(const std::uint16_t* __restrict__ qkv,
                                      const RowMeta* __restrict__ meta,
                                      const std::uint16_t* __restrict__ rotations,
                                      std::uint16_t* __restrict__ query,
                                      std::uint16_t* __restrict__ cache_k,
                                      std::uint16_t* __restrict__ cache_v)
{
    pdl_prologue();
    const int row = blockIdx.x;
    const int t = threadIdx.x;
    const RowMeta m = meta[row];
    const std::uint16_t* src = qkv + static_cast<size_t>(row) * 1536;
    const unsigned q = reinterpret_cast<const unsigned*>(src)[t];
    const unsigned k = reinterpret_cast<const unsigned*>(src + 512)[t];
    const unsigned v = reinterpret_cast<const unsigned*>(src + 1024)[t];
    unsigned qo = q, ko = k;
    if (m.rotary >= 0)
    {
        const unsigned c = reinterpret_cast<const unsigned*>(rotations + m.rotary * 128)[t & 63];
        const float cosine = from_bf16(c & 0xffffu), sine = from_bf16(c >> 16);
        auto rotate = [&](unsigned pair)
        {
            const float real = from_bf16(pair & 0xffffu), imaginary = from_bf16(pair >> 16);
            const float imaginary_sine = __fmul_rn(imaginary, sine);
            const float real_sine = __fmul_rn(real, sine);
            return pack2(to_bf16(__fmaf_rn(real, cosine, -imaginary_sine)),
                         to_bf16(__fmaf_rn(imaginary, cosine, real_sine)));
        };
        qo = rotate(q);
        ko = rotate(k);
    }
    reinterpret_cast<unsigned*>(query + static_cast<size_t>(row) * 512)[t] = qo;
    reinterpret_cast<unsigned*>(cache_k + static_cast<size_t>(m.slot) * 512)[t] = ko;
    reinterpret_cast<unsigned*>(cache_v + static_cast<size_t>(m.slot) * 512)[t] = v;
}

// --------------------------------------------------------------- positions --
__global__ void add_positions_kernel(const std::uint16_t* __restrict__ src,
                                     const int* __restrict__ source_row,
                                     const int* __restrict__ book,
                                     const std::uint16_t* __restrict__ positions,
                                     std::uint16_t* __restrict__ out)
{
    pdl_prologue();
    const int row = blockIdx.x;
    const int t = threadIdx.x; // 256 threads x 2 values
    const unsigned a =
        reinterpret_cast<const unsigned*>(src + static_cast<size_t>(source_row[row]) * 512)[t];
    const unsigned p = reinterpret_cast<const unsigned*>(positions + book[row] * 512)[t];
    const std::uint16_t lo = to_bf16(__fadd_rn(from_bf16(a & 0xffffu), from_bf16(p & 0xffffu)));
    const std::uint16_t hi = to_bf16(__fadd_rn(from_bf16(a >> 16), from_bf16(p >> 16)));
    reinterpret_cast<unsigned*>(out + static_cast<size_t>(row) * 512)[t] = pack2(lo, hi);
}

// ------------------------------------------------------ softmax + masses --
// 256 threads per 1024-wide row; thread t owns entries [4t, 4t+4).
struct ArgMax
{
    float value;
    int index;
};

// Reference max: sequential (m < x ? x : m) keeps the earliest maximal entry.
__device__ __forceinline__ ArgMax better(ArgMax a, ArgMax b)
{
    return (a.value < b.value || (a.value == b.value && b.index < a.index)) ? b : a;
}

__global__ void softmax_tree_kernel(const std::uint16_t* __restrict__ logits,
                                    std::uint16_t* __restrict__ probs_bf16,
                                    float* __restrict__ probs_f32, float* __restrict__ tree,
                                    unsigned* error_word)
{
    pdl_prologue();
    __shared__ ArgMax warp_best[8];
    __shared__ float block_sums[16];
    __shared__ float level_sums[8]; // 128-wide sums (one per warp)
    __shared__ float total_shared;
    const int row = blockIdx.x;
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
    const uint2 raw = reinterpret_cast<const uint2*>(logits + static_cast<size_t>(row) * 1024)[t];
    float x[4] = {from_bf16(raw.x & 0xffffu), from_bf16(raw.x >> 16), from_bf16(raw.y & 0xffffu),
                  from_bf16(raw.y >> 16)};
    bool finite = isfinite(x[0]) && isfinite(x[1]) && isfinite(x[2]) && isfinite(x[3]);
    if (!__syncthreads_and(finite))
    {
        if (t == 0 && error_word)
            atomicOr(error_word, error_nonfinite);
    }
    ArgMax best{x[0], 4 * t};
#pragma unroll
    for (int i = 1; i < 4; ++i)
        best = better(best, ArgMax{x[i], 4 * t + i});
#pragma unroll
    for (int offset = 16; offset > 0; offset >>= 1)
    {
        ArgMax other{__shfl_xor_sync(0xffffffffu, best.value, offset),
                     __shfl_xor_sync(0xffffffffu, best.index, offset)};
        best = better(best, other);
    }
    if (lane == 0)
        warp_best[warp] = best;
    __syncthreads();
    best = warp_best[0];
#pragma unroll
    for (int w = 1; w < 8; ++w)
        best = better(best, warp_best[w]);
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
        block_sums[warp * 2 + lane / 16] = s;
    __syncthreads();
    if (t < 8)
    {
        // Sixteen 64-blocks: balanced tree over blocks (lanes 0-7 of warp 0),
        // then the carry's final fold (numeric.cuh: carry_fold_power_of_two).
        float b = ftz_add(block_sums[2 * t], block_sums[2 * t + 1]);
        b = ftz_add(b, __shfl_xor_sync(0x000000ffu, b, 1));
        b = ftz_add(b, __shfl_xor_sync(0x000000ffu, b, 2));
        b = ftz_add(b, __shfl_xor_sync(0x000000ffu, b, 4));
        if (t == 0)
            total_shared = carry_fold_power_of_two(b);
    }
    __syncthreads();
    const float reciprocal = __fdiv_rn(1.0f, total_shared);
    std::uint16_t p[4];
    float pf[4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
    {
        p[i] = to_bf16(__fmul_rn(e[i], reciprocal));
        pf[i] = from_bf16(p[i]);
    }
    if (probs_bf16)
        reinterpret_cast<uint2*>(probs_bf16 + static_cast<size_t>(row) * 1024)[t] =
            make_uint2(pack2(p[0], p[1]), pack2(p[2], p[3]));
    if (probs_f32)
        reinterpret_cast<float4*>(probs_f32 + static_cast<size_t>(row) * 1024)[t] =
            make_float4(pf[0], pf[1], pf[2], pf[3]);
    if (!tree)
        return;
    // Left-child masses of the 1023 internal nodes of the bisection heap:
    // internal node i covers an aligned range; its left child is heap node
    // 2i+1.  An aligned range of size 2^L starting at b is heap node
    // (2^(10-L) - 1) + b / 2^L; when that node is a left child (odd heap
    // index) its mass goes to slot (heap - 1) / 2.
    float* out = tree + static_cast<size_t>(row) * 1023;
    auto emit = [&](int level, int begin, float mass)
    {
        const int heap = ((1 << (10 - level)) - 1) + (begin >> level);
        if (heap & 1)
            out[(heap - 1) >> 1] = mass;
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
        level_sums[warp] = m; // 128-wide range [128w, 128w+128)
    __syncthreads();
    if (t == 0)
    {
        const float l8[4] = {ftz_add(level_sums[0], level_sums[1]),
                             ftz_add(level_sums[2], level_sums[3]),
                             ftz_add(level_sums[4], level_sums[5]),
                             ftz_add(level_sums[6], level_sums[7])};
#pragma unroll
        for (int i = 0; i < 4; ++i)
            emit(8, 256 * i, l8[i]);
        emit(9, 0, ftz_add(l8[0], l8[1]));
        emit(9, 512, ftz_add(l8[2], l8[3]));
    }
}

__device__ __forceinline__ std::uint16_t conditional_q15(float left, float mass)
{
    const float value = ftz_div(ftz_mul(left, 32768.0f), mass);
    if (!isfinite(value) || value >= 0x1p63f || value < -0x1p63f)
        return 1;
    const long long integer = __float2ll_rn(value);
    const int low = static_cast<int>(static_cast<unsigned>(static_cast<unsigned long long>(integer)));
    return static_cast<std::uint16_t>(low < 1 ? 1 : (low > 32767 ? 32767 : low));
}

__global__ void categorical_path_kernel(const float* __restrict__ tree,
                                        const std::uint16_t* __restrict__ token,
                                        const int* __restrict__ token_index, int rows,
                                        std::uint16_t* __restrict__ q15)
{
    pdl_prologue();
    const int row = blockIdx.x * blockDim.x + threadIdx.x;
    if (row >= rows)
        return;
    const int symbol = token[token_index ? token_index[row] : row];
    const float* left_masses = tree + static_cast<size_t>(row) * 1023;
    int node = 0, base = 0, count = 1024;
    float mass = 1.0f;
#pragma unroll 1
    for (int depth = 0; depth < 10; ++depth)
    {
        const int half = count / 2;
        const float left = left_masses[node];
        q15[static_cast<size_t>(row) * 10 + depth] = conditional_q15(left, mass);
        if (symbol >= base + half)
        {
            base += half;
            count -= half;
            mass = ftz_sub(mass, left);
            node = 2 * node + 2;
        }
        else
        {
            count = half;
            mass = left;
            node = 2 * node + 1;
        }
    }
}

__global__ void gelu_table_kernel(std::uint16_t* table)
{
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    const float x = from_bf16(static_cast<std::uint16_t>(i));
    const float cubic = __fmul_rn(0x1.2444f2p-5f, x);
    float z = __fmaf_rn(cubic, x, 0x1.988454p-1f);
    z = __fmul_rn(z, x);
    const float half = __fmul_rn(x, 0.5f);
    z = __fmul_rn(z, -2.0f);
    const float exponential = original_exp(z);
    const float denominator = __fadd_rn(exponential, 1.0f);
    const float sigmoid = __fdiv_rn(2.0f, denominator);
    const float tanh_ = __fsub_rn(sigmoid, 1.0f);
    const float plus = __fadd_rn(tanh_, 1.0f);
    table[i] = to_bf16(__fmul_rn(half, plus));
}
} // namespace

void embed_sum(const std::uint16_t* embeddings, const std::uint16_t* tokens, const int* offsets,
               const int* counts, int rows, std::uint16_t* out, cudaStream_t stream)
{
    if (rows > 0)
    {
        launch_pdl(embed_sum_kernel, dim3(rows), dim3(128), 0, stream, embeddings, tokens, offsets, counts, out);
        note_launch();
    }
}

void layer_norm(const std::uint16_t* x, const std::uint16_t* gain, const std::uint16_t* bias,
                int rows, std::uint16_t* y, std::int8_t* yq, float* yscale, unsigned* error_word,
                cudaStream_t stream)
{
    if (rows > 0)
    {
        launch_pdl(layer_norm_kernel, dim3((rows * 32 + 255) / 256), dim3(256), 0, stream, x, gain, bias,
                   rows, y, yq, yscale, error_word);
        note_launch();
    }
}

void rotary_scatter(const std::uint16_t* qkv, const RowMeta* meta, const std::uint16_t* rotations,
                    int rows, std::uint16_t* query, std::uint16_t* cache_k, std::uint16_t* cache_v,
                    cudaStream_t stream)
{
    if (rows > 0)
    {
        launch_pdl(rotary_scatter_kernel, dim3(rows), dim3(256), 0, stream, qkv, meta, rotations, query,
                   cache_k, cache_v);
        note_launch();
    }
}

void add_positions(const std::uint16_t* src, const int* source_row, const int* book,
                   const std::uint16_t* positions, int rows, std::uint16_t* out,
                   cudaStream_t stream)
{
    if (rows > 0)
    {
        launch_pdl(add_positions_kernel, dim3(rows), dim3(256), 0, stream, src, source_row, book, positions, out);
        note_launch();
    }
}

void softmax_tree(const std::uint16_t* logits, int rows, std::uint16_t* probs_bf16,
                  float* probs_f32, float* tree, unsigned* error_word, cudaStream_t stream)
{
    if (rows > 0)
    {
        launch_pdl(softmax_tree_kernel, dim3(rows), dim3(256), 0, stream, logits, probs_bf16, probs_f32,
                   tree, error_word);
        note_launch();
    }
}

void categorical_path_q15(const float* tree, const std::uint16_t* token, const int* token_index,
                          int rows, std::uint16_t* q15, cudaStream_t stream)
{
    if (rows > 0)
    {
        launch_pdl(categorical_path_kernel, dim3((rows + 127) / 128), dim3(128), 0, stream, tree, token,
                   token_index, rows, q15);
        note_launch();
    }
}

namespace
{
__global__ void scatter_rows_kernel(const std::uint16_t* __restrict__ src,
                                    const int* __restrict__ src_index,
                                    const int* __restrict__ dst_index, std::uint16_t* __restrict__ dst)
{
    pdl_prologue();
    const int j = blockIdx.x;
    reinterpret_cast<unsigned*>(dst + static_cast<size_t>(dst_index[j]) * 512)[threadIdx.x] =
        reinterpret_cast<const unsigned*>(src + static_cast<size_t>(src_index[j]) * 512)[threadIdx.x];
}
} // namespace

void scatter_rows(const std::uint16_t* src, const int* src_index, const int* dst_index, int rows,
                  std::uint16_t* dst, cudaStream_t stream)
{
    if (rows > 0)
    {
        launch_pdl(scatter_rows_kernel, dim3(rows), dim3(256), 0, stream, src, src_index, dst_index, dst);
        note_launch();
    }
}

void build_gelu_table(std::uint16_t* table, cudaStream_t stream)
{
    gelu_table_kernel<<<256, 256, 0, stream>>>(table);
    note_launch();
}
} // namespace tsacb::dev
