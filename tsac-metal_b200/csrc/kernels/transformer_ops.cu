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
#include "kernels/row_ops.cuh"
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
// 128 threads x 8 values per 1024-wide row.  With `yq`, the row is also
// BF8L-quantized (the quantize_bf8l_kernel operations): warp w holds 256-block
// w with lane l owning values 8l..8l+7, the bf8l_block layout.
__global__ void embed_sum_kernel(const std::uint16_t* __restrict__ table,
                                 const std::uint16_t* __restrict__ tokens,
                                 const int* __restrict__ offsets, const int* __restrict__ counts,
                                 std::uint16_t* __restrict__ out, std::int8_t* __restrict__ yq,
                                 float* __restrict__ yscale, unsigned* error_word)
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
    const uint4 packed = make_uint4(pack2(acc[0], acc[1]), pack2(acc[2], acc[3]), pack2(acc[4], acc[5]),
                                    pack2(acc[6], acc[7]));
    *reinterpret_cast<uint4*>(out + static_cast<size_t>(row) * 1024 + c0) = packed;
    if (yq)
    {
        const int lane = threadIdx.x & 31, block = threadIdx.x >> 5;
        bool finite = true;
        const Bf8lLane q = bf8l_block(packed, finite);
        if (!__all_sync(0xffffffffu, finite) && lane == 0 && error_word)
            atomicOr(error_word, error_nonfinite);
        *reinterpret_cast<uint2*>(yq + static_cast<size_t>(row) * 1024 + c0) = make_uint2(q.packed[0], q.packed[1]);
        if (lane == 0)
            yscale[row * 4 + block] = q.scale;
    }
}

// ------------------------------------------------------------ layer norm --
// One warp per row (row_ops.cuh: layer_norm_row).
__global__ void layer_norm_kernel(const std::uint16_t* __restrict__ x,
                                  const std::uint16_t* __restrict__ gain,
                                  const std::uint16_t* __restrict__ bias, int rows,
                                  std::uint16_t* __restrict__ y, std::int8_t* __restrict__ yq,
                                  float* __restrict__ yscale, unsigned* error_word)
{
    pdl_release();
    const NormLane consts = load_norm_lane(gain, bias); // model constants: before the wait
    pdl_wait();
    const int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (row >= rows)
        return;
    const bool finite = layer_norm_row(x + static_cast<size_t>(row) * 512, consts,
                                       y ? y + static_cast<size_t>(row) * 512 : nullptr,
                                       yq ? yq + static_cast<size_t>(row) * 512 : nullptr,
                                       yq ? yscale + row * 2 : nullptr);
    if (!finite && lane == 0 && error_word && yq)
        atomicOr(error_word, error_nonfinite);
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
// 256 threads per 1024-wide row (row_ops.cuh: softmax_tree_row).
__global__ void softmax_tree_kernel(const std::uint16_t* __restrict__ logits,
                                    std::uint16_t* __restrict__ probs_bf16,
                                    float* __restrict__ probs_f32, float* __restrict__ tree,
                                    unsigned* error_word)
{
    // Wait, then let the next kernel launch: the range decoder that follows
    // reads its cursor before its own wait and relies on this order.
    pdl_prologue();
    __shared__ SoftmaxShared sh;
    const size_t row = blockIdx.x;
    const bool finite = softmax_tree_row(logits + row * 1024, probs_bf16 ? probs_bf16 + row * 1024 : nullptr,
                                         probs_f32 ? probs_f32 + row * 1024 : nullptr,
                                         tree ? tree + row * 1023 : nullptr, sh);
    if (!finite && threadIdx.x == 0 && error_word)
        atomicOr(error_word, error_nonfinite);
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
               const int* counts, int rows, std::uint16_t* out, cudaStream_t stream,
               std::int8_t* yq, float* yscale, unsigned* error_word)
{
    if (rows > 0)
    {
        launch_pdl(embed_sum_kernel, dim3(rows), dim3(128), 0, stream, embeddings, tokens, offsets, counts, out,
                   yq, yscale, error_word);
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
