// Causal attention of the TSAC probability model (4 heads x 128) over a bf16
// K/V cache, restating scalar::Attention (src/scalar/attention.cpp:12-131):
//   per head, keys in 64-key blocks; score = (serial fma over the 128
//   coordinates) * 0.0883883461356163; block max; e = original_exp(s - max);
//   value sums serial over the block's keys (bf16-rounded when the history is
//   longer than 64 keys or the row is a replay prefill); blocks merged in
//   order with old/new scales original_exp(-|dmax|); out = bf16(num / total).
//
// B200 mapping (flash-decoding with an order-exact combine):
//   kernel 1, one CTA per (row, head, 64-key block): stage the block's K and V
//   in shared memory (rows padded to 65 words, conflict-free), 64 threads run
//   the serial score chains, 128 threads the serial value chains; it writes
//   (block max, block sum, 128 value sums).
//   kernel 2, one CTA per (row, head): the sequential merge over blocks, which
//   is cheap (16 steps at 1024 keys) and keeps the reference's order.
#include "kernels/numeric.cuh"
#include "kernels/row_ops.cuh"
#include "kernels/launch_count.hpp"
#include "kernels/pdl.cuh"
#include "kernels/transformer_ops.cuh"

namespace tsacb::dev
{
namespace
{
constexpr int HEADS = ATT_HEADS, HW = ATT_HW, WIDTH = ATT_WIDTH, BLOCK = ATT_BLOCK, PSTRIDE = HW + 2;

// One CTA per (row, head, 64-key block) (row_ops.cuh: attention_block_core).
// SINGLE: the whole history fits one 64-key block (codebook stack, short
// temporal histories); the kernel then applies the one-block merge itself and
// writes the bf16 output, with exactly the combine kernel's operations.
template <bool SINGLE>
__global__ void __launch_bounds__(128)
    attention_block_kernel(const std::uint16_t* __restrict__ query,
                           const RowMeta* __restrict__ meta,
                           const std::uint16_t* __restrict__ cache_k,
                           const std::uint16_t* __restrict__ cache_v, int max_blocks,
                           float* __restrict__ partials, std::uint16_t* __restrict__ output)
{
    pdl_prologue();
    __shared__ AttentionShared sh;
    const int block = blockIdx.y;
    const int task = blockIdx.x; // row * HEADS + head
    const int row = task / HEADS, head = task % HEADS;
    const RowMeta m = meta[row];
    const int start = block * BLOCK;
    if (start >= m.time)
        return;
    const int count = m.time - start < BLOCK ? m.time - start : BLOCK;
    const int t = threadIdx.x;
    const AttentionBlock b = attention_block_core(query + static_cast<size_t>(row) * WIDTH + head * HW, m, head,
                                                  cache_k, cache_v, start, count, sh, 0, t);
    if constexpr (SINGLE)
    {
        output[static_cast<size_t>(row) * WIDTH + head * HW + t] = attention_single_output(b);
        return;
    }
    float* out = partials + (static_cast<size_t>(task) * max_blocks + block) * PSTRIDE;
    out[2 + t] = b.sum;
    if (t == 0)
    {
        out[0] = b.maximum;
        out[1] = b.block_sum;
    }
}

__global__ void __launch_bounds__(128)
    attention_combine_kernel(const RowMeta* __restrict__ meta, const float* __restrict__ partials,
                             int max_blocks, std::uint16_t* __restrict__ out)
{
    pdl_prologue();
    const int task = blockIdx.x;
    const int row = task / HEADS, head = task % HEADS;
    const int t = threadIdx.x;
    const int blocks = (meta[row].time + BLOCK - 1) / BLOCK;
    float running = -INFINITY, total = 0.0f, numerator = 0.0f;
    for (int b = 0; b < blocks; ++b)
    {
        const float* p = partials + (static_cast<size_t>(task) * max_blocks + b) * PSTRIDE;
        const float maximum = p[0];
        const float difference = __fsub_rn(maximum, running);
        const float factor = original_exp(-fabsf(difference));
        const float old_scale = running > maximum ? 1.0f : factor;
        const float new_scale = running > maximum ? factor : 1.0f;
        const float old_total = __fmul_rn(total, old_scale);
        total = __fmaf_rn(p[1], new_scale, old_total);
        const float old = __fmul_rn(numerator, old_scale);
        numerator = __fmaf_rn(p[2 + t], new_scale, old);
        running = running < maximum ? maximum : running;
    }
    const float reciprocal = __fdiv_rn(1.0f, total);
    out[static_cast<size_t>(row) * WIDTH + head * HW + t] = to_bf16(__fmul_rn(numerator, reciprocal));
}
} // namespace

size_t attention_partials_bytes(int rows, int max_time)
{
    const int blocks = (max_time + BLOCK - 1) / BLOCK;
    return static_cast<size_t>(rows) * HEADS * blocks * PSTRIDE * sizeof(float);
}

void attention(const std::uint16_t* query, const RowMeta* meta, const std::uint16_t* cache_k,
               const std::uint16_t* cache_v, int rows, int max_time, float* partials,
               std::uint16_t* out, cudaStream_t stream)
{
    if (rows <= 0)
        return;
    const int blocks = (max_time + BLOCK - 1) / BLOCK;
    if (blocks == 1)
    {
        launch_pdl(attention_block_kernel<true>, dim3(rows * HEADS, 1), dim3(128), 0, stream, query,
                   meta, cache_k, cache_v, 1, static_cast<float*>(nullptr), out);
        note_launch();
        return;
    }
    launch_pdl(attention_block_kernel<false>, dim3(rows * HEADS, blocks), dim3(128), 0, stream, query,
               meta, cache_k, cache_v, blocks, partials, static_cast<std::uint16_t*>(nullptr));
    note_launch();
    launch_pdl(attention_combine_kernel, dim3(rows * HEADS), dim3(128), 0, stream, meta,
               static_cast<const float*>(partials), blocks, out);
    note_launch();
}
} // namespace tsacb::dev
