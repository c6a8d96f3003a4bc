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
//   Histories of one block skip kernel 2; when the caller wants the output
//   BF8L-quantized for the next projection, one CTA per (row, head pair)
//   also quantizes its 256 outputs, saving the separate quantize pass.
#include "kernels/numeric.cuh"
#include "kernels/row_ops.cuh"
#include "kernels/launch_count.hpp"
#include "kernels/pdl.cuh"
#include "kernels/transformer_ops.cuh"

#include <mutex>

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

// Prefill rows: consecutive rows of one sequence read the same key blocks.
// One CTA per (TILE consecutive rows, head, 64-key block) stages the block once
// for the rows that share a sequence base (a row of another base restages)
// and runs each row's block arithmetic (attention_block_compute, unchanged)
// in turn, writing the same partials as attention_block_kernel<false>.
constexpr int TILE = 8;

__global__ void __launch_bounds__(128)
    attention_tile_kernel(const std::uint16_t* __restrict__ query, const RowMeta* __restrict__ meta,
                          const std::uint16_t* __restrict__ cache_k, const std::uint16_t* __restrict__ cache_v,
                          int rows, int max_blocks, float* __restrict__ partials)
{
    pdl_prologue();
    __shared__ AttentionShared sh;
    const int block = blockIdx.y;
    const int group = blockIdx.x / HEADS, head = blockIdx.x % HEADS;
    const int r0 = group * TILE, r1 = r0 + TILE < rows ? r0 + TILE : rows;
    const int start = block * BLOCK;
    const int t = threadIdx.x;
    int staged_base = -1, staged_count = 0;
    for (int row = r0; row < r1; ++row)
    {
        const RowMeta m = meta[row];
        if (start >= m.time)
            continue;
        const int count = m.time - start < BLOCK ? m.time - start : BLOCK;
        if (m.base != staged_base || count > staged_count)
        {
            // The most keys any remaining row of this base reads from the block.
            int need = count;
            for (int k = row + 1; k < r1; ++k)
            {
                const RowMeta n = meta[k];
                if (n.base == m.base && n.time > start)
                    need = max(need, n.time - start < BLOCK ? n.time - start : BLOCK);
            }
            attention_stage(m.base, head, cache_k, cache_v, start, need, sh, t);
            staged_base = m.base;
            staged_count = need;
        }
        const AttentionBlock b = attention_block_compute(query + static_cast<size_t>(row) * WIDTH + head * HW, m,
                                                         count, sh, 0, t);
        float* out = partials + (static_cast<size_t>(row * HEADS + head) * max_blocks + block) * PSTRIDE;
        out[2 + t] = b.sum;
        if (t == 0)
        {
            out[0] = b.maximum;
            out[1] = b.block_sum;
        }
    }
}

// One-block histories with the output BF8L-quantized for the next
// projection: one CTA per (row, head pair), i.e. per 256-value quantization
// block.  Two 128-thread groups (named barriers 1 and 2) each run one head's
// block and its one-block merge, exactly as attention_block_kernel<true>;
// the 256 bf16 outputs are then quantized with the quantize_bf8l_kernel
// operations (block max of |flush(v)|, bf16 scale, rint(v / scale) clamped).
__global__ void __launch_bounds__(256)
    attention_pair_quantize_kernel(const std::uint16_t* __restrict__ query,
                                   const RowMeta* __restrict__ meta,
                                   const std::uint16_t* __restrict__ cache_k,
                                   const std::uint16_t* __restrict__ cache_v,
                                   std::int8_t* __restrict__ yq, float* __restrict__ yscale,
                                   unsigned* error_word)
{
    pdl_prologue();
    extern __shared__ __align__(16) unsigned char attention_smem[];
    auto* groups = reinterpret_cast<AttentionShared*>(attention_smem);
    __shared__ float warp_max[8];
    const int row = blockIdx.x >> 1, pair = blockIdx.x & 1;
    const int group = threadIdx.x >> 7, t = threadIdx.x & 127;
    const int head = 2 * pair + group;
    const RowMeta m = meta[row];
    if (m.time <= 0) // uniform across the CTA: both groups share the row
        return;
    const int count = m.time < BLOCK ? m.time : BLOCK;
    const AttentionBlock b = attention_block_core(query + static_cast<size_t>(row) * WIDTH + head * HW, m, head,
                                                  cache_k, cache_v, 0, count, groups[group], 1 + group, t);
    const float x = from_bf16(attention_single_output(b));
    float block_max = fmaxf(0.0f, fabsf(flush(x)));
#pragma unroll
    for (int offset = 16; offset > 0; offset >>= 1)
        block_max = fmaxf(block_max, __shfl_xor_sync(0xffffffffu, block_max, offset));
    if ((threadIdx.x & 31) == 0)
        warp_max[threadIdx.x >> 5] = block_max;
    const bool finite = __syncthreads_and(isfinite(x));
#pragma unroll
    for (int w = 0; w < 8; ++w)
        block_max = fmaxf(block_max, warp_max[w]);
    float d = ftz_div(block_max, 127.0f);
    d = d < 1e-35f ? 1e-35f : d;
    const float scale = from_bf16(to_bf16(d));
    const float reciprocal = ftz_div(1.0f, scale);
    float r = rintf(ftz_mul(x, reciprocal));
    r = r < -128.0f ? -128.0f : (r > 127.0f ? 127.0f : r);
    yq[static_cast<size_t>(row) * WIDTH + pair * 256 + threadIdx.x] = static_cast<std::int8_t>(static_cast<int>(r));
    if (threadIdx.x == 0)
    {
        yscale[row * 2 + pair] = scale;
        if (!finite && error_word)
            atomicOr(error_word, error_nonfinite);
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

bool attention(const std::uint16_t* query, const RowMeta* meta, const std::uint16_t* cache_k,
               const std::uint16_t* cache_v, int rows, int max_time, float* partials,
               std::uint16_t* out, cudaStream_t stream, std::int8_t* yq, float* yscale,
               unsigned* error_word, bool sequence_rows)
{
    if (rows <= 0)
        return false;
    const int blocks = (max_time + BLOCK - 1) / BLOCK;
    if (blocks == 1 && yq)
    {
        constexpr size_t smem = 2 * sizeof(AttentionShared);
        static std::once_flag attribute_once[64];
        int device = 0;
        cudaGetDevice(&device);
        if (device >= 0 && device < 64)
            std::call_once(attribute_once[device],
                           []
                           {
                               cudaFuncSetAttribute(attention_pair_quantize_kernel,
                                                    cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                    static_cast<int>(smem));
                           });
        launch_pdl(attention_pair_quantize_kernel, dim3(rows * 2), dim3(256), smem, stream, query, meta,
                   cache_k, cache_v, yq, yscale, error_word);
        note_launch();
        return true;
    }
    if (blocks == 1)
    {
        launch_pdl(attention_block_kernel<true>, dim3(rows * HEADS, 1), dim3(128), 0, stream, query,
                   meta, cache_k, cache_v, 1, static_cast<float*>(nullptr), out);
        note_launch();
        return false;
    }
    if (sequence_rows)
        launch_pdl(attention_tile_kernel, dim3((rows + TILE - 1) / TILE * HEADS, blocks), dim3(128), 0, stream,
                   query, meta, cache_k, cache_v, rows, blocks, partials);
    else
        launch_pdl(attention_block_kernel<false>, dim3(rows * HEADS, blocks), dim3(128), 0, stream, query,
                   meta, cache_k, cache_v, blocks, partials, static_cast<std::uint16_t*>(nullptr));
    note_launch();
    launch_pdl(attention_combine_kernel, dim3(rows * HEADS), dim3(128), 0, stream, meta,
               static_cast<const float*>(partials), blocks, out);
    note_launch();
    return false;
}
} // namespace tsacb::dev
