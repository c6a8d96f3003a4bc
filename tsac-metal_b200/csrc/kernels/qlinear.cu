// BF8L quantized linear layer of the TSAC probability model.
//
// Contract (PackedLinear::apply_into, src/common/packed_linear.tpp:85-123, with
// scalar::bf8l src/scalar/probability.cpp:16-40 and
// scalar::Kernels::linear_column src/scalar/packed_linear.cpp:8-30):
//   1. each input column (K bf16) is quantized per 256-value block:
//        m = max |flush(x)|, s = bf16(max(m/127, 1e-35)), q = clamp(rint(x/s))
//      (divide/multiply flushed as x86 FTZ);
//   2. per output o and block b the int8 dot is exact int32;
//   3. sum = fma(float(dot_b), w_scale[b][o] * a_scale[b], sum) in block order,
//      then out = bf16(sum + bias[o]);
//   4. optional fused epilogues that the reference runs as separate passes:
//      +residual with bf16 rounding (probability_add_bf16) and a GELU lookup.
//
// Layout in HBM: weights canonical int8 [N][K] (K fastest, the package's own
// source plane), w_scale f32 [K/256][N], bias f32 [N], activations bf16 [M][K].
// Quantized activations: int8 [M][K] + f32 scale [M][K/256] in caller scratch.
#include "kernels/qlinear.cuh"
#include "kernels/async_copy.cuh"
#include "kernels/launch_count.hpp"
#include "kernels/numeric.cuh"
#include "kernels/row_ops.cuh"
#include "kernels/pdl.cuh"
#include "kernels/qlinear_epilogue.cuh"
#include "kernels/qlinear_tc.cuh"

#include <atomic>

namespace tsacb::dev
{
namespace
{
// One warp per (row, 256-block).
__global__ void quantize_bf8l_kernel(const std::uint16_t* __restrict__ x, int k, int rows,
                                     std::int8_t* __restrict__ q, float* __restrict__ scales,
                                     unsigned* error_word)
{
    pdl_prologue();
    const int blocks = k / 256;
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (warp >= rows * blocks)
    {
        return;
    }
    const int row = warp / blocks, block = warp % blocks;
    const uint4 raw = *reinterpret_cast<const uint4*>(x + static_cast<size_t>(row) * k + block * 256 + lane * 8);
    bool finite = true;
    const Bf8lLane r = bf8l_block(raw, finite);
    if (!__all_sync(0xffffffffu, finite) && lane == 0 && error_word)
    {
        atomicOr(error_word, error_nonfinite);
    }
    *reinterpret_cast<uint2*>(q + static_cast<size_t>(row) * k + block * 256 + lane * 8) =
        make_uint2(r.packed[0], r.packed[1]);
    if (lane == 0)
    {
        scales[row * blocks + block] = r.scale;
    }
}

// Decode-shaped launch (fewer than GEMM_MIN_M columns).  A CTA owns 16 output features x
// 32 columns (four 8-column m-tiles).  Its 8 warps split K into 64-byte chunks
// (warp w takes quarter w % 4 of the 256-blocks b = w / 4, w / 4 + 2, ...) and
// form int8 dots on the tensor cores with mma.sync m16n8k32 (s8 x s8 -> s32:
// integer sums are exact in any order, so each block dot equals the
// reference's).  Each lane loads 16 contiguous bytes of a weight row and of an
// activation row per chunk and feeds them to two MMAs; A and B use the same
// byte-to-k assignment, so every byte pair meets exactly once.  Quarter dots
// meet in shared memory (integer atomics, exact), and 256 threads then fold
// the blocks in order, two outputs each: sum = fma(dot, w_scale * x_scale, sum).
// Row count from which the tcgen05 GEMM (qlinear_tc.cu) takes over: below it
// the weights are read once per 32 rows here, which costs less than a GEMM
// tile pass over them.
constexpr int GEMM_MIN_M = 256;
constexpr int MMA_MT = 4; // 8-column m-tiles per CTA

__device__ __forceinline__ void mma_s8(int (&d)[4], unsigned a0, unsigned a1, unsigned a2,
                                       unsigned a3, unsigned b0, unsigned b1)
{
    asm volatile("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32"
                 " {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
                 : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
                 : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

struct MmaArgs
{
    const std::int8_t* w;
    const float* wscale;
    const std::int8_t* xq; // quantized activations
    const float* xscale;
    int m_rows, n_cols, k;
    Epilogue e;
    std::uint16_t* y;
    QkvScatter qkv; // QKV_OUT destinations
};

// Shared memory of the decode-shaped kernel: the block dots, then the fold
// operands (activation scales of the CTA's rows, weight scales, biases).
__host__ __device__ constexpr size_t mma_dots_bytes(int k)
{
    return static_cast<size_t>(k / 256) * MMA_MT * 128 * sizeof(int);
}

__host__ __device__ constexpr size_t mma_smem_bytes(int k)
{
    return mma_dots_bytes(k) + static_cast<size_t>(k / 256) * (8 * MMA_MT + 16) * sizeof(float) + 16 * sizeof(float);
}


// Weight chunks (per warp) loaded before the programmatic-dependency wait:
// the model's K <= 2048 layers fit entirely.
constexpr int MMA_PRE_CHUNKS = 4;

template <bool QKV_OUT>
__global__ void __launch_bounds__(256) qlinear_mma_kernel(MmaArgs a)
{
    pdl_release();
    extern __shared__ __align__(16) unsigned char mma_smem[];
    int* dots = reinterpret_cast<int*>(mma_smem); // [block][m-tile][lane][4]
    const int k = a.k, m_rows = a.m_rows, n_cols = a.n_cols;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, t = lane & 3;
    const int n0 = blockIdx.x * 16, m0 = blockIdx.y * (8 * MMA_MT);
    const int blocks = k / 256;
    for (int i = threadIdx.x; i < blocks * MMA_MT * 128; i += 256)
        dots[i] = 0;
    const int quarter = warp & 3;
    const std::int8_t* wa = a.w + static_cast<size_t>(n0 + g) * k + quarter * 64 + t * 16;
    const std::int8_t* wb = wa + static_cast<size_t>(8) * k;
    // Model constants first (no predecessor writes them): this warp's weight
    // chunks in registers; the fold's weight scales and biases below.
    uint4 pre_lo[MMA_PRE_CHUNKS], pre_hi[MMA_PRE_CHUNKS];
#pragma unroll
    for (int it = 0; it < MMA_PRE_CHUNKS; ++it)
    {
        const int b = (warp >> 2) + 2 * it;
        if (b < blocks)
        {
            pre_lo[it] = __ldg(reinterpret_cast<const uint4*>(wa + b * 256));
            pre_hi[it] = __ldg(reinterpret_cast<const uint4*>(wb + b * 256));
        }
    }
    // The fold's weight scales [block][16 outputs] and biases: asynchronous
    // copies into shared memory, which hold no registers.
    float* xs_tile = reinterpret_cast<float*>(mma_smem + mma_dots_bytes(k)); // [32 rows][blocks]
    float* ws_tile = xs_tile + 8 * MMA_MT * blocks;                          // [blocks][16]
    float* bias_tile = ws_tile + 16 * blocks;                                // [16]
    for (int i = threadIdx.x; i < 16 * blocks; i += 256)
        cp_async_4(ws_tile + i, a.wscale + static_cast<size_t>(i >> 4) * n_cols + n0 + (i & 15));
    if (threadIdx.x < 16)
        cp_async_4(bias_tile + threadIdx.x, a.e.bias + n0 + threadIdx.x);
    pdl_wait();
    __syncthreads();
    // Predecessor outputs the fold reads, requested now so their latency
    // overlaps the activation loads and the MMAs instead of following them:
    // the CTA's activation scales (asynchronous copies into shared memory),
    // and per thread its residual values and QKV row slots.
    for (int i = threadIdx.x; i < 8 * MMA_MT * blocks; i += 256)
        if (m0 + i / blocks < m_rows)
            cp_async_4(xs_tile + i, a.xscale + static_cast<size_t>(m0) * blocks + i);
    std::uint16_t pre_res[2] = {0, 0};
    int pre_slot[2] = {0, 0}, pre_rotary[2] = {-1, -1};
#pragma unroll
    for (int half = 0; half < 2; ++half)
    {
        const int id = threadIdx.x + half * 256;
        const int n = n0 + (id & 15), m = m0 + (id >> 4);
        if (m >= m_rows)
            continue;
        if (a.e.residual)
            pre_res[half] = a.e.residual[static_cast<size_t>(m) * a.e.residual_stride + n];
        if constexpr (QKV_OUT)
        {
            pre_slot[half] = a.qkv.meta[m].slot;
            pre_rotary[half] = a.qkv.meta[m].rotary;
        }
    }
    // One 64-byte chunk of every 256-block b this warp owns (b = warp / 4,
    // warp / 4 + 2, ...): int8 MMAs of the 16 weight rows with the CTA's four
    // 8-column m-tiles, quarter dots merged in shared memory.
    const auto chunk = [&](int b, const uint4& a_lo, const uint4& a_hi)
    {
        uint4 x[MMA_MT];
#pragma unroll
        for (int mt = 0; mt < MMA_MT; ++mt)
        {
            const int m = m0 + mt * 8 + g;
            x[mt] = m < m_rows ? __ldg(reinterpret_cast<const uint4*>(
                                     a.xq + static_cast<size_t>(m) * k + b * 256 + quarter * 64 + t * 16))
                               : make_uint4(0, 0, 0, 0);
        }
#pragma unroll
        for (int mt = 0; mt < MMA_MT; ++mt)
        {
            int d[4] = {0, 0, 0, 0};
            mma_s8(d, a_lo.x, a_hi.x, a_lo.y, a_hi.y, x[mt].x, x[mt].y);
            mma_s8(d, a_lo.z, a_hi.z, a_lo.w, a_hi.w, x[mt].z, x[mt].w);
            int* slot = dots + ((b * MMA_MT + mt) * 32 + lane) * 4;
#pragma unroll
            for (int c = 0; c < 4; ++c)
                atomicAdd(slot + c, d[c]);
        }
    };
#pragma unroll
    for (int it = 0; it < MMA_PRE_CHUNKS; ++it)
    {
        const int b = (warp >> 2) + 2 * it;
        if (b < blocks)
            chunk(b, pre_lo[it], pre_hi[it]);
    }
    for (int b = (warp >> 2) + 2 * MMA_PRE_CHUNKS; b < blocks; b += 2)
        chunk(b, __ldg(reinterpret_cast<const uint4*>(wa + b * 256)),
              __ldg(reinterpret_cast<const uint4*>(wb + b * 256)));
    cp_async_wait_all();
    __syncthreads();
    // Fold: output (nl, ml), nl = 0..15, ml = 0..31; fragment element c of
    // lane (g, t) holds (n = g + 8 (c / 2), m = 2 t + c % 2) of its m-tile.
#pragma unroll
    for (int half = 0; half < 2; ++half)
    {
        const int id = threadIdx.x + half * 256;
        const int nl = id & 15, ml = id >> 4;
        const int n = n0 + nl, m = m0 + ml;
        const bool valid = m < m_rows;
        std::uint16_t out = 0;
        if (valid)
        {
            const int mt = ml >> 3, col = ml & 7;
            const int frag_lane = (nl & 7) * 4 + (col >> 1);
            const int c = (nl >> 3) * 2 + (col & 1);
            float sum = 0.0f;
            for (int b = 0; b < blocks; ++b)
            {
                const float scale = __fmul_rn(ws_tile[b * 16 + nl], xs_tile[ml * blocks + b]);
                const int dot = dots[((b * MMA_MT + mt) * 32 + frag_lane) * 4 + c];
                sum = __fmaf_rn(static_cast<float>(dot), scale, sum);
            }
            out = finish_loaded(sum, bias_tile[nl], a.e.residual != nullptr, pre_res[half], a.e.lut);
        }
        if constexpr (QKV_OUT)
        {
            // Rotary + K/V cache scatter of the bf16 projection (the
            // rotary_scatter_kernel's operations): lanes n and n ^ 1 hold a
            // (real, imaginary) pair.
            const unsigned other = __shfl_xor_sync(0xffffffffu, static_cast<unsigned>(out), 1);
            if (!valid)
                continue;
            const int slot = pre_slot[half], rotary = pre_rotary[half];
            if (n < 1024)
            {
                const bool even = (n & 1) == 0;
                std::uint16_t result = out;
                if (rotary >= 0)
                {
                    const int pair = (n & 511) >> 1;
                    const unsigned cs = reinterpret_cast<const unsigned*>(a.qkv.rotations + rotary * 128)[pair & 63];
                    const float cosine = from_bf16(cs & 0xffffu), sine = from_bf16(cs >> 16);
                    const float real = from_bf16(even ? out : static_cast<std::uint16_t>(other));
                    const float imaginary = from_bf16(even ? static_cast<std::uint16_t>(other) : out);
                    if (even)
                        result = to_bf16(__fmaf_rn(real, cosine, -__fmul_rn(imaginary, sine)));
                    else
                        result = to_bf16(__fmaf_rn(imaginary, cosine, __fmul_rn(real, sine)));
                }
                if (n < 512)
                    a.qkv.query[static_cast<size_t>(m) * 512 + n] = result;
                else
                    a.qkv.cache_k[static_cast<size_t>(slot) * 512 + (n - 512)] = result;
            }
            else
            {
                a.qkv.cache_v[static_cast<size_t>(slot) * 512 + (n - 1024)] = out;
            }
        }
        else
        {
            if (valid)
                a.y[static_cast<size_t>(m) * n_cols + n] = out;
        }
    }
}

template <bool QKV_OUT> void set_mma_smem_limit()
{
    cudaFuncSetAttribute(qlinear_mma_kernel<QKV_OUT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         static_cast<int>(mma_smem_bytes(8192)));
}

void launch_small(const QLinearArgs& a, const Epilogue& e, cudaStream_t stream)
{
    const size_t smem = mma_smem_bytes(a.k);
    if (smem > 48 * 1024)
        qlinear_init();
    const dim3 grid(a.n / 16, (a.m + 8 * MMA_MT - 1) / (8 * MMA_MT));
    const MmaArgs args{a.weights, a.weight_scales, a.xq, a.xscale, a.m, a.n, a.k, e, a.y, a.qkv};
    if (a.qkv.meta)
        launch_pdl(qlinear_mma_kernel<true>, grid, dim3(256), smem, stream, args);
    else
        launch_pdl(qlinear_mma_kernel<false>, grid, dim3(256), smem, stream, args);
    note_launch();
}

} // namespace

void qlinear_init()
{
    // The decode-shaped kernel keeps its block dots and fold operands in
    // shared memory (70 KB at k = 8192).  The attribute belongs to each device's context, so it is
    // set once per device (a bit per ordinal; setting it twice from racing
    // threads is harmless).
    static std::atomic<unsigned long long> ready{0};
    int device = 0;
    if (cudaGetDevice(&device) != cudaSuccess || device < 0 || device >= 64)
        return;
    const unsigned long long bit = 1ull << device;
    if (ready.load(std::memory_order_acquire) & bit)
        return;
    set_mma_smem_limit<false>();
    set_mma_smem_limit<true>();
    if (cudaGetLastError() == cudaSuccess)
        ready.fetch_or(bit, std::memory_order_acq_rel);
}

size_t qlinear_scratch_bytes(size_t m, size_t k)
{
    return ((m * k + 255) / 256) * 256 + m * (k / 256) * 4;
}

void qlinear_quantize(const std::uint16_t* x, int m, int k, std::int8_t* xq, float* xscale,
                      unsigned* error_word, cudaStream_t stream)
{
    const int warps = m * (k / 256);
    const int threads = 256;
    launch_pdl(quantize_bf8l_kernel, dim3((warps * 32 + threads - 1) / threads), dim3(threads), 0,
               stream, x, k, m, xq, xscale, error_word);
    note_launch();
}

bool qlinear_uses_gemm(int m, int n, int k)
{
    return m >= GEMM_MIN_M && qlinear_tc_supported(m, n, k);
}

bool qlinear_qkv_fusable(int m, int n)
{
    return m >= 1 && n == 1536 && !qlinear_uses_gemm(m, n, 512);
}

void qlinear_matmul(const QLinearArgs& a, cudaStream_t stream)
{
    const Epilogue e{a.bias, a.residual, a.lut, a.residual_stride < 0 ? a.n : a.residual_stride};
    if (!a.qkv.meta && qlinear_uses_gemm(a.m, a.n, a.k))
        qlinear_tc(a.weights, a.weight_scales, a.xq, a.xscale, a.m, a.n, a.k, e, a.y, a.error_word, stream);
    else
        launch_small(a, e, stream);
}
} // namespace tsacb::dev
