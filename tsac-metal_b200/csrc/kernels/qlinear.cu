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
#include "kernels/launch_count.hpp"
#include "kernels/numeric.cuh"

#include <atomic>

namespace tsacb::dev
{
namespace
{
// One warp per (row, 256-block): lane holds 8 consecutive values.
__global__ void quantize_bf8l_kernel(const std::uint16_t* __restrict__ x, int k, int rows,
                                     std::int8_t* __restrict__ q, float* __restrict__ scales,
                                     unsigned* error_word)
{
    const int blocks = k / 256;
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (warp >= rows * blocks)
    {
        return;
    }
    const int row = warp / blocks, block = warp % blocks;
    const std::uint16_t* src = x + static_cast<size_t>(row) * k + block * 256 + lane * 8;
    const uint4 raw = *reinterpret_cast<const uint4*>(src);
    const std::uint16_t* h = reinterpret_cast<const std::uint16_t*>(&raw);
    float v[8];
    float m = 0.0f;
    bool finite = true;
#pragma unroll
    for (int i = 0; i < 8; ++i)
    {
        v[i] = from_bf16(h[i]);
        finite = finite && isfinite(v[i]);
        m = fmaxf(m, fabsf(flush(v[i])));
    }
#pragma unroll
    for (int offset = 16; offset > 0; offset >>= 1)
    {
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, offset));
    }
    if (!__all_sync(0xffffffffu, finite) && lane == 0 && error_word)
    {
        atomicOr(error_word, error_nonfinite);
    }
    float d = ftz_div(m, 127.0f);
    d = d < 1e-35f ? 1e-35f : d;
    const std::uint16_t s = to_bf16(d);
    const float scale = from_bf16(s);
    const float reciprocal = ftz_div(1.0f, scale);
    unsigned packed[2] = {0, 0};
#pragma unroll
    for (int i = 0; i < 8; ++i)
    {
        float r = rintf(ftz_mul(v[i], reciprocal));
        r = r < -128.0f ? -128.0f : (r > 127.0f ? 127.0f : r);
        const unsigned byte = static_cast<unsigned>(static_cast<int>(r)) & 0xffu;
        packed[i / 4] |= byte << (8 * (i % 4));
    }
    *reinterpret_cast<uint2*>(q + static_cast<size_t>(row) * k + block * 256 + lane * 8) =
        make_uint2(packed[0], packed[1]);
    if (lane == 0)
    {
        scales[row * blocks + block] = scale;
    }
}

struct Epilogue
{
    const float* bias;
    const std::uint16_t* residual; // [M][N] or null
    const std::uint16_t* lut;      // 65536-entry bf16 map or null
};

__device__ __forceinline__ std::uint16_t finish(float sum, int m, int n, int ncols,
                                                const Epilogue& e)
{
    std::uint16_t y = to_bf16(__fadd_rn(sum, e.bias[n]));
    if (e.residual)
    {
        y = to_bf16(__fadd_rn(from_bf16(e.residual[static_cast<size_t>(m) * ncols + n]),
                              from_bf16(y)));
    }
    if (e.lut)
    {
        y = e.lut[y];
    }
    return y;
}

// Tiled GEMM for large M: 64x64 output tile, one 256-deep K block per step,
// 256 threads each owning a 4x4 sub-tile; dp4a keeps the block dot exact.
constexpr int BM = 64, BN = 64, BK = 256;

__global__ void __launch_bounds__(256)
    qlinear_gemm_kernel(const std::int8_t* __restrict__ w, const float* __restrict__ wscale,
                        const std::int8_t* __restrict__ xq, const float* __restrict__ xscale,
                        int m_rows, int n_cols, int k, Epilogue e, std::uint16_t* __restrict__ y)
{
    __shared__ __align__(16) int As[BK / 4][BM];
    __shared__ __align__(16) int Bs[BK / 4][BN];
    const int tid = threadIdx.x;
    const int tx = tid & 15, ty = tid >> 4;
    const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
    const int blocks = k / 256;
    float sum[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j)
            sum[i][j] = 0.0f;
    for (int b = 0; b < blocks; ++b)
    {
        // Stage the 64x256 A and B tiles, transposed to [k/4][row] words.
#pragma unroll
        for (int it = 0; it < 4; ++it)
        {
            const int row = tid & 63, chunk = (tid >> 6) + 4 * it; // 16-byte chunk 0..15
            uint4 a = make_uint4(0, 0, 0, 0), bw;
            if (m0 + row < m_rows)
            {
                a = *reinterpret_cast<const uint4*>(xq + static_cast<size_t>(m0 + row) * k +
                                                    b * 256 + chunk * 16);
            }
            bw = *reinterpret_cast<const uint4*>(w + static_cast<size_t>(n0 + row) * k + b * 256 +
                                                 chunk * 16);
            As[chunk * 4 + 0][row] = a.x;
            As[chunk * 4 + 1][row] = a.y;
            As[chunk * 4 + 2][row] = a.z;
            As[chunk * 4 + 3][row] = a.w;
            Bs[chunk * 4 + 0][row] = bw.x;
            Bs[chunk * 4 + 1][row] = bw.y;
            Bs[chunk * 4 + 2][row] = bw.z;
            Bs[chunk * 4 + 3][row] = bw.w;
        }
        __syncthreads();
        int acc[4][4];
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int j = 0; j < 4; ++j)
                acc[i][j] = 0;
#pragma unroll 8
        for (int k4 = 0; k4 < BK / 4; ++k4)
        {
            const int4 a = *reinterpret_cast<const int4*>(&As[k4][ty * 4]);
            const int4 bb = *reinterpret_cast<const int4*>(&Bs[k4][tx * 4]);
            const int av[4] = {a.x, a.y, a.z, a.w};
            const int bv[4] = {bb.x, bb.y, bb.z, bb.w};
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j)
                    acc[i][j] = __dp4a(av[i], bv[j], acc[i][j]);
        }
        // Ordered block fold: sum = fma(dot, w_scale * a_scale, sum).
#pragma unroll
        for (int i = 0; i < 4; ++i)
        {
            const int m = m0 + ty * 4 + i;
            const float as = m < m_rows ? xscale[m * blocks + b] : 0.0f;
#pragma unroll
            for (int j = 0; j < 4; ++j)
            {
                const int n = n0 + tx * 4 + j;
                const float scale = __fmul_rn(wscale[b * n_cols + n], as);
                sum[i][j] = __fmaf_rn(static_cast<float>(acc[i][j]), scale, sum[i][j]);
            }
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i)
    {
        const int m = m0 + ty * 4 + i;
        if (m >= m_rows)
        {
            continue;
        }
        std::uint16_t out[4];
#pragma unroll
        for (int j = 0; j < 4; ++j)
        {
            out[j] = finish(sum[i][j], m, n0 + tx * 4 + j, n_cols, e);
        }
        *reinterpret_cast<uint2*>(y + static_cast<size_t>(m) * n_cols + n0 + tx * 4) =
            make_uint2(out[0] | (unsigned(out[1]) << 16), out[2] | (unsigned(out[3]) << 16));
    }
}

// Decode-shaped launch for up to 64 columns.  A CTA owns R output rows; every
// (row, 256-block) item is one half-warp's job: each lane holds 16 weight
// bytes and, column by column, forms its 16-byte int8 dot with the column's
// activations (read through L1, shared by all rows of the CTA), reduced exactly
// over the half-warp.  Block dots land in shared memory; then one thread per
// (row, column) folds them in block order.  Short dependency chains and
// (rows x blocks) items keep every warp busy at decode sizes.
constexpr int SMALL_MAX_M = 64;

__global__ void __launch_bounds__(256)
    qlinear_small_kernel(const std::int8_t* __restrict__ w, const float* __restrict__ wscale,
                         const std::int8_t* __restrict__ xq, const float* __restrict__ xscale,
                         int m_rows, int n_cols, int k, int rows_per_cta, Epilogue e,
                         std::uint16_t* __restrict__ y)
{
    // Shared memory: the quantized activations [m_rows][k] (staged once with
    // independent 16-byte loads, so their L2 latency is paid once), then the
    // block dots [rows_per_cta][blocks][m_rows].
    extern __shared__ __align__(16) unsigned char small_smem[];
    std::int8_t* xs = reinterpret_cast<std::int8_t*>(small_smem);
    int* dots = reinterpret_cast<int*>(small_smem + static_cast<size_t>(m_rows) * k);
    const int blocks = k / 256;
    const int n0 = blockIdx.x * rows_per_cta;
    const int half = threadIdx.x >> 4, l16 = threadIdx.x & 15;
    const unsigned mask = (threadIdx.x & 16) ? 0xffff0000u : 0x0000ffffu;
    const int items = rows_per_cta * blocks;
    for (int i = threadIdx.x * 16; i < m_rows * k; i += blockDim.x * 16)
        *reinterpret_cast<uint4*>(xs + i) = __ldg(reinterpret_cast<const uint4*>(xq + i));
    __syncthreads();
    for (int item = half; item < items; item += 16)
    {
        const int r = item / blocks, b = item % blocks;
        const int n = n0 + r;
        uint4 wv = make_uint4(0, 0, 0, 0);
        if (n < n_cols)
            wv = __ldg(reinterpret_cast<const uint4*>(w + static_cast<size_t>(n) * k + b * 256 + l16 * 16));
#pragma unroll 4
        for (int c = 0; c < m_rows; ++c)
        {
            const uint4 xv = *reinterpret_cast<const uint4*>(xs + static_cast<size_t>(c) * k +
                                                             b * 256 + l16 * 16);
            int d = __dp4a(static_cast<int>(wv.x), static_cast<int>(xv.x), 0);
            d = __dp4a(static_cast<int>(wv.y), static_cast<int>(xv.y), d);
            d = __dp4a(static_cast<int>(wv.z), static_cast<int>(xv.z), d);
            d = __dp4a(static_cast<int>(wv.w), static_cast<int>(xv.w), d);
            d += __shfl_xor_sync(mask, d, 8, 16);
            d += __shfl_xor_sync(mask, d, 4, 16);
            d += __shfl_xor_sync(mask, d, 2, 16);
            d += __shfl_xor_sync(mask, d, 1, 16);
            if (l16 == 0)
                dots[(r * blocks + b) * m_rows + c] = d;
        }
    }
    __syncthreads();
    for (int t = threadIdx.x; t < rows_per_cta * m_rows; t += blockDim.x)
    {
        const int r = t / m_rows, c = t % m_rows;
        const int n = n0 + r;
        if (n >= n_cols)
            continue;
        float sum = 0.0f;
#pragma unroll 8
        for (int b = 0; b < blocks; ++b)
        {
            const float scale = __fmul_rn(__ldg(wscale + b * n_cols + n), __ldg(xscale + c * blocks + b));
            sum = __fmaf_rn(static_cast<float>(dots[(r * blocks + b) * m_rows + c]), scale, sum);
        }
        y[static_cast<size_t>(c) * n_cols + n] = finish(sum, c, n, n_cols, e);
    }
}

// Rows per CTA: enough (row, block) items for the 16 half-warps, and at least
// 4 so that few CTAs restage the same activations.
int small_rows(int k)
{
    const int blocks = k / 256;
    return blocks >= 4 ? 4 : 16 / blocks;
}

size_t small_smem_bytes(int m, int k)
{
    return static_cast<size_t>(m) * k + static_cast<size_t>(small_rows(k)) * (k / 256) * m * sizeof(int);
}

constexpr size_t SMALL_MAX_SMEM = 200 * 1024;

void launch_small(const QLinearArgs& a, const Epilogue& e, cudaStream_t stream)
{
    const int rows = small_rows(a.k);
    const size_t smem = small_smem_bytes(a.m, a.k);
    if (smem > 48 * 1024)
        qlinear_init();
    qlinear_small_kernel<<<(a.n + rows - 1) / rows, 256, smem, stream>>>(
        a.weights, a.weight_scales, a.xq, a.xscale, a.m, a.n, a.k, rows, e, a.y);
    note_launch();
}

} // namespace

void qlinear_init()
{
    // The decode-shaped kernel stages its int8 activations plus the block dots
    // in shared memory, up to SMALL_MAX_SMEM bytes.  The attribute belongs to
    // each device's context, so it is set once per device (a bit per ordinal;
    // setting it twice from racing threads is harmless).
    static std::atomic<unsigned long long> ready{0};
    int device = 0;
    if (cudaGetDevice(&device) != cudaSuccess || device < 0 || device >= 64)
        return;
    const unsigned long long bit = 1ull << device;
    if (ready.load(std::memory_order_acquire) & bit)
        return;
    if (cudaFuncSetAttribute(qlinear_small_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(SMALL_MAX_SMEM)) == cudaSuccess)
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
    quantize_bf8l_kernel<<<(warps * 32 + threads - 1) / threads, threads, 0, stream>>>(
        x, k, m, xq, xscale, error_word);
    note_launch();
}

void qlinear_matmul(const QLinearArgs& a, cudaStream_t stream)
{
    const Epilogue e{a.bias, a.residual, a.lut};
    if (a.m <= SMALL_MAX_M && small_smem_bytes(a.m, a.k) <= SMALL_MAX_SMEM)
        launch_small(a, e, stream);
    else
    {
        const dim3 grid(a.n / BN, (a.m + BM - 1) / BM);
        qlinear_gemm_kernel<<<grid, 256, 0, stream>>>(a.weights, a.weight_scales, a.xq, a.xscale,
                                                      a.m, a.n, a.k, e, a.y);
        note_launch();
    }
}
} // namespace tsacb::dev
