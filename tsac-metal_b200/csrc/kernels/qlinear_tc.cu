// tcgen05 int8 GEMM for quantized linear layers with many rows (the encoder's
// known-token prefill: every frame of every lane of every recording at once).
//
// Same contract as qlinear.cu (PackedLinear::apply_into,
// src/common/packed_linear.tpp:85-123; linear_column,
// src/scalar/packed_linear.cpp:8-30): per output (m, o) and 256-wide block b
// the int8 dot is exact, and the blocks fold in order as
//   sum = fma(float(dot_b), w_scale[b][o] * a_scale[m][b], sum),
// then out = bf16(sum + bias[o]) with the fused residual / lookup epilogue.
//
// B200 mapping, one persistent CTA per SM, ten warps:
//   warp 0      TMA producer: per 128-byte K chunk, the activation tile
//               [128 rows][128 int8] and the weight tile [128 outputs][128
//               int8], 128-byte swizzled, into a 4-stage ring.
//   warp 1      TMEM owner and MMA issuer: tcgen05.mma kind::i8 (s8 x s8 ->
//               s32, M = 128, N = 128, K = 32), 8 per 256-block, into one of
//               two TMEM accumulators; tcgen05.commit frees each smem stage
//               and hands each finished block dot to the epilogue.  Integer
//               accumulation is exact, so a block dot equals the reference's.
//   warps 2..9  epilogue, two warps per TMEM lane quarter (one output row per
//               thread, 64 columns each): per block, tcgen05.ld of the dots,
//               release of the accumulator (the MMA warp fills the other one
//               meanwhile), then the ordered FP32 fold in registers; after the
//               last block, bias / residual / lookup and bf16 stores.
// Every wait is bounded (tc_common.cuh); a wait that gives up sets
// error_timeout, ends the other roles through the abort flag, and the CTA
// still drains its copies and MMAs and frees its TMEM before exiting.
#include "kernels/launch_count.hpp"
#include "kernels/numeric.cuh"
#include "kernels/error_bits.hpp"
#include "kernels/pdl.cuh"
#include "kernels/qlinear_epilogue.cuh"
#include "kernels/qlinear_tc.cuh"
#include "kernels/tc_common.cuh"

namespace tsacb::dev
{
namespace
{
using namespace tc;

constexpr int QBM = 128;          // rows per tile (TMEM lanes)
constexpr int QBN = 128;          // output features per tile
constexpr int QBK = 128;          // int8 per K chunk: one 128-byte swizzle row
constexpr int QSTAGES = 4;
constexpr int Q_THREADS = 320;
constexpr int Q_TILE = QBM * QBK; // bytes of one operand tile (QBM == QBN)
constexpr int Q_STAGE = 2 * Q_TILE;
constexpr int Q_SMEM = QSTAGES * Q_STAGE + 1024 /* alignment */ + 256 /* barriers */;
constexpr int Q_TMEM_COLS = 2 * QBN;
constexpr int Q_COLS = QBN / 2;   // columns per epilogue thread
static_assert(Q_SMEM <= 227 * 1024, "stage ring exceeds the per-CTA shared memory limit");

// Instruction descriptor: D s32, A and B signed int8, both K-major, M = 128, N = QBN.
__device__ __forceinline__ uint32_t i8_idesc()
{
    return (2u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(QBN >> 3) << 17) |
           (static_cast<uint32_t>(QBM >> 4) << 24);
}

__device__ __forceinline__ void mma_i8(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc,
                                       uint32_t accumulate)
{
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "setp.ne.b32 p, %4, 0;\n\t"
                 "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
                 "l"(a), "l"(b), "r"(idesc), "r"(accumulate));
}

struct TcArgs
{
    const float* wscale; // [K/256][N]
    const float* xscale; // [M][K/256]
    int m, n, k;
    Epilogue e;
    std::uint16_t* y;    // [M][N] bf16
    unsigned* error_word;
};

__global__ void __launch_bounds__(Q_THREADS, 1)
    qlinear_tc_kernel(const __grid_constant__ CUtensorMap map_x, const __grid_constant__ CUtensorMap map_w,
                      const TcArgs a)
{
    pdl_prologue();
    extern __shared__ unsigned char smem_raw[];
    unsigned char* smem = reinterpret_cast<unsigned char*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + QSTAGES * Q_STAGE);
    // bars: full[QSTAGES], empty[QSTAGES], acc_full[2], acc_empty[2], drain
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * QSTAGES + 5);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    const uint32_t full0 = smem_u32(bars), empty0 = smem_u32(bars + QSTAGES);
    const uint32_t acc_full0 = smem_u32(bars + 2 * QSTAGES), acc_empty0 = acc_full0 + 16;
    const uint32_t drain = acc_full0 + 32;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int m_tiles = (a.m + QBM - 1) / QBM;
    const int n_tiles = a.n / QBN;
    const long long tiles = static_cast<long long>(m_tiles) * n_tiles;
    const int chunks = a.k / QBK;
    const int blocks = a.k / 256;

    if (threadIdx.x == 0)
    {
        for (int s = 0; s < QSTAGES; ++s)
        {
            bar_init(full0 + 8 * s, 1);
            bar_init(empty0 + 8 * s, 1);
        }
        for (int c = 0; c < 2; ++c)
        {
            bar_init(acc_full0 + 8 * c, 1);
            bar_init(acc_empty0 + 8 * c, Q_THREADS - 64);
        }
        bar_init(drain, 1);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1)
    {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_u32(tmem_slot)),
                     "r"(Q_TMEM_COLS));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0)
    {
        if (lane == 0)
        {
            // ---------------------------------------------------- producer --
            int stage = 0;
            uint32_t phase = 0;
            long long issued = 0;
            bool ok = true;
            for (long long tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x)
            {
                const int m0 = static_cast<int>(tile / n_tiles) * QBM;
                const int n0 = static_cast<int>(tile % n_tiles) * QBN;
                for (int c = 0; c < chunks; ++c)
                {
                    if (!bar_wait(empty0 + 8 * stage, phase ^ 1u, abort_flag))
                    {
                        ok = false;
                        break;
                    }
                    const uint32_t base = smem_u32(smem + stage * Q_STAGE);
                    const uint32_t bar = full0 + 8 * stage;
                    bar_expect_tx(bar, Q_STAGE);
                    tma_2d(base, &map_x, c * QBK, m0, bar);
                    tma_2d(base + Q_TILE, &map_w, c * QBK, n0, bar);
                    ++issued;
                    if (++stage == QSTAGES)
                    {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
            }
            if (!ok)
            {
                *abort_flag = 1;
                if (a.error_word)
                    atomicOr(a.error_word, error_timeout);
                const long long pending = issued < QSTAGES ? issued : QSTAGES;
                volatile int never = 0;
                for (long long j = 1; j <= pending; ++j)
                {
                    const long long n = issued - j;
                    bar_wait(full0 + 8 * static_cast<int>(n % QSTAGES), static_cast<uint32_t>((n / QSTAGES) & 1),
                             &never);
                }
            }
        }
    }
    else if (warp == 1)
    {
        if (lane == 0)
        {
            // --------------------------------------------------------- MMA --
            const uint32_t idesc = i8_idesc();
            int stage = 0;
            uint32_t phase = 0;
            long long block_no = 0; // blocks issued by this CTA, alternating accumulators
            bool ok = true, any = false;
            for (long long tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x)
            {
                for (int b = 0; b < blocks && ok; ++b, ++block_no)
                {
                    const uint32_t acc = static_cast<uint32_t>(block_no & 1);
                    const uint32_t use = static_cast<uint32_t>((block_no >> 1) & 1);
                    if (!bar_wait(acc_empty0 + 8 * acc, use ^ 1u, abort_flag))
                    {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t d = tmem + acc * QBN;
                    for (int half = 0; half < 2; ++half)
                    {
                        if (!bar_wait(full0 + 8 * stage, phase, abort_flag))
                        {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        const uint32_t base = smem_u32(smem + stage * Q_STAGE);
#pragma unroll
                        for (int kk = 0; kk < QBK / 32; ++kk)
                            mma_i8(d, sw128_desc(base + kk * 32), sw128_desc(base + Q_TILE + kk * 32), idesc,
                                   (half | kk) != 0 ? 1u : 0u);
                        any = true;
                        mma_commit(empty0 + 8 * stage);
                        if (++stage == QSTAGES)
                        {
                            stage = 0;
                            phase ^= 1u;
                        }
                    }
                    if (ok)
                        mma_commit(acc_full0 + 8 * acc);
                }
            }
            if (!ok)
            {
                *abort_flag = 1;
                if (a.error_word)
                    atomicOr(a.error_word, error_timeout);
            }
            if (any)
            {
                mma_commit(drain);
                volatile int never = 0;
                bar_wait(drain, 0, &never);
            }
        }
    }
    else
    {
        // ---------------------------------------------------------- epilogue --
        const int quarter = warp & 3;
        const int row_in_tile = quarter * 32 + lane;
        const int col_begin = ((warp - 2) / 4) * Q_COLS;
        const uint32_t lane_base = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
        long long block_no = 0;
        bool ok = true;
        for (long long tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x)
        {
            const int m = static_cast<int>(tile / n_tiles) * QBM + row_in_tile;
            const int n0 = static_cast<int>(tile % n_tiles) * QBN + col_begin;
            const bool in_range = m < a.m;
            float sum[Q_COLS];
#pragma unroll
            for (int j = 0; j < Q_COLS; ++j)
                sum[j] = 0.0f;
            for (int b = 0; b < blocks; ++b, ++block_no)
            {
                const uint32_t acc = static_cast<uint32_t>(block_no & 1);
                const uint32_t use = static_cast<uint32_t>((block_no >> 1) & 1);
                if (!bar_wait(acc_full0 + 8 * acc, use, abort_flag))
                {
                    ok = false;
                    break;
                }
                tc_fence_after();
                uint32_t dot[Q_COLS];
#pragma unroll
                for (int c = 0; c < Q_COLS / 16; ++c)
                    tmem_load16(lane_base + acc * QBN + static_cast<uint32_t>(col_begin + 16 * c),
                                *reinterpret_cast<uint32_t(*)[16]>(dot + 16 * c));
                tmem_wait_loads();
                tc_fence_before();
                bar_arrive(acc_empty0 + 8 * acc);
                const float xs = in_range ? __ldg(a.xscale + static_cast<size_t>(m) * blocks + b) : 0.0f;
                const float* ws = a.wscale + static_cast<size_t>(b) * a.n + n0;
#pragma unroll
                for (int j = 0; j < Q_COLS; j += 4)
                {
                    const float4 w4 = __ldg(reinterpret_cast<const float4*>(ws + j));
                    const float wv[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
                    for (int q = 0; q < 4; ++q)
                        sum[j + q] = __fmaf_rn(static_cast<float>(static_cast<int>(dot[j + q])),
                                               __fmul_rn(wv[q], xs), sum[j + q]);
                }
            }
            if (!ok)
            {
                *abort_flag = 1;
                if (a.error_word)
                    atomicOr(a.error_word, error_timeout);
                break;
            }
            if (!in_range)
                continue;
            std::uint16_t* out = a.y + static_cast<size_t>(m) * a.n + n0;
#pragma unroll
            for (int j = 0; j < Q_COLS; j += 8)
            {
                std::uint16_t v[8];
#pragma unroll
                for (int q = 0; q < 8; ++q)
                    v[q] = finish(sum[j + q], m, n0 + j + q, a.e);
                *reinterpret_cast<uint4*>(out + j) =
                    make_uint4(v[0] | (unsigned(v[1]) << 16), v[2] | (unsigned(v[3]) << 16),
                               v[4] | (unsigned(v[5]) << 16), v[6] | (unsigned(v[7]) << 16));
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(Q_TMEM_COLS));
}

bool make_i8_map(CUtensorMap* map, const std::int8_t* base, int inner, int rows)
{
    const auto fn = encode_fn();
    if (!fn)
        return false;
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(inner), static_cast<cuuint64_t>(rows)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(inner)};
    const cuuint32_t box[2] = {QBK, QBM};
    const cuuint32_t elem[2] = {1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<std::int8_t*>(base), dims, strides, box, elem,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}
} // namespace

bool qlinear_tc_supported(int m, int n, int k)
{
    return m >= QBM && n >= QBN && n % QBN == 0 && k >= 256 && k % 256 == 0;
}

cudaError_t qlinear_tc(const std::int8_t* weights, const float* weight_scales, const std::int8_t* xq,
                       const float* xscale, int m, int n, int k, const Epilogue& e, std::uint16_t* y,
                       unsigned* error_word, cudaStream_t stream)
{
    if (!qlinear_tc_supported(m, n, k))
        return cudaErrorInvalidValue;
    CUtensorMap map_x, map_w;
    if (!make_i8_map(&map_x, xq, k, m) || !make_i8_map(&map_w, weights, k, n))
        return cudaErrorInvalidValue;
    static std::once_flag attr_once[64];
    int device = 0;
    cudaGetDevice(&device);
    if (device >= 0 && device < 64)
        std::call_once(attr_once[device],
                       []
                       {
                           cudaFuncSetAttribute(qlinear_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                Q_SMEM);
                       });
    const long long tiles = static_cast<long long>((m + QBM - 1) / QBM) * (n / QBN);
    const int grid = static_cast<int>(tiles < sm_count() ? tiles : sm_count());
    const TcArgs args{weight_scales, xscale, m, n, k, e, y, error_word};
    launch_pdl(qlinear_tc_kernel, dim3(grid), dim3(Q_THREADS), Q_SMEM, stream, map_x, map_w, args);
    note_launch();
    return cudaGetLastError();
}
} // namespace tsacb::dev
