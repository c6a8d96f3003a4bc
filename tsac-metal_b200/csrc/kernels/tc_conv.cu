// tcgen05 implicit-GEMM convolution (DAC synthesis), 3xTF32.
//
// One persistent CTA per SM, ten warps:
//   warp 0      TMA producer: per k-block (tap, 32 input channels) it loads the
//               input head/tail tiles [128 rows][32 ch] and the weight head/tail
//               tiles [BN out][32 ch], 128-byte swizzled, into a STAGES-deep ring.
//   warp 1      TMEM owner and MMA issuer: 4 k-steps x 3 tcgen05.mma (kind::tf32,
//               M=128, N=BN, K=8) per k-block into the tile's four TMEM
//               accumulators; tcgen05.commit frees the smem stage and, per
//               tile, hands the accumulators to the epilogue.
//   warps 2..9  epilogue, two warps per TMEM lane quarter splitting the
//               columns: tcgen05.ld of the accumulators (one TMEM lane = one
//               output row per thread), + bias (+ residual), optional Snake of
//               the next layer, head/tail split, zero rows outside sequences,
//               fp32 stores.  The accumulators are summed into registers and
//               released first, so the rest overlaps the next tile's MMAs.
// M = 128 output rows (time), N = BN output channels, K = taps x cin.
//
// Every wait is bounded (about one second of global time).  A wait that gives
// up raises error_timeout in the error word and an abort flag that ends the
// other roles' loops; the producer then waits (bounded) for its loads in
// flight, the MMA warp for its MMAs, and the TMEM is freed before the CTA exits.
#include "kernels/dac_math.cuh"
#include "kernels/launch_count.hpp"
#include "kernels/numeric.cuh"
#include "kernels/tc_conv.cuh"
#include "kernels/tc_common.cuh"

#include <mutex>

namespace tsacb::dev
{
namespace
{
using namespace tc;

constexpr int BM = 128;        // rows per tile (TMEM lanes)
constexpr int TC_THREADS = 320; // producer warp, MMA warp, 8 epilogue warps
constexpr int BK = 32;         // fp32 per k-block row: one 128-byte swizzle row

// Four TMEM accumulators per tile (BN columns each): the hi*hi products of
// k-step j go to accumulator j mod 3 and the hi*lo + lo*hi corrections to the
// fourth.  The tensor core's fp32 accumulation rounds toward zero, so its
// error grows with the length of each accumulation chain; three short main
// chains and a correction chain 2^11 times smaller in magnitude, summed with
// round-to-nearest adds in the epilogue, keep the error near fp32 rounding.
constexpr int ACCS = 4;
// Input windows: per (tile, 32-channel chunk) one TMA load of the rows every
// tap of the tile reads, BM + span rows with span = (taps - 1) |tap_step| <=
// MAX_SPAN; each tap's A operand starts at its own row of the window.
constexpr int MAX_SPAN = 64;
constexpr int A_STAGES = 2;
constexpr int TMEM_COLS = 512;
// Shared memory: the windows of a launch (sized by its span, 1024-byte
// aligned for the 128-byte swizzle), then as many weight (B) stages as the
// rest of the 227 KB holds.
constexpr int SMEM_BYTES = 227 * 1024;
constexpr int SMEM_RESERVED = 1024 /* alignment */ + 256 /* barriers */;
constexpr int MAX_B_STAGES = 8;

__host__ __device__ constexpr int window_bytes(int span)
{
    return ((BM + span) * BK * 4 + 1023) & ~1023; // one head or tail window
}

template <int BN> __host__ __device__ constexpr int stage_bytes()
{
    return 2 * BN * BK * 4; // weight head + tail of one (tap, chunk)
}

template <int BN> __host__ __device__ constexpr int weight_stages(int span)
{
    const int s = (SMEM_BYTES - SMEM_RESERVED - A_STAGES * 2 * window_bytes(span)) / stage_bytes<BN>();
    return s < MAX_B_STAGES ? s : MAX_B_STAGES;
}
static_assert(weight_stages<128>(MAX_SPAN) >= 4 && weight_stages<96>(MAX_SPAN) >= 4,
              "the weight ring keeps at least four stages at the largest span");
static_assert((2 * MAX_B_STAGES + 5 + 2 * A_STAGES) * 8 + 8 <= 256, "barrier block exceeds its reservation");

// Instruction descriptor: D f32, A and B tf32, both K-major, M = 128, N = BN.
template <int BN> __device__ __forceinline__ uint32_t tf32_idesc()
{
    return (1u << 4) | (2u << 7) | (2u << 10) | (static_cast<uint32_t>(BN >> 3) << 17) |
           (static_cast<uint32_t>(BM >> 4) << 24);
}

__device__ __forceinline__ void mma_tf32(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc,
                                         uint32_t accumulate)
{
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "setp.ne.b32 p, %4, 0;\n\t"
                 "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
                 "l"(a), "l"(b), "r"(idesc), "r"(accumulate));
}

// Nearest TF32 value (ties away from zero) of a finite fp32; the truncated
// value where rounding would overflow to infinity.
__device__ __forceinline__ float tf32_round(float x)
{
    // Magnitudes from 0x7f7ff000 up would round to infinity (or are
    // infinity / NaN already): those are truncated.
    const unsigned bits = __float_as_uint(x);
    return __uint_as_float((bits & 0x7fffffffu) >= 0x7f7ff000u ? (bits & 0xffffe000u)
                                                               : ((bits + 0x1000u) & 0xffffe000u));
}

// Head/tail split: hi = nearest TF32 of x, lo = nearest TF32 of the exact
// remainder x - hi; x - (hi + lo) <= 2^-22 |x|.
__device__ __forceinline__ void tf32_split(float x, float& hi, float& lo)
{
    hi = tf32_round(x);
    // The remainder is at most 2^-11 |x|, far from overflow: no guard needed
    // (a nonfinite x leaves hi nonfinite, and the caller reports it).
    lo = __uint_as_float((__float_as_uint(__fsub_rn(x, hi)) + 0x1000u) & 0xffffe000u);
}

// Snake with the division by (alpha + eps) as a product with its precomputed
// reciprocal: within one rounding of snake_value's quotient, inside the tensor
// path's stated tolerance, and a short fixed sequence instead of a divide.
__device__ __forceinline__ float snake_scaled(float v, float alpha, float inverse)
{
    // The quadrant is rounded, and its parity read, by adding 1.5 * 2^23: the
    // same quadrant as rintf for |phase * 2/pi| < 2^22, without a float ->
    // int conversion.  Beyond that the parity may pick the other branch; the
    // result is still a value in [0, 1], so the added term stays within
    // [0, inverse].  One polynomial serves both parities: for an odd quadrant
    // sin^2(phase) = cos^2(x) = 1 - sin^2(x), and |x| <= pi/4 keeps
    // sin^2(x) <= 1/2, so the subtraction loses nothing.
    const float phase = __fmul_rn(alpha, v);
    const float shifted = __fadd_rn(__fmul_rn(phase, __uint_as_float(0x3f22f983u)), 12582912.0f);
    const float quadrant = __fsub_rn(shifted, 12582912.0f);
    const bool odd = (__float_as_uint(shifted) & 1u) != 0;
    const float x = reduce_quadrant(phase, quadrant);
    const float s = sine_reduced(x, __fmul_rn(x, x));
    const float s2 = __fmul_rn(s, s);
    return __fadd_rn(v, __fmul_rn(odd ? __fsub_rn(1.0f, s2) : s2, inverse));
}

struct TileCoord
{
    int phase;
    long long m;
    int n;
};

__device__ __forceinline__ TileCoord tile_coord(long long tile, long long m_tiles, int n_tiles)
{
    TileCoord t;
    t.n = static_cast<int>(tile % n_tiles);
    const long long pm = tile / n_tiles;
    t.m = pm % m_tiles;
    t.phase = static_cast<int>(pm / m_tiles);
    return t;
}

template <int BN>
__global__ void __launch_bounds__(TC_THREADS, 1)
    tc_conv_kernel(const __grid_constant__ CUtensorMap map_xhi,
                   const __grid_constant__ CUtensorMap map_xlo,
                   const __grid_constant__ CUtensorMap map_whi,
                   const __grid_constant__ CUtensorMap map_wlo, const TcConvGeometry g,
                   const TcConvEpilogue e)
{
    static_assert(ACCS * BN <= TMEM_COLS, "accumulators exceed the TMEM allocation");
    static_assert((BN / 2) % 16 == 0, "each epilogue warp takes whole 16-column chunks");
    constexpr int STAGE = stage_bytes<BN>();
    const int span = (g.taps - 1) * (g.tap_step < 0 ? -g.tap_step : g.tap_step);
    const int WIN_BYTES = window_bytes(span);
    const int STAGES = weight_stages<BN>(span);
    constexpr int B_BYTES = BN * BK * 4;
    extern __shared__ unsigned char smem_raw[];
    unsigned char* smem = reinterpret_cast<unsigned char*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    unsigned char* windows = smem;                            // [A_STAGES][head, tail][WIN_BYTES]
    unsigned char* weights = smem + A_STAGES * 2 * WIN_BYTES; // [STAGES][head, tail][B_BYTES]
    uint64_t* bars = reinterpret_cast<uint64_t*>(weights + STAGES * STAGE);
    // bars: full[STAGES], empty[STAGES], acc_full[2], acc_empty[2], drain,
    // win_full[A_STAGES], win_empty[A_STAGES]
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 5 + 2 * A_STAGES);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    const uint32_t full0 = smem_u32(bars), empty0 = smem_u32(bars + STAGES);
    const uint32_t acc_full0 = smem_u32(bars + 2 * STAGES), acc_empty0 = acc_full0 + 16;
    const uint32_t drain = acc_full0 + 32;
    const uint32_t win_full0 = drain + 8, win_empty0 = win_full0 + 8 * A_STAGES;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const long long m_tiles = (g.rows + BM - 1) / BM;
    const int n_tiles = g.cout / BN;
    const long long tiles = m_tiles * n_tiles * g.phases;
    const int chunks = g.cin / BK;
    // Window geometry: the window starts `low` rows from the tile's first
    // input row; tap t's operand starts at window row t * tap_step - low.
    const int low = g.tap_step < 0 ? (g.taps - 1) * g.tap_step : 0;
    const int win_rows = BM + (g.taps - 1) * (g.tap_step < 0 ? -g.tap_step : g.tap_step);

    if (threadIdx.x == 0)
    {
        for (int s = 0; s < STAGES; ++s)
        {
            bar_init(full0 + 8 * s, 1);
            bar_init(empty0 + 8 * s, 1);
        }
        for (int a = 0; a < 2; ++a)
        {
            bar_init(acc_full0 + 8 * a, 1);
            bar_init(acc_empty0 + 8 * a, TC_THREADS - 64);
        }
        for (int w = 0; w < A_STAGES; ++w)
        {
            bar_init(win_full0 + 8 * w, 1);
            bar_init(win_empty0 + 8 * w, 1);
        }
        bar_init(drain, 1);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1)
    {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_u32(tmem_slot)),
                     "r"(TMEM_COLS));
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
            int stage = 0, wstage = 0;
            uint32_t phase = 0, wphase = 0;
            long long issued = 0, win_issued = 0;
            bool ok = true;
            for (long long tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x)
            {
                const TileCoord t = tile_coord(tile, m_tiles, n_tiles);
                const int win_row = static_cast<int>(t.m * BM + g.row_shift[t.phase] + low);
                for (int cb = 0; cb < chunks && ok; ++cb)
                {
                    if (!bar_wait(win_empty0 + 8 * wstage, wphase ^ 1u, abort_flag))
                    {
                        ok = false;
                        break;
                    }
                    {
                        const uint32_t base = smem_u32(windows + wstage * 2 * WIN_BYTES);
                        const uint32_t bar = win_full0 + 8 * wstage;
                        bar_expect_tx(bar, 2u * static_cast<uint32_t>(win_rows) * BK * 4);
                        tma_2d(base, &map_xhi, cb * BK, win_row, bar);
                        tma_2d(base + WIN_BYTES, &map_xlo, cb * BK, win_row, bar);
                        ++win_issued;
                        if (++wstage == A_STAGES)
                        {
                            wstage = 0;
                            wphase ^= 1u;
                        }
                    }
                    for (int tap = 0; tap < g.taps; ++tap)
                    {
                        if (!bar_wait(empty0 + 8 * stage, phase ^ 1u, abort_flag))
                        {
                            ok = false;
                            break;
                        }
                        const int slice = t.phase * g.taps + tap;
                        const uint32_t base = smem_u32(weights + stage * STAGE);
                        const uint32_t bar = full0 + 8 * stage;
                        bar_expect_tx(bar, STAGE);
                        tma_3d(base, &map_whi, cb * BK, t.n * BN, slice, bar);
                        tma_3d(base + B_BYTES, &map_wlo, cb * BK, t.n * BN, slice, bar);
                        ++issued;
                        if (++stage == STAGES)
                        {
                            stage = 0;
                            phase ^= 1u;
                        }
                    }
                }
            }
            if (!ok)
            {
                *abort_flag = 1;
                if (e.error_word)
                    atomicOr(e.error_word, error_timeout);
                // Loads in flight land in the last (up to) STAGES weight stages
                // and A_STAGES windows issued; wait for them (bounded) before
                // the CTA may exit.
                volatile int never = 0;
                const long long pending = issued < STAGES ? issued : STAGES;
                for (long long k = 1; k <= pending; ++k)
                {
                    const long long n = issued - k;
                    bar_wait(full0 + 8 * static_cast<int>(n % STAGES), static_cast<uint32_t>((n / STAGES) & 1),
                             &never);
                }
                const long long win_pending = win_issued < A_STAGES ? win_issued : A_STAGES;
                for (long long k = 1; k <= win_pending; ++k)
                {
                    const long long n = win_issued - k;
                    bar_wait(win_full0 + 8 * static_cast<int>(n % A_STAGES),
                             static_cast<uint32_t>((n / A_STAGES) & 1), &never);
                }
            }
        }
    }
    else if (warp == 1)
    {
        if (lane == 0)
        {
            // --------------------------------------------------------- MMA --
            const uint32_t idesc = tf32_idesc<BN>();
            int stage = 0, wstage = 0;
            uint32_t phase = 0, wphase = 0;
            int local = 0;
            bool ok = true, any = false;
            for (long long tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x, ++local)
            {
                // One tile in flight: wait until the epilogue has read the
                // previous tile's accumulators.
                if (!bar_wait(acc_empty0, (static_cast<uint32_t>(local) & 1u) ^ 1u, abort_flag))
                {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t corr = tmem + static_cast<uint32_t>(3 * BN);
                int step = 0; // k-step within the tile
                for (int cb = 0; cb < chunks && ok; ++cb)
                {
                    if (!bar_wait(win_full0 + 8 * wstage, wphase, abort_flag))
                    {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t win = smem_u32(windows + wstage * 2 * WIN_BYTES);
                    for (int tap = 0; tap < g.taps; ++tap)
                    {
                        if (!bar_wait(full0 + 8 * stage, phase, abort_flag))
                        {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        const uint32_t a_row = static_cast<uint32_t>(tap * g.tap_step - low) * (BK * 4);
                        const uint32_t base = smem_u32(weights + stage * STAGE);
#pragma unroll
                        for (int k = 0; k < BK / 8; ++k, ++step)
                        {
                            const uint64_t ahi = sw128_desc(win + a_row + k * 32);
                            const uint64_t alo = sw128_desc(win + WIN_BYTES + a_row + k * 32);
                            const uint64_t bhi = sw128_desc(base + k * 32);
                            const uint64_t blo = sw128_desc(base + B_BYTES + k * 32);
                            const uint32_t main = tmem + static_cast<uint32_t>((step % 3) * BN);
                            mma_tf32(main, ahi, bhi, idesc, step >= 3 ? 1u : 0u);
                            mma_tf32(corr, ahi, blo, idesc, step > 0 ? 1u : 0u);
                            mma_tf32(corr, alo, bhi, idesc, 1u);
                        }
                        any = true;
                        mma_commit(empty0 + 8 * stage);
                        if (++stage == STAGES)
                        {
                            stage = 0;
                            phase ^= 1u;
                        }
                    }
                    if (!ok)
                        break;
                    mma_commit(win_empty0 + 8 * wstage);
                    if (++wstage == A_STAGES)
                    {
                        wstage = 0;
                        wphase ^= 1u;
                    }
                }
                if (!ok)
                    break;
                mma_commit(acc_full0);
            }
            if (!ok)
            {
                *abort_flag = 1;
                if (e.error_word)
                    atomicOr(e.error_word, error_timeout);
            }
            if (any)
            {
                // All MMAs this thread issued complete before TMEM is freed.
                mma_commit(drain);
                volatile int never = 0;
                bar_wait(drain, 0, &never);
            }
        }
    }
    else
    {
        // ---------------------------------------------------------- epilogue --
        // Two warps per TMEM lane quarter (a warp reaches lanes 32 (warp % 4)
        // .. +31), each taking half of the tile's columns.  The four
        // accumulators are first combined into registers and the TMEM is
        // released, so the next tile's MMAs run while this tile's bias,
        // residual, Snake, split and stores complete.
        constexpr int COLS = BN / 2, CHUNKS = COLS / 16;
        const int quarter = warp & 3;
        const int row_in_tile = quarter * 32 + lane;
        const int col_begin = ((warp - 2) / 4) * COLS;
        int local = 0;
        bool finite = true;
        for (long long tile = blockIdx.x; tile < tiles; tile += gridDim.x, ++local)
        {
            if (!bar_wait(acc_full0, static_cast<uint32_t>(local) & 1u, abort_flag))
            {
                *abort_flag = 1;
                if (e.error_word)
                    atomicOr(e.error_word, error_timeout);
                break;
            }
            tc_fence_after();
            const TileCoord t = tile_coord(tile, m_tiles, n_tiles);
            const long long i = t.m * BM + row_in_tile;
            const bool in_range = i < g.rows;
            const long long o = i * g.out_stride + t.phase;
            const bool valid = in_range && e.valid[o / g.out_scale] != 0;
            const uint32_t taddr = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
            float sum[COLS];
#pragma unroll
            for (int c = 0; c < CHUNKS; ++c)
            {
                const uint32_t at = taddr + static_cast<uint32_t>(col_begin + 16 * c);
                uint32_t a0[16], a1[16], a2[16], a3[16];
                tmem_load16(at, a0);
                tmem_load16(at + BN, a1);
                tmem_load16(at + 2 * BN, a2);
                tmem_load16(at + 3 * BN, a3);
                tmem_wait_loads();
#pragma unroll
                for (int j = 0; j < 16; ++j)
                    sum[16 * c + j] = __fadd_rn(__fadd_rn(__fadd_rn(__uint_as_float(a0[j]), __uint_as_float(a1[j])),
                                                          __uint_as_float(a2[j])),
                                                __uint_as_float(a3[j]));
            }
            tc_fence_before();
            bar_arrive(acc_empty0);
            if (!in_range)
                continue;
#pragma unroll
            for (int c = 0; c < CHUNKS; ++c)
            {
                const int c0 = col_begin + 16 * c;
                const float* v = sum + 16 * c;
                const int col = t.n * BN + c0;
                const size_t at = static_cast<size_t>(o) * g.cout + col;
                float raw[16], act[16], res[16];
                // The residual row segment in four 16-byte loads (it may be
                // the raw output itself: each element is read before this
                // thread writes it).
#pragma unroll
                for (int j = 0; j < 16; j += 4)
                {
                    const float4 r4 = valid && e.residual ? *reinterpret_cast<const float4*>(e.residual + at + j)
                                                          : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                    res[j] = r4.x;
                    res[j + 1] = r4.y;
                    res[j + 2] = r4.z;
                    res[j + 3] = r4.w;
                }
                // Per-channel constants in 16-byte loads (16-byte aligned:
                // col is a multiple of 16).
                float bias[16], alpha[16], inverse[16];
#pragma unroll
                for (int j = 0; j < 16; j += 4)
                {
                    const float4 b4 = __ldg(reinterpret_cast<const float4*>(e.bias + col + j));
                    bias[j] = b4.x;
                    bias[j + 1] = b4.y;
                    bias[j + 2] = b4.z;
                    bias[j + 3] = b4.w;
                    const float4 a4 = e.alpha ? __ldg(reinterpret_cast<const float4*>(e.alpha + col + j))
                                              : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                    alpha[j] = a4.x;
                    alpha[j + 1] = a4.y;
                    alpha[j + 2] = a4.z;
                    alpha[j + 3] = a4.w;
                    const float4 i4 = e.alpha ? __ldg(reinterpret_cast<const float4*>(e.alpha_inverse + col + j))
                                              : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                    inverse[j] = i4.x;
                    inverse[j + 1] = i4.y;
                    inverse[j + 2] = i4.z;
                    inverse[j + 3] = i4.w;
                }
#pragma unroll
                for (int j = 0; j < 16; ++j)
                {
                    float r = 0.0f;
                    if (valid)
                    {
                        r = __fadd_rn(v[j], bias[j]);
                        if (e.residual)
                            r = __fadd_rn(res[j], r);
                    }
                    raw[j] = r;
                    act[j] = (valid && e.alpha) ? snake_scaled(r, alpha[j], inverse[j]) : r;
                    // Snake adds a finite amount, so act is finite iff raw is.
                    finite = finite && isfinite(act[j]);
                }
                if (e.raw)
                {
#pragma unroll
                    for (int j = 0; j < 16; j += 4)
                        *reinterpret_cast<float4*>(e.raw + at + j) =
                            make_float4(raw[j], raw[j + 1], raw[j + 2], raw[j + 3]);
                }
                if (e.hi)
                {
                    if (e.lo)
                    {
#pragma unroll
                        for (int j = 0; j < 16; j += 4)
                        {
                            float h[4], l[4];
#pragma unroll
                            for (int q = 0; q < 4; ++q)
                                tf32_split(act[j + q], h[q], l[q]);
                            *reinterpret_cast<float4*>(e.hi + at + j) = make_float4(h[0], h[1], h[2], h[3]);
                            *reinterpret_cast<float4*>(e.lo + at + j) = make_float4(l[0], l[1], l[2], l[3]);
                        }
                    }
                    else
                    {
#pragma unroll
                        for (int j = 0; j < 16; j += 4)
                            *reinterpret_cast<float4*>(e.hi + at + j) =
                                make_float4(act[j], act[j + 1], act[j + 2], act[j + 3]);
                    }
                }
            }
        }
        if (!finite && e.error_word)
            atomicOr(e.error_word, error_nonfinite);
    }

    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                     "r"(TMEM_COLS));
}

__global__ void pad_split_rows_kernel(const float* __restrict__ src, long long rows, int channels,
                                      const long long* __restrict__ row_map, float* __restrict__ hi,
                                      float* __restrict__ lo)
{
    const long long total = rows * channels;
    for (long long k = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; k < total;
         k += static_cast<long long>(gridDim.x) * blockDim.x)
    {
        const long long r = k / channels;
        const int c = static_cast<int>(k - r * channels);
        const float v = src[k];
        const size_t at = static_cast<size_t>(row_map[r]) * channels + c;
        if (lo)
        {
            float h, l;
            tf32_split(v, h, l);
            hi[at] = h;
            lo[at] = l;
        }
        else
        {
            hi[at] = v;
        }
    }
}

// ------------------------------------------------------------ host side --
bool make_map(CUtensorMap* map, const float* base, int rank, const cuuint64_t* dims,
              const cuuint64_t* strides, const cuuint32_t* box)
{
    const auto fn = encode_fn();
    if (!fn)
        return false;
    const cuuint32_t elem[3] = {1, 1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, rank, const_cast<float*>(base), dims, strides,
              box, elem, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int BN>
cudaError_t launch(const TcConvOperands& op, const TcConvGeometry& g, const TcConvEpilogue& e,
                   cudaStream_t stream)
{
    CUtensorMap xhi, xlo, whi, wlo;
    const cuuint64_t xdims[2] = {static_cast<cuuint64_t>(g.cin), static_cast<cuuint64_t>(g.in_rows)};
    const cuuint64_t xstrides[1] = {static_cast<cuuint64_t>(g.cin) * 4};
    const int span = (g.taps - 1) * (g.tap_step < 0 ? -g.tap_step : g.tap_step);
    const cuuint32_t xbox[2] = {BK, static_cast<cuuint32_t>(BM + span)};
    const int slices = g.taps * g.phases;
    const cuuint64_t wdims[3] = {static_cast<cuuint64_t>(g.cin), static_cast<cuuint64_t>(g.cout),
                                 static_cast<cuuint64_t>(slices)};
    const cuuint64_t wstrides[2] = {static_cast<cuuint64_t>(g.cin) * 4,
                                    static_cast<cuuint64_t>(g.cin) * g.cout * 4};
    const cuuint32_t wbox[3] = {BK, BN, 1};
    if (!make_map(&xhi, op.x_hi, 2, xdims, xstrides, xbox) ||
        !make_map(&xlo, op.x_lo, 2, xdims, xstrides, xbox) ||
        !make_map(&whi, op.w_hi, 3, wdims, wstrides, wbox) ||
        !make_map(&wlo, op.w_lo, 3, wdims, wstrides, wbox))
        return cudaErrorInvalidValue;
    constexpr int smem = SMEM_BYTES;
    static std::once_flag attr_once[64];
    int device = 0;
    cudaGetDevice(&device);
    if (device >= 0 && device < 64)
        std::call_once(attr_once[device],
                       []
                       {
                           cudaFuncSetAttribute(tc_conv_kernel<BN>,
                                                cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
                       });
    const long long tiles = ((g.rows + BM - 1) / BM) * (g.cout / BN) * g.phases;
    const int grid = static_cast<int>(tiles < sm_count() ? tiles : sm_count());
    tc_conv_kernel<BN><<<grid, TC_THREADS, smem, stream>>>(xhi, xlo, whi, wlo, g, e);
    note_launch();
    return cudaGetLastError();
}
} // namespace

bool tc_conv_supported(int cin, int cout)
{
    return cin >= BK && cin % BK == 0 && cout > 0 && (cout % 128 == 0 || cout % 96 == 0);
}

cudaError_t tc_conv(const TcConvOperands& op, const TcConvGeometry& g, const TcConvEpilogue& e,
                    cudaStream_t stream)
{
    if (!tc_conv_supported(g.cin, g.cout) || g.rows <= 0 || g.phases < 1 || g.phases > 8 ||
        g.taps < 1 || g.taps * g.phases > 16 || g.out_scale < 1 || g.in_rows >= (1ll << 31) ||
        (g.taps - 1) * (g.tap_step < 0 ? -g.tap_step : g.tap_step) > MAX_SPAN)
        return cudaErrorInvalidValue;
    if (g.cout % 128 == 0)
        return launch<128>(op, g, e, stream);
    return launch<96>(op, g, e, stream);
}

void pad_split_rows(const float* src, long long rows, int channels, const long long* row_map,
                    float* hi, float* lo, cudaStream_t stream)
{
    if (rows <= 0)
        return;
    const long long total = rows * channels;
    long long blocks = (total + 255) / 256;
    blocks = blocks > 148 * 16 ? 148 * 16 : blocks;
    pad_split_rows_kernel<<<static_cast<int>(blocks), 256, 0, stream>>>(src, rows, channels,
                                                                         row_map, hi, lo);
    note_launch();
}
} // namespace tsacb::dev
