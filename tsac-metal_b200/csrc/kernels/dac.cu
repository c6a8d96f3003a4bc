// DAC analysis/synthesis kernels and the residual vector quantizer.
//
// Reference arithmetic restated (reference project paths):
//   scalar::Conv1d::sample   src/scalar/dsp.cpp:11-35 (serial unfused mul+add over
//                            (tap, input channel), invalid taps skipped, + bias)
//   source_frame geometry    src/common/dsp.tpp:141-178
//   Snake / dac_sine_squared src/scalar/dsp.cpp:55-119, epsilon 0x3089705f
//                            (src/weights/normalization.hpp:9)
//   residual unit add        src/common/analysis.tpp:59-66, synthesis.tpp:59-66
//   RVQ encode               src/common/rvq.tpp:37-57, src/common/rvq.cpp:126-146,
//                            src/weights/preparation.cpp:69-114
//   RVQ decode               src/common/rvq.cpp:76-120
//
// B200 mapping of the exact-order convolution: the reference's per-output
// serial chain is kept (products and sums rounded separately, taps outer,
// input channels inner), and parallelism comes from outputs.  A CTA owns a
// 128-frame x 128-channel output tile (64 for 64-channel layers), 512 (256)
// threads each accumulating 4 frames x 8 channels in registers; per (tap,
// 64-channel chunk) it stages the input rows channel-major and the weight
// slice in shared memory, double-buffered through registers, so every staged
// value is reused 4x or 8x from registers and a thread's operands are 16-byte loads.
// Device weights are laid out [tap][in][out] so the weight slice loads are
// contiguous.
#include "kernels/dac.cuh"
#include "kernels/dac_math.cuh"
#include "kernels/launch_count.hpp"
#include "kernels/numeric.cuh"

#include <mutex>

namespace tsacb::dev
{
namespace
{
__global__ void snake_kernel(const float* __restrict__ x, const float* __restrict__ alpha,
                             int channels, long long count, float* __restrict__ y,
                             unsigned* error_word)
{
    const float eps = __uint_as_float(0x3089705fu);
    bool ok = true;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < count;
         i += static_cast<long long>(gridDim.x) * blockDim.x)
    {
        const float a = alpha[i % channels];
        const float v = x[i];
        const float phase = __fmul_rn(a, v);
        ok = ok && isfinite(v) && isfinite(phase);
        const float out = __fadd_rn(v, __fdiv_rn(sine_squared(phase), __fadd_rn(a, eps)));
        ok = ok && isfinite(out);
        y[i] = out;
    }
    if (!ok && error_word)
        atomicOr(error_word, error_nonfinite);
}

constexpr int TF = 128, CK = 64;

// Output frame of tile row r and the input frame feeding it through `tap`.
struct TileGeometry
{
    int f_first; // ordinary: first output frame; transposed: first phase index i0
    int phase;
    __device__ __forceinline__ int out_frame(const ConvShape& s, int r) const
    {
        return s.transposed ? phase + s.stride * (f_first + r) : f_first + r;
    }
    __device__ __forceinline__ int in_frame(const ConvShape& s, int r, int tap) const
    {
        if (s.transposed)
        {
            return f_first + r + (phase + s.padding - tap) / s.stride;
        }
        return (f_first + r) * s.stride + tap * s.dilation - s.padding;
    }
    // Row r of the tile takes `tap` (the reference skips taps outside the window).
    __device__ __forceinline__ bool takes(const ConvShape& s, const Sequence& q, int r, int tap) const
    {
        const int src = in_frame(s, r, tap);
        const int f = out_frame(s, r);
        return f < q.out_frames && src >= 0 && src < q.in_frames &&
               (!s.transposed || f + s.padding >= tap);
    }
};

// Shared memory of one pipeline stage: the input chunk stored channel-major
// (xs[c][row], so a thread's 4 consecutive rows are one 16-byte load) and the
// weight chunk [c][output].
template <int TO> struct ConvStage
{
    float xs[CK][TF + 4];
    float ws[CK][TO];
};

template <int TO> constexpr size_t conv_smem_bytes()
{
    return 2 * sizeof(ConvStage<TO>);
}

// Exact-order convolution.  A CTA owns a 128-frame x TO-channel output tile
// (TO = 128 with 512 threads, 64 with 256); each thread holds 4 frames x 8
// channels of serial chains in registers: channels tx*4..tx*4+3 and
// TO/2 + tx*4..+3, so the 8 threads of a shared-memory wavefront read 128
// contiguous weight bytes (no bank conflicts).  Per (tap, 64-channel chunk)
// "step", the chunk's inputs and weights are staged in shared memory; the
// next step's global loads are issued into registers before the current
// step's arithmetic and stored after it (two stages, one barrier per step).
// Per output the order is the reference's: taps ascending, channels
// ascending, sum = sum + x * w with the product and the sum each rounded; a
// row skips taps whose input frame lies outside its window.
// One multiply-accumulate term of a chain.  Exact (the reference's order):
// the product and the sum are each rounded.  FAST (the certified fast
// analysis only): one fused multiply-add, a single rounding per term and half
// the issued instructions; its results differ from the reference's in the
// last bits, so the caller checks every decision that depends on them.
template <bool FAST> __device__ __forceinline__ float accumulate(float sum, float x, float w)
{
    if constexpr (FAST)
        return __fmaf_rn(x, w, sum);
    else
        return __fadd_rn(sum, __fmul_rn(x, w));
}

template <int TO, int THREADS, bool FAST>
__global__ void __launch_bounds__(THREADS, 512 / THREADS)
    conv1d_kernel(ConvLaunch l)
{
    constexpr int TR = 4;
    constexpr int CG = TO / 8;           // column groups (threads across outputs)
    static_assert(THREADS / CG * TR == TF, "tile rows");
    constexpr int XV = TF * CK / 4 / THREADS; // input float4 per thread per step
    constexpr int WV = CK * TO / 4 / THREADS; // weight float4 per thread per step
    extern __shared__ __align__(16) unsigned char conv_smem[];
    auto* stage = reinterpret_cast<ConvStage<TO>*>(conv_smem);
    const ConvShape s = l.shape;
    const int4 tile = l.tiles[blockIdx.x];
    const Sequence seq = l.sequences[tile.x];
    const TileGeometry g{tile.y, tile.z};
    const int o0 = blockIdx.y * TO;
    const int tid = threadIdx.x, tx = tid % CG, ty = tid / CG;

    // Taps used by any / every row of the tile (uniform across the CTA).
    const int tap_count = s.transposed ? 2 : s.kernel;
    const int tap_first = s.transposed ? (g.phase + s.padding) % s.stride : 0;
    unsigned any_mask = 0, all_mask = 0;
    for (int ti = 0; ti < tap_count; ++ti)
    {
        const int tap = s.transposed ? tap_first + ti * s.stride : ti;
        const bool mine = tid < TF && g.takes(s, seq, tid, tap);
        const bool row_ok = tid >= TF || mine;
        if (__syncthreads_or(mine))
            any_mask |= 1u << ti;
        if (__syncthreads_and(row_ok))
            all_mask |= 1u << ti;
    }
    const int chunks = (s.cin + CK - 1) / CK;
    const int steps = __popc(any_mask) * chunks;

    float sum[TR][8];
#pragma unroll
    for (int i = 0; i < TR; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j)
            sum[i][j] = 0.0f;

    // Step k -> (tap index, chunk): taps in ascending order, skipping unused ones.
    auto step_tap = [&](int k, int& ti, int& c0)
    {
        int n = k / chunks;
        c0 = (k - n * chunks) * CK;
        unsigned m = any_mask;
        for (; n > 0; --n)
            m &= m - 1;
        ti = __ffs(m) - 1;
    };
    float xr[4 * XV];
    float4 wr[WV];
    auto load = [&](int k)
    {
        int ti, c0;
        step_tap(k, ti, c0);
        const int tap = s.transposed ? tap_first + ti * s.stride : ti;
        const int cn = s.cin - c0 < CK ? s.cin - c0 : CK;
#pragma unroll
        for (int it = 0; it < XV; ++it)
        {
            const int idx = it * THREADS + tid;
            const int r = idx & (TF - 1), cg = idx >> 7; // channels 4cg .. 4cg+3
            const int src = g.in_frame(s, r, tap);
            const bool in = src >= 0 && src < seq.in_frames;
            const float* xp = l.x + static_cast<size_t>(seq.in_offset + (in ? src : 0)) * s.cin + c0 + 4 * cg;
            if (in && 4 * cg + 3 < cn && (s.cin & 3) == 0)
            {
                const float4 v = __ldg(reinterpret_cast<const float4*>(xp));
                xr[4 * it] = v.x;
                xr[4 * it + 1] = v.y;
                xr[4 * it + 2] = v.z;
                xr[4 * it + 3] = v.w;
            }
            else
            {
#pragma unroll
                for (int j = 0; j < 4; ++j)
                    xr[4 * it + j] = in && 4 * cg + j < cn ? __ldg(xp + j) : 0.0f;
            }
        }
#pragma unroll
        for (int it = 0; it < WV; ++it)
        {
            const int idx = it * THREADS + tid;
            const int c = idx / (TO / 4), o4 = idx % (TO / 4);
            float4 v = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            if (c < cn && o0 + 4 * o4 < s.cout)
                v = __ldg(reinterpret_cast<const float4*>(
                    l.weights + (static_cast<size_t>(tap) * s.cin + c0 + c) * s.cout + o0 + 4 * o4));
            wr[it] = v;
        }
    };
    auto store = [&](ConvStage<TO>& st)
    {
#pragma unroll
        for (int it = 0; it < XV; ++it)
        {
            const int idx = it * THREADS + tid;
            const int r = idx & (TF - 1), cg = idx >> 7;
#pragma unroll
            for (int j = 0; j < 4; ++j)
                st.xs[4 * cg + j][r] = xr[4 * it + j];
        }
#pragma unroll
        for (int it = 0; it < WV; ++it)
        {
            const int idx = it * THREADS + tid;
            const int c = idx / (TO / 4), o4 = idx % (TO / 4);
            *reinterpret_cast<float4*>(&st.ws[c][4 * o4]) = wr[it];
        }
    };

    if (steps > 0)
    {
        load(0);
        store(stage[0]);
    }
    __syncthreads();
    for (int k = 0; k < steps; ++k)
    {
        const ConvStage<TO>& st = stage[k & 1];
        if (k + 1 < steps)
            load(k + 1);
        int ti, c0;
        step_tap(k, ti, c0);
        const int cn = s.cin - c0 < CK ? s.cin - c0 : CK;
        if ((all_mask >> ti) & 1u)
        {
#pragma unroll 4
            for (int c = 0; c < cn; ++c)
            {
                const float4 w0 = *reinterpret_cast<const float4*>(&st.ws[c][tx * 4]);
                const float4 w1 = *reinterpret_cast<const float4*>(&st.ws[c][TO / 2 + tx * 4]);
                const float4 xv = *reinterpret_cast<const float4*>(&st.xs[c][ty * TR]);
                const float wa[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
                const float xa[TR] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
                for (int i = 0; i < TR; ++i)
#pragma unroll
                    for (int j = 0; j < 8; ++j)
                        sum[i][j] = accumulate<FAST>(sum[i][j], xa[i], wa[j]);
            }
        }
        else
        {
            const int tap = s.transposed ? tap_first + ti * s.stride : ti;
            unsigned valid = 0;
#pragma unroll
            for (int i = 0; i < TR; ++i)
                if (g.takes(s, seq, ty * TR + i, tap))
                    valid |= 1u << i;
#pragma unroll 1
            for (int c = 0; c < cn; ++c)
            {
                const float4 w0 = *reinterpret_cast<const float4*>(&st.ws[c][tx * 4]);
                const float4 w1 = *reinterpret_cast<const float4*>(&st.ws[c][TO / 2 + tx * 4]);
                const float wa[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
                for (int i = 0; i < TR; ++i)
                {
                    const float xv = st.xs[c][ty * TR + i];
                    const bool take = (valid >> i) & 1u;
#pragma unroll
                    for (int j = 0; j < 8; ++j)
                    {
                        const float n = accumulate<FAST>(sum[i][j], xv, wa[j]);
                        sum[i][j] = take ? n : sum[i][j];
                    }
                }
            }
        }
        if (k + 1 < steps)
            store(stage[(k + 1) & 1]);
        __syncthreads();
    }

    // Epilogue: + bias, then residual + result; optionally Snake of the next
    // layer into `act` (the reference applies it to the stored sum).
    bool ok = true;
#pragma unroll
    for (int i = 0; i < TR; ++i)
    {
        const int r = ty * TR + i;
        const int f = g.out_frame(s, r);
        if (f >= seq.out_frames)
            continue;
        const size_t row = static_cast<size_t>(seq.out_offset + f) * s.cout;
#pragma unroll
        for (int j = 0; j < 8; ++j)
        {
            const int o = o0 + (j < 4 ? tx * 4 + j : TO / 2 + tx * 4 + j - 4);
            if (o >= s.cout)
                continue;
            float v = __fadd_rn(sum[i][j], __ldg(l.bias + o));
            if (l.residual)
                v = __fadd_rn(l.residual[row + o], v);
            ok = ok && isfinite(v);
            if (l.y)
                l.y[row + o] = v;
            if (l.act)
            {
                const float a = snake_value(v, __ldg(l.alpha + o));
                ok = ok && isfinite(a);
                l.act[row + o] = a;
            }
        }
    }
    if (!ok && l.error_word)
        atomicOr(l.error_word, error_nonfinite);
}

// Narrow outputs (DAC exit convolution to 1-2 PCM channels): one thread per
// output, the whole serial chain in registers.
__global__ void conv1d_narrow_kernel(const float* __restrict__ x, const float* __restrict__ w,
                                     const float* __restrict__ bias, float* __restrict__ y,
                                     const Sequence* __restrict__ sequences, int sequence_count,
                                     ConvShape s, long long total, unsigned* error_word)
{
    const long long id = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x;
    if (id >= total)
        return;
    // Locate the sequence by scanning (sequence counts are small).
    long long rest = id;
    int q = 0;
    for (; q < sequence_count; ++q)
    {
        const long long n = static_cast<long long>(sequences[q].out_frames) * s.cout;
        if (rest < n)
            break;
        rest -= n;
    }
    const Sequence seq = sequences[q];
    const int f = static_cast<int>(rest / s.cout), o = static_cast<int>(rest % s.cout);
    float sum = 0.0f;
    for (int tap = 0; tap < s.kernel; ++tap)
    {
        const int src = f * s.stride + tap * s.dilation - s.padding;
        if (src < 0 || src >= seq.in_frames)
            continue;
        const float* xr = x + static_cast<size_t>(seq.in_offset + src) * s.cin;
        const float* wr = w + static_cast<size_t>(tap) * s.cin * s.cout + o;
        for (int c = 0; c < s.cin; ++c)
            sum = __fadd_rn(sum, __fmul_rn(xr[c], wr[static_cast<size_t>(c) * s.cout]));
    }
    const float v = __fadd_rn(sum, bias[o]);
    if (!isfinite(v) && error_word)
        atomicOr(error_word, error_nonfinite);
    y[static_cast<size_t>(seq.out_offset + f) * s.cout + o] = v;
}

// The same per-output chains from shared memory.  A CTA owns NARROW_TILE
// consecutive output frames of one sequence: it stages the input rows they
// read ([row][channel] in global memory, loaded coalesced) transposed to
// [channel][row] (consecutive threads then read consecutive words) and the
// weights, and each thread runs its frame's chains (taps ascending, channels
// ascending, out-of-window taps skipped) exactly as conv1d_narrow_kernel.
constexpr int NARROW_TILE = 128;

__host__ __device__ constexpr int narrow_span(int stride, int kernel, int dilation)
{
    return (NARROW_TILE - 1) * stride + (kernel - 1) * dilation + 1;
}

template <int COUT> // 1 or 2 output channels, or 0: any (run one after another)
__global__ void __launch_bounds__(NARROW_TILE)
    conv1d_narrow_tile_kernel(const float* __restrict__ x, const float* __restrict__ w,
                              const float* __restrict__ bias, float* __restrict__ y,
                              const Sequence* __restrict__ sequences, int sequence_count, ConvShape s,
                              unsigned* error_word)
{
    extern __shared__ float narrow_smem[];
    const int span = narrow_span(s.stride, s.kernel, s.dilation);
    const int pitch = span + 1;
    float* xs = narrow_smem;             // [cin][pitch]
    float* ws = xs + s.cin * pitch;      // [tap][cin][cout]
    const int t = threadIdx.x;
    int tile = blockIdx.x, q = 0;
    for (; q < sequence_count; ++q)
    {
        const int n = (sequences[q].out_frames + NARROW_TILE - 1) / NARROW_TILE;
        if (tile < n)
            break;
        tile -= n;
    }
    if (q == sequence_count)
        return; // uniform: the grid holds exactly the tiles
    const Sequence seq = sequences[q];
    const int f0 = tile * NARROW_TILE;
    const int r0 = f0 * s.stride - s.padding; // input row of window row 0
    const int weights = s.kernel * s.cin * s.cout;
    for (int i = t; i < weights; i += NARROW_TILE)
        ws[i] = __ldg(w + i);
    // Window rows in memory order: element i is (row i / cin, channel i % cin).
    int row = t / s.cin, c = t % s.cin;
    for (int i = t; i < span * s.cin; i += NARROW_TILE)
    {
        const int src = r0 + row;
        xs[c * pitch + row] =
            src >= 0 && src < seq.in_frames ? __ldg(x + static_cast<size_t>(seq.in_offset + src) * s.cin + c) : 0.0f;
        c += NARROW_TILE;
        while (c >= s.cin)
        {
            c -= s.cin;
            ++row;
        }
    }
    __syncthreads();
    const int f = f0 + t;
    if (f >= seq.out_frames)
        return;
    bool finite = true;
    if constexpr (COUT > 0)
    {
        // The COUT chains advance together (one input load feeds them), each
        // in its own order.
        float sum[COUT];
#pragma unroll
        for (int o = 0; o < COUT; ++o)
            sum[o] = 0.0f;
        for (int tap = 0; tap < s.kernel; ++tap)
        {
            const int src = f * s.stride + tap * s.dilation - s.padding;
            if (src < 0 || src >= seq.in_frames)
                continue;
            const float* xr = xs + (src - r0);
            const float* wr = ws + tap * s.cin * COUT;
#pragma unroll 8
            for (int ch = 0; ch < s.cin; ++ch)
            {
                const float xv = xr[ch * pitch];
#pragma unroll
                for (int o = 0; o < COUT; ++o)
                    sum[o] = __fadd_rn(sum[o], __fmul_rn(xv, wr[ch * COUT + o]));
            }
        }
#pragma unroll
        for (int o = 0; o < COUT; ++o)
        {
            const float v = __fadd_rn(sum[o], __ldg(bias + o));
            finite = finite && isfinite(v);
            y[static_cast<size_t>(seq.out_offset + f) * COUT + o] = v;
        }
    }
    else
    {
        for (int o = 0; o < s.cout; ++o)
        {
            float sum = 0.0f;
            for (int tap = 0; tap < s.kernel; ++tap)
            {
                const int src = f * s.stride + tap * s.dilation - s.padding;
                if (src < 0 || src >= seq.in_frames)
                    continue;
                const float* xr = xs + (src - r0);
                const float* wr = ws + tap * s.cin * s.cout + o;
#pragma unroll 8
                for (int ch = 0; ch < s.cin; ++ch)
                    sum = __fadd_rn(sum, __fmul_rn(xr[ch * pitch], wr[ch * s.cout]));
            }
            const float v = __fadd_rn(sum, __ldg(bias + o));
            finite = finite && isfinite(v);
            y[static_cast<size_t>(seq.out_offset + f) * s.cout + o] = v;
        }
    }
    if (!finite && error_word)
        atomicOr(error_word, error_nonfinite);
}

template <int COUT>
void launch_narrow_tiles(const float* x, const float* w, const float* bias, float* y, const Sequence* sequences,
                         int sequence_count, const ConvShape& s, unsigned* error_word, cudaStream_t stream,
                         long long tiles, size_t smem, size_t smem_limit)
{
    static std::once_flag attr_once[64];
    int device = 0;
    cudaGetDevice(&device);
    if (device >= 0 && device < 64)
        std::call_once(attr_once[device],
                       [smem_limit]
                       {
                           cudaFuncSetAttribute(conv1d_narrow_tile_kernel<COUT>,
                                                cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                static_cast<int>(smem_limit));
                       });
    conv1d_narrow_tile_kernel<COUT><<<static_cast<int>(tiles), NARROW_TILE, smem, stream>>>(
        x, w, bias, y, sequences, sequence_count, s, error_word);
}

// ---------------------------------------------------------------- RVQ ----
struct ArgMax
{
    float value;
    int index;
};

// Strict `>` over ascending indices keeps the lowest index among equal maxima.
__device__ __forceinline__ ArgMax better(ArgMax a, ArgMax b)
{
    return (a.value < b.value || (a.value == b.value && b.index < a.index)) ? b : a;
}

// The runner-up similarity of a search (MARGIN variant): the largest value
// among the candidates other than the selected one (equal maxima count, so an
// exact tie leaves a zero margin).
struct TopTwo
{
    ArgMax best;
    float second;
};

__device__ __forceinline__ TopTwo merge(TopTwo a, const TopTwo& b)
{
    const ArgMax winner = better(a.best, b.best);
    const float loser = (winner.index == a.best.index && winner.value == a.best.value) ? b.best.value
                                                                                       : a.best.value;
    a.second = fmaxf(fmaxf(a.second, b.second), loser);
    a.best = winner;
    return a;
}

// MARGIN: also flags the frame in uncertain[frame] when, for any book, the
// winning similarity beats the runner-up by less than `margin` (or is not
// finite); the certified fast analysis recomputes such frames exactly.
template <bool MARGIN>
__global__ void __launch_bounds__(256)
    rvq_encode_kernel(const float* __restrict__ latent, const RvqBookDevice* __restrict__ books,
                      int book_count, std::uint16_t* __restrict__ tokens, int token_stride,
                      unsigned* error_word, float margin, unsigned char* __restrict__ uncertain)
{
    __shared__ float residual[1024];
    __shared__ float projected[8];
    __shared__ float query[8];
    __shared__ ArgMax warp_best[8];
    __shared__ float warp_second[8];
    __shared__ int selected;
    bool doubtful = false;
    const int frame = blockIdx.x, t = threadIdx.x, lane = t & 31, warp = t >> 5;
    for (int i = t; i < 1024; i += 256)
        residual[i] = latent[static_cast<size_t>(frame) * 1024 + i];
    __syncthreads();
    bool ok = true;
    for (int b = 0; b < book_count; ++b)
    {
        const RvqBookDevice book = books[b];
        // In-projection 1024 -> 8: eight serial chains (one per output, lane 0 of warps 0-7).
        if (lane == 0)
        {
            const float* wr = book.input_weights + warp * 1024;
            float sum = 0.0f;
            for (int i = 0; i < 1024; ++i)
                sum = __fadd_rn(sum, __fmul_rn(residual[i], wr[i]));
            projected[warp] = __fadd_rn(sum, book.input_bias[warp]);
        }
        __syncthreads();
        if (t == 0)
        {
            // normalize_search: pair tree of squares, RMS with epsilon 0x2b8cbccc.
            float sq[8];
            for (int i = 0; i < 8; ++i)
                sq[i] = __fmul_rn(projected[i], projected[i]);
            for (int width = 8; width > 1; width /= 2)
                for (int i = 0; i < width / 2; ++i)
                    sq[i] = __fadd_rn(sq[2 * i], sq[2 * i + 1]);
            ok = ok && isfinite(sq[0]);
            const float mean = __fmul_rn(sq[0], 0.125f);
            const float inverse_rms =
                __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, __uint_as_float(0x2b8cbcccu))));
            const float inverse_width = __fdiv_rn(1.0f, __fsqrt_rn(8.0f));
            for (int i = 0; i < 8; ++i)
                query[i] = __fmul_rn(__fmul_rn(projected[i], inverse_rms), inverse_width);
        }
        __syncthreads();
        TopTwo top{{-INFINITY, 1 << 20}, -INFINITY};
        for (int index = t; index < 1024; index += 256)
        {
            const float* v = book.search + index * 8;
            float similarity = 0.0f;
#pragma unroll
            for (int i = 0; i < 8; ++i)
                similarity = __fmaf_rn(v[i], query[i], similarity);
            // Candidates that never exceed -inf (NaN) are never selected, as in the reference.
            if (similarity > -INFINITY || index == 0)
            {
                const TopTwo one{{similarity > -INFINITY ? similarity : -INFINITY, index}, -INFINITY};
                top = MARGIN ? merge(top, one) : TopTwo{better(top.best, one.best), -INFINITY};
            }
        }
#pragma unroll
        for (int offset = 16; offset > 0; offset >>= 1)
        {
            const TopTwo other{{__shfl_xor_sync(0xffffffffu, top.best.value, offset),
                                __shfl_xor_sync(0xffffffffu, top.best.index, offset)},
                               __shfl_xor_sync(0xffffffffu, top.second, offset)};
            top = MARGIN ? merge(top, other) : TopTwo{better(top.best, other.best), -INFINITY};
        }
        if (lane == 0)
        {
            warp_best[warp] = top.best;
            warp_second[warp] = top.second;
        }
        __syncthreads();
        if (t == 0)
        {
            TopTwo all{warp_best[0], warp_second[0]};
            for (int i = 1; i < 8; ++i)
                all = MARGIN ? merge(all, TopTwo{warp_best[i], warp_second[i]})
                             : TopTwo{better(all.best, warp_best[i]), -INFINITY};
            // A reference search that never passes -inf keeps index 0.
            selected = all.best.value > -INFINITY ? all.best.index : 0;
            tokens[static_cast<size_t>(frame) * token_stride + b] =
                static_cast<std::uint16_t>(selected);
            if (MARGIN)
                doubtful = doubtful || !(__fsub_rn(all.best.value, all.second) >= margin) ||
                           !isfinite(all.best.value);
        }
        __syncthreads();
        const float* cb = book.codebook + selected * 8;
        for (int j = t; j < 1024; j += 256)
        {
            const float* wr = book.output_weights + j * 8;
            float sum = 0.0f;
#pragma unroll
            for (int i = 0; i < 8; ++i)
                sum = __fmaf_rn(wr[i], cb[i], sum);
            const float contribution = __fadd_rn(sum, book.output_bias[j]);
            residual[j] = __fsub_rn(residual[j], contribution);
            ok = ok && isfinite(residual[j]);
        }
        __syncthreads();
    }
    if (!__syncthreads_and(ok) && t == 0 && error_word)
        atomicOr(error_word, error_nonfinite);
    if (MARGIN && t == 0)
        uncertain[frame] = doubtful ? 1 : 0;
}

__global__ void rvq_decode_kernel(const std::uint16_t* __restrict__ tokens, int token_stride,
                                  const RvqBookDevice* __restrict__ books, int book_count,
                                  float* __restrict__ latent)
{
    const int frame = blockIdx.x;
    for (int j = threadIdx.x; j < 1024; j += blockDim.x)
    {
        float acc = 0.0f;
        for (int b = 0; b < book_count; ++b)
        {
            const RvqBookDevice book = books[b];
            const int token = tokens[static_cast<size_t>(frame) * token_stride + b] & 1023;
            const float* wr = book.output_weights + j * 8;
            const float* cb = book.codebook + token * 8;
            float sum = 0.0f;
#pragma unroll
            for (int i = 0; i < 8; ++i)
                sum = __fmaf_rn(wr[i], cb[i], sum);
            acc = __fadd_rn(acc, __fadd_rn(sum, book.output_bias[j]));
        }
        latent[static_cast<size_t>(frame) * 1024 + j] = acc;
    }
}

__global__ void check_finite_kernel(const float* __restrict__ x, long long count,
                                    unsigned* error_word)
{
    bool ok = true;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < count;
         i += static_cast<long long>(gridDim.x) * blockDim.x)
        ok = ok && isfinite(x[i]);
    if (!ok)
        atomicOr(error_word, error_nonfinite);
}
} // namespace

void snake(const float* x, const float* alpha, int channels, long long frames, float* y,
           unsigned* error_word, cudaStream_t stream)
{
    const long long count = frames * channels;
    if (count <= 0)
        return;
    long long blocks = (count + 255) / 256;
    blocks = blocks > 148 * 16 ? 148 * 16 : blocks;
    snake_kernel<<<static_cast<int>(blocks), 256, 0, stream>>>(x, alpha, channels, count, y,
                                                               error_word);
    note_launch();
}

int conv_tile_frames(const ConvShape&)
{
    return TF;
}

template <int TO, int THREADS, bool FAST> void launch_conv(const ConvLaunch& l, cudaStream_t stream)
{
    constexpr size_t smem = conv_smem_bytes<TO>();
    static std::once_flag attr_once[64];
    int device = 0;
    cudaGetDevice(&device);
    if (device >= 0 && device < 64)
        std::call_once(attr_once[device],
                       []
                       {
                           cudaFuncSetAttribute(conv1d_kernel<TO, THREADS, FAST>,
                                                cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                static_cast<int>(smem));
                       });
    const dim3 grid(l.tile_count, (l.shape.cout + TO - 1) / TO);
    conv1d_kernel<TO, THREADS, FAST><<<grid, THREADS, smem, stream>>>(l);
    note_launch();
}

void conv1d(const ConvLaunch& l, cudaStream_t stream)
{
    if (l.tile_count <= 0)
        return;
    // 128-channel tiles of 512 threads (4 x 8 chains each, one CTA per SM)
    // where the layer is at least that wide; 64-channel tiles of 256 threads
    // for the 64-channel layers.  (The 256-thread tile at two CTAs per SM on
    // the wide layers measured 0.59 of FP32 issue against 0.63.)
    if (l.shape.cout >= 128)
        l.fast ? launch_conv<128, 512, true>(l, stream) : launch_conv<128, 512, false>(l, stream);
    else
        l.fast ? launch_conv<64, 256, true>(l, stream) : launch_conv<64, 256, false>(l, stream);
}

void conv1d_narrow(const float* x, const float* w, const float* bias, float* y,
                   const Sequence* sequences, int sequence_count, const ConvShape& s,
                   long long total_outputs, unsigned* error_word, cudaStream_t stream,
                   long long tiles)
{
    if (total_outputs <= 0)
        return;
    // Staged form where the window and weights fit in shared memory.
    constexpr size_t smem_limit = 200 * 1024;
    const size_t smem = (static_cast<size_t>(s.cin) * (narrow_span(s.stride, s.kernel, s.dilation) + 1) +
                         static_cast<size_t>(s.kernel) * s.cin * s.cout) *
                        sizeof(float);
    if (!s.transposed && tiles > 0 && tiles < (1ll << 31) && smem <= smem_limit)
    {
        if (s.cout == 1)
            launch_narrow_tiles<1>(x, w, bias, y, sequences, sequence_count, s, error_word, stream, tiles, smem,
                                   smem_limit);
        else if (s.cout == 2)
            launch_narrow_tiles<2>(x, w, bias, y, sequences, sequence_count, s, error_word, stream, tiles, smem,
                                   smem_limit);
        else
            launch_narrow_tiles<0>(x, w, bias, y, sequences, sequence_count, s, error_word, stream, tiles, smem,
                                   smem_limit);
        note_launch();
        return;
    }
    conv1d_narrow_kernel<<<static_cast<int>((total_outputs + 127) / 128), 128, 0, stream>>>(
        x, w, bias, y, sequences, sequence_count, s, total_outputs, error_word);
    note_launch();
}

void rvq_encode(const float* latent, int frames, const RvqBookDevice* books, int book_count,
                std::uint16_t* tokens, int token_stride, unsigned* error_word, cudaStream_t stream)
{
    if (frames > 0)
    {
        rvq_encode_kernel<false><<<frames, 256, 0, stream>>>(latent, books, book_count, tokens, token_stride,
                                                             error_word, 0.0f, nullptr);
        note_launch();
    }
}

void rvq_encode_margins(const float* latent, int frames, const RvqBookDevice* books, int book_count,
                        std::uint16_t* tokens, int token_stride, float margin, unsigned char* uncertain,
                        unsigned* error_word, cudaStream_t stream)
{
    if (frames > 0)
    {
        rvq_encode_kernel<true><<<frames, 256, 0, stream>>>(latent, books, book_count, tokens, token_stride,
                                                            error_word, margin, uncertain);
        note_launch();
    }
}

void rvq_decode(const std::uint16_t* tokens, int token_stride, int frames,
                const RvqBookDevice* books, int book_count, float* latent, cudaStream_t stream)
{
    if (frames > 0)
    {
        rvq_decode_kernel<<<frames, 256, 0, stream>>>(tokens, token_stride, books, book_count,
                                                      latent);
        note_launch();
    }
}

void check_finite(const float* x, long long count, unsigned* error_word, cudaStream_t stream)
{
    if (count > 0)
    {
        check_finite_kernel<<<148 * 4, 256, 0, stream>>>(x, count, error_word);
        note_launch();
    }
}

namespace
{
__global__ void pcm_regroup_kernel(const float* __restrict__ src, long long samples,
                                   long long channel_stride, long long sample_stride, int groups,
                                   int mc, long long padded, float* __restrict__ dst,
                                   unsigned* error_word)
{
    const long long total = static_cast<long long>(groups) * padded * mc;
    bool ok = true;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<long long>(gridDim.x) * blockDim.x)
    {
        const int c = static_cast<int>(i % mc);
        const long long f = (i / mc) % padded;
        const int g = static_cast<int>(i / (static_cast<long long>(mc) * padded));
        float v = 0.0f;
        if (f < samples)
        {
            v = src[static_cast<long long>(g * mc + c) * channel_stride + f * sample_stride];
            ok = ok && isfinite(v);
        }
        dst[i] = v;
    }
    if (!ok && error_word)
        atomicOr(error_word, error_nonfinite);
}
} // namespace

void pcm_regroup(const float* src, long long samples, long long channel_stride,
                 long long sample_stride, int groups, int model_channels, long long padded,
                 float* dst, unsigned* error_word, cudaStream_t stream)
{
    const long long total = static_cast<long long>(groups) * padded * model_channels;
    if (total <= 0)
        return;
    long long blocks = (total + 255) / 256;
    blocks = blocks > 148 * 8 ? 148 * 8 : blocks;
    pcm_regroup_kernel<<<static_cast<int>(blocks), 256, 0, stream>>>(
        src, samples, channel_stride, sample_stride, groups, model_channels, padded, dst,
        error_word);
    note_launch();
}
} // namespace tsacb::dev
