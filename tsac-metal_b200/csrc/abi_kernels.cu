// C ABI: per-kernel entry points (device pointers, caller's stream).  These
// are the calls the parity tests and the kernel microbenchmarks drive; the
// whole-codec entry points build on the same launches.
#include "cuda_util.cuh"
#include "kernels/dac.cuh"
#include "kernels/qlinear.cuh"
#include "kernels/range_decode.cuh"
#include "kernels/transformer_ops.cuh"

#include <vector>

#include <mutex>

namespace
{
std::once_flag init_flag;

void init_kernels()
{
    std::call_once(init_flag, [] { tsacb::dev::qlinear_init(); });
}
} // namespace

extern "C"
{
size_t tsac_cuda_qlinear_scratch_bytes(size_t m, size_t k)
{
    return tsacb::dev::qlinear_scratch_bytes(m, k);
}

int tsac_cuda_qlinear(const int8_t* weights, const float* weight_scales, const float* bias,
                      size_t k, size_t n, const uint16_t* x, size_t m, const uint16_t* residual,
                      uint16_t* y, void* scratch, size_t scratch_bytes, unsigned* error_word,
                      void* stream)
{
    return tsacb::guarded(
        [&]
        {
            using namespace tsacb;
            require_device();
            require(weights && weight_scales && bias && x && y && scratch, "null argument");
            require(k >= 256 && k % 256 == 0 && k <= 8192, "qlinear input width must be 256..8192, a multiple of 256");
            require(n >= 64 && n % 64 == 0, "qlinear output width must be a positive multiple of 64");
            require(m > 0 && m <= (1u << 20), "qlinear column count out of range");
            require(scratch_bytes >= dev::qlinear_scratch_bytes(m, k), "qlinear scratch too small");
            require(aligned16(weights) && aligned16(x) && aligned16(scratch) && aligned16(y),
                    "qlinear buffers must be 16-byte aligned");
            init_kernels();
            auto* xq = static_cast<std::int8_t*>(scratch);
            auto* xs = reinterpret_cast<float*>(static_cast<char*>(scratch) + ((m * k + 255) / 256) * 256);
            const auto s = static_cast<cudaStream_t>(stream);
            dev::qlinear_quantize(x, static_cast<int>(m), static_cast<int>(k), xq, xs, error_word, s);
            dev::QLinearArgs a;
            a.weights = weights;
            a.weight_scales = weight_scales;
            a.bias = bias;
            a.xq = xq;
            a.xscale = xs;
            a.residual = residual;
            a.y = y;
            a.m = static_cast<int>(m);
            a.n = static_cast<int>(n);
            a.k = static_cast<int>(k);
            a.error_word = error_word;
            dev::qlinear_matmul(a, s);
            cuda_check(cudaGetLastError(), "qlinear launch");
        });
}

size_t tsac_cuda_attention_scratch_bytes(size_t rows, size_t max_time)
{
    return tsacb::dev::attention_partials_bytes(static_cast<int>(rows), static_cast<int>(max_time));
}

int tsac_cuda_attention(const uint16_t* query, const int* rows_meta, const uint16_t* keys,
                        const uint16_t* values, size_t rows, size_t max_time, uint16_t* out,
                        void* scratch, size_t scratch_bytes, void* stream)
{
    return tsacb::guarded(
        [&]
        {
            using namespace tsacb;
            require_device();
            require(query && rows_meta && keys && values && out, "null argument");
            require(rows > 0 && rows <= (1u << 20), "attention row count out of range");
            require(max_time > 0 && max_time <= 65535u * 64u, "attention history length out of range");
            require(rows * 4 <= 0x7fffffffu, "attention grid too large");
            require(max_time <= 64 ||
                        (scratch && scratch_bytes >= dev::attention_partials_bytes(static_cast<int>(rows),
                                                                                   static_cast<int>(max_time))),
                    "attention scratch too small");
            require(aligned16(query) && aligned16(keys) && aligned16(values) && aligned16(out),
                    "attention buffers must be 16-byte aligned");
            dev::attention(query, reinterpret_cast<const dev::RowMeta*>(rows_meta), keys, values,
                           static_cast<int>(rows), static_cast<int>(max_time), static_cast<float*>(scratch), out,
                           static_cast<cudaStream_t>(stream));
            cuda_check(cudaGetLastError(), "attention launch");
        });
}

size_t tsac_cuda_conv1d_scratch_bytes(size_t out_frames, int stride, int transposed)
{
    const size_t tiles = (out_frames + 127) / 128 + (transposed ? static_cast<size_t>(stride) : 1);
    return 256 + tiles * sizeof(int4);
}

int tsac_cuda_conv1d(const float* x, size_t frames, const float* weights, const float* bias,
                     const float* residual, float* y, size_t cin, size_t cout, size_t kernel,
                     size_t stride, size_t padding, size_t dilation, int transposed,
                     void* scratch, size_t scratch_bytes, unsigned* error_word, void* stream)
{
    return tsacb::guarded(
        [&]
        {
            using namespace tsacb;
            require_device();
            require(x && weights && bias && y && scratch, "null argument");
            require(cin && cout && kernel && stride && dilation && frames, "empty convolution dimension");
            require(!transposed || dilation == 1, "transposed dilation unsupported");
            require(cin <= (1u << 16) && cout <= (1u << 16) && frames <= (1u << 28),
                    "convolution dimension out of range");
            const size_t span = (kernel - 1) * dilation + 1;
            size_t out_frames;
            if (!transposed)
            {
                require(frames + 2 * padding >= span, "convolution has no output frames");
                out_frames = (frames + 2 * padding - span) / stride + 1;
            }
            else
            {
                const size_t full = (frames - 1) * stride + span;
                require(full > 2 * padding, "transposed convolution has no output frames");
                out_frames = full - 2 * padding;
            }
            require(scratch_bytes >= tsac_cuda_conv1d_scratch_bytes(out_frames, static_cast<int>(stride), transposed),
                    "conv1d scratch too small");
            std::vector<int4> tiles;
            if (transposed)
            {
                for (size_t phase = 0; phase < stride; ++phase)
                {
                    const size_t count = out_frames > phase ? (out_frames - phase + stride - 1) / stride : 0;
                    for (size_t i0 = 0; i0 < count; i0 += 128)
                        tiles.push_back({0, static_cast<int>(i0), static_cast<int>(phase), 0});
                }
            }
            else
            {
                for (size_t f0 = 0; f0 < out_frames; f0 += 128)
                    tiles.push_back({0, static_cast<int>(f0), 0, 0});
            }
            const dev::Sequence seq{0, static_cast<int>(frames), 0, static_cast<int>(out_frames)};
            const auto s = static_cast<cudaStream_t>(stream);
            auto* base = static_cast<char*>(scratch);
            cuda_check(cudaMemcpyAsync(base, &seq, sizeof(seq), cudaMemcpyHostToDevice, s), "H2D");
            cuda_check(cudaMemcpyAsync(base + 256, tiles.data(), tiles.size() * sizeof(int4),
                                       cudaMemcpyHostToDevice, s),
                       "H2D");
            const dev::ConvShape shape{static_cast<int>(cin), static_cast<int>(cout),
                                       static_cast<int>(kernel), static_cast<int>(stride),
                                       static_cast<int>(padding), static_cast<int>(dilation),
                                       transposed != 0};
            if (cout < 16)
            {
                require(!transposed && !residual, "narrow convolution is ordinary without residual");
                dev::conv1d_narrow(x, weights, bias, y, reinterpret_cast<const dev::Sequence*>(base), 1,
                                   shape, static_cast<long long>(out_frames * cout), error_word, s);
            }
            else
            {
                const dev::ConvLaunch l{error_word, x, weights, bias, residual, y,
                                        reinterpret_cast<const dev::Sequence*>(base),
                                        reinterpret_cast<const int4*>(base + 256),
                                        static_cast<int>(tiles.size()), shape};
                dev::conv1d(l, s);
            }
            // The host tile table must outlive the asynchronous copy.
            cuda_check(cudaStreamSynchronize(s), "conv1d");
        });
}

size_t tsac_cuda_range_cursor_bytes(void)
{
    return sizeof(tsacb::dev::RangeCursor);
}

int tsac_cuda_range_start(const uint8_t* bytes, const uint64_t* offsets, const uint64_t* sizes,
                          void* cursors, size_t streams, unsigned* error_word, void* stream)
{
    return tsacb::guarded(
        [&]
        {
            using namespace tsacb;
            require_device();
            require(bytes && offsets && sizes && cursors, "null argument");
            require(streams <= (1u << 24), "range decoder stream count out of range");
            dev::range_start(bytes, offsets, sizes, static_cast<dev::RangeCursor*>(cursors),
                             static_cast<int>(streams), error_word, static_cast<cudaStream_t>(stream));
            cuda_check(cudaGetLastError(), "range start launch");
        });
}

int tsac_cuda_range_decode(const uint8_t* bytes, const uint64_t* offsets, const uint64_t* sizes,
                           void* cursors, size_t streams, const int* rows, size_t count,
                           const float* masses, uint16_t* symbols, unsigned* error_word, void* stream)
{
    return tsacb::guarded(
        [&]
        {
            using namespace tsacb;
            require_device();
            require(bytes && offsets && sizes && cursors && (count == 0 || (rows && masses && symbols)),
                    "null argument");
            require(streams <= (1u << 24) && count <= (1u << 24), "range decoder size out of range");
            dev::range_decode(bytes, offsets, sizes, static_cast<dev::RangeCursor*>(cursors),
                              static_cast<int>(streams), rows, static_cast<int>(count), masses, symbols,
                              error_word, static_cast<cudaStream_t>(stream));
            cuda_check(cudaGetLastError(), "range decode launch");
        });
}

int tsac_cuda_snake(const float* x, size_t channels, size_t frames, const float* alpha, float* y,
                    unsigned* error_word, void* stream)
{
    return tsacb::guarded(
        [&]
        {
            using namespace tsacb;
            require_device();
            require(x && alpha && y && channels, "null argument");
            dev::snake(x, alpha, static_cast<int>(channels), static_cast<long long>(frames), y,
                       error_word, static_cast<cudaStream_t>(stream));
            cuda_check(cudaGetLastError(), "snake launch");
        });
}
}
