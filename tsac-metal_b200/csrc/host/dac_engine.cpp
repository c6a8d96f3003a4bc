#include "dac_engine.hpp"

#include "kernel_timer.hpp"
#include "snake_inverse.hpp"
#include "tf32_split.hpp"
#include "kernels/error_bits.hpp"
#include "kernels/tc_conv.cuh"

#include <algorithm>
#include <array>

namespace tsacb
{
namespace
{
// Reference folded weights -> device [tap][in][out] (layout only).
std::vector<float> device_layout(const PreparedConv& c)
{
    const auto& s = c.spec;
    const std::size_t cin = s.input_channels, cout = s.output_channels, k = s.kernel;
    std::vector<float> out(c.weights.size());
    for (std::size_t tap = 0; tap < k; ++tap)
        for (std::size_t in = 0; in < cin; ++in)
            for (std::size_t o = 0; o < cout; ++o)
                out[(tap * cin + in) * cout + o] =
                    s.transposed ? c.weights[o + tap * cout + in * cout * k]
                                 : c.weights[in + tap * cin + o * cin * k];
    return out;
}

// Tensor-core operands of a synthesis convolution (tc_conv.cuh geometry), or
// false when the shape stays on the exact kernels.  Ordinary: "same" length
// (2 padding == (kernel - 1) dilation, stride 1), slices = taps.  Transposed:
// kernel 2s, padding s/2, output = input x s; phase r of the output takes taps
// b = (r + p) mod s and b + s from input rows i + (r + p) div s and one less.
bool build_tensor_operands(DeviceConv& d, const PreparedConv& c, cudaStream_t stream)
{
    const auto& s = c.spec;
    const int cin = static_cast<int>(s.input_channels), cout = static_cast<int>(s.output_channels);
    const int k = static_cast<int>(s.kernel);
    if (!dev::tc_conv_supported(cin, cout))
        return false;
    std::vector<float> w;
    if (!s.transposed)
    {
        if (s.stride != 1 || 2 * s.padding != (s.kernel - 1) * s.dilation || k > 16)
            return false;
        d.tc_taps = k;
        d.tc_phases = 1;
        d.tc_step = static_cast<int>(s.dilation);
        d.tc_shift[0] = -static_cast<int>(s.padding);
        w.resize(static_cast<std::size_t>(k) * cout * cin);
        for (int tap = 0; tap < k; ++tap)
            for (int o = 0; o < cout; ++o)
                for (int in = 0; in < cin; ++in)
                    w[(static_cast<std::size_t>(tap) * cout + o) * cin + in] =
                        c.weights[in + static_cast<std::size_t>(tap) * cin + static_cast<std::size_t>(o) * cin * k];
    }
    else
    {
        const int st = static_cast<int>(s.stride), p = static_cast<int>(s.padding);
        if (k != 2 * st || 2 * p != st || st > 8)
            return false;
        d.tc_taps = 2;
        d.tc_phases = st;
        d.tc_step = -1;
        w.resize(static_cast<std::size_t>(st) * 2 * cout * cin);
        for (int r = 0; r < st; ++r)
        {
            d.tc_shift[r] = (r + p) / st;
            const int b = (r + p) % st;
            for (int j = 0; j < 2; ++j)
            {
                const int tap = b + j * st, slice = r * 2 + j;
                for (int o = 0; o < cout; ++o)
                    for (int in = 0; in < cin; ++in)
                        w[(static_cast<std::size_t>(slice) * cout + o) * cin + in] =
                            c.weights[o + static_cast<std::size_t>(tap) * cout + static_cast<std::size_t>(in) * cout * k];
            }
        }
    }
    std::vector<float> hi, lo;
    split_tf32(w, hi, lo);
    d.tc_hi = upload(hi, stream);
    d.tc_lo = upload(lo, stream);
    return true;
}

// Output length of a convolution (src/common/dsp.tpp:141-156).
int output_frames(const Conv1dSpec& s, int frames)
{
    const int span = (static_cast<int>(s.kernel) - 1) * static_cast<int>(s.dilation) + 1;
    const int padding = 2 * static_cast<int>(s.padding);
    if (!s.transposed)
    {
        require(frames + padding >= span, "convolution has no output frames");
        return (frames + padding - span) / static_cast<int>(s.stride) + 1;
    }
    const int full = (frames - 1) * static_cast<int>(s.stride) + span;
    require(full > padding, "transposed convolution has no output frames");
    return full - padding;
}
} // namespace

DacEngine::DacEngine(const PreparedDac& dac, cudaStream_t stream)
    : synthesis_(dac.synthesis), channels_(dac.channels), stream_(stream), error_(sizeof(unsigned))
{
    for (const auto& c : dac.convs)
    {
        require(!c.spec.transposed || c.spec.dilation == 1, "transposed dilation unsupported");
        DeviceConv d;
        d.spec = c.spec;
        d.weights = upload(device_layout(c), stream);
        d.bias = upload(c.bias, stream);
        if (synthesis_ && c.spec.output_channels >= 16)
            tensor_ready_ = build_tensor_operands(d, c, stream) && tensor_ready_;
        convs_.push_back(std::move(d));
    }
    // The synthesis graph this engine drives: the entry convolution, then per
    // stage one transposed convolution and three residual units, then the exit.
    tensor_ready_ = tensor_ready_ && synthesis_ && convs_.size() == 30;
    for (const auto& a : dac.alphas)
    {
        alphas_.push_back(upload(a, stream));
        alpha_width_.push_back(static_cast<int>(a.size()));
        // The tensor-core epilogue's Snake (a stated tolerance, not
        // bit-exactness) multiplies by these instead of dividing.
        if (synthesis_)
            alpha_inverses_.push_back(upload(snake_inverse(a), stream));
    }
    cuda_ok(cudaMemsetAsync(error_.as<void>(), 0, sizeof(unsigned), stream), "memset");
    cuda_ok(cudaStreamSynchronize(stream), "DAC weight upload");
}

void DacEngine::check_errors(const char* what)
{
    unsigned word = 0;
    cuda_ok(cudaMemcpyAsync(&word, error_.as<void>(), 4, cudaMemcpyDeviceToHost, stream_), "D2H");
    cuda_ok(cudaStreamSynchronize(stream_), what);
    if (word)
    {
        cuda_ok(cudaMemsetAsync(error_.as<void>(), 0, 4, stream_), "memset");
        if (word & dev::error_timeout)
            throw DeviceError(std::string("tensor-core pipeline wait timed out (") + what + ")");
        throw NumericError(std::string("nonfinite DSP value (") + what + ")");
    }
}

void DacEngine::snake(int index, const float* x, float* y, long long frames)
{
    KernelTimer::Scope timing("snake", stream_,
                              8.0 * static_cast<double>(frames) * alpha_width_[static_cast<std::size_t>(index)]);
    dev::snake(x, alphas_[static_cast<std::size_t>(index)].as<float>(),
               alpha_width_[static_cast<std::size_t>(index)], frames, y, error_word(), stream_);
}

void DacEngine::conv(int index, const float* x, float* y, const float* residual,
                     const std::vector<int>& in_frames, std::vector<int>& out_frames,
                     const std::vector<long long>* in_offsets, int alpha, float* act)
{
    const auto& c = convs_[static_cast<std::size_t>(index)];
    const auto& sp = c.spec;
    dev::ConvShape shape{static_cast<int>(sp.input_channels), static_cast<int>(sp.output_channels),
                         static_cast<int>(sp.kernel), static_cast<int>(sp.stride),
                         static_cast<int>(sp.padding), static_cast<int>(sp.dilation),
                         sp.transposed};
    std::vector<dev::Sequence> seqs;
    std::vector<int4> tiles;
    out_frames.clear();
    int in_off = 0, out_off = 0;
    const int tf = dev::conv_tile_frames(shape);
    for (std::size_t q = 0; q < in_frames.size(); ++q)
    {
        const int of = output_frames(sp, in_frames[q]);
        const long long start = in_offsets ? (*in_offsets)[q] : in_off;
        require(start + in_frames[q] < (1ll << 31), "convolution input exceeds 2^31 rows");
        seqs.push_back({static_cast<int>(start), in_frames[q], out_off, of});
        out_frames.push_back(of);
        if (sp.transposed)
        {
            for (int phase = 0; phase < shape.stride; ++phase)
            {
                const int count = of > phase ? (of - phase + shape.stride - 1) / shape.stride : 0;
                for (int i0 = 0; i0 < count; i0 += tf)
                    tiles.push_back({static_cast<int>(q), i0, phase, 0});
            }
        }
        else
        {
            for (int f0 = 0; f0 < of; f0 += tf)
                tiles.push_back({static_cast<int>(q), f0, 0, 0});
        }
        in_off += in_frames[q];
        out_off += of;
    }
    const std::string key = "conv" + std::to_string(index);
    auto* d_seq = ws_.get<dev::Sequence>(key + "s", seqs.size());
    cuda_ok(cudaMemcpyAsync(d_seq, seqs.data(), seqs.size() * sizeof(dev::Sequence),
                            cudaMemcpyHostToDevice, stream_),
            "H2D");
    double macs = 0;
    for (int of : out_frames)
        macs += static_cast<double>(of) * shape.cout * shape.cin * (sp.transposed ? 2 : shape.kernel);
    KernelTimer::Scope timing(shape.cout < 16        ? "conv_narrow"
                              : sp.transposed        ? "conv_transposed"
                              : fast_analysis_       ? "conv_fast"
                                                     : "conv_exact",
                              stream_, 2.0 * macs);
    if (shape.cout < 16)
    {
        long long narrow_tiles = 0;
        for (int of : out_frames)
            narrow_tiles += (of + 127) / 128;
        dev::conv1d_narrow(x, c.weights.as<float>(), c.bias.as<float>(), y, d_seq,
                           static_cast<int>(seqs.size()), shape,
                           static_cast<long long>(out_off) * shape.cout, error_word(), stream_, narrow_tiles);
        require(residual == nullptr && act == nullptr, "narrow convolution has no residual or Snake output");
        return;
    }
    auto* d_tiles = ws_.get<int4>(key + "t", tiles.size());
    cuda_ok(cudaMemcpyAsync(d_tiles, tiles.data(), tiles.size() * sizeof(int4),
                            cudaMemcpyHostToDevice, stream_),
            "H2D");
    dev::ConvLaunch l{error_word(), x, c.weights.as<float>(), c.bias.as<float>(), residual, y,
                      d_seq, d_tiles, static_cast<int>(tiles.size()), shape};
    l.fast = fast_analysis_;
    if (act)
    {
        l.alpha = alphas_[static_cast<std::size_t>(alpha)].as<float>();
        l.act = act;
    }
    dev::conv1d(l, stream_);
}

void DacEngine::analyze(const float* pcm, const std::vector<long long>& offsets,
                        const std::vector<int>& frames, float* latent, bool fast)
{
    require(!synthesis_, "analysis on a synthesis model");
    struct Mode
    {
        bool& flag;
        Mode(bool& f, bool value) : flag(f)
        {
            flag = value;
        }
        ~Mode()
        {
            flag = false;
        }
    } mode(fast_analysis_, fast);
    require(offsets.size() == frames.size(), "analysis window table mismatch");
    std::vector<int> f0(frames.size()), f1;
    long long total = 0;
    for (std::size_t i = 0; i < frames.size(); ++i)
    {
        f0[i] = frames[i] * 512;
        total += f0[i];
    }
    // Widest activation: 64 channels at full rate (= 512*64 per frame ... all
    // stages hold frames*512*64/... floats; stage sizes shrink as width grows).
    const std::size_t biggest = static_cast<std::size_t>(total) * 64;
    // a: the residual stream (raw sums); p / q: Snake of it for the next
    // convolution, written by the producing convolution's epilogue.
    auto* a = ws_.get<float>("a", biggest);
    float* p = ws_.get<float>("t1", biggest);
    float* q = ws_.get<float>("t2", biggest);
    std::vector<int> cur = f0;
    conv(0, pcm, a, nullptr, cur, f1, &offsets, 0, p);
    cur = f1;
    for (int stage = 0; stage < 4; ++stage)
    {
        for (int unit = 0; unit < 3; ++unit)
        {
            const int base = 1 + stage * 7 + unit * 2; // convolution index
            const int alpha = stage * 7 + unit * 2;    // activation index of the unit's first Snake
            conv(base, p, nullptr, nullptr, cur, f1, nullptr, alpha + 1, q);
            const int next = unit < 2 ? alpha + 2 : stage * 7 + 6;
            conv(base + 1, q, a, a, cur, f1, nullptr, next, p);
        }
        const int next = stage < 3 ? (stage + 1) * 7 : 28;
        conv(1 + stage * 7 + 6, p, a, nullptr, cur, f1, nullptr, next, q);
        std::swap(p, q);
        cur = f1;
    }
    conv(29, p, latent, nullptr, cur, f1);
    cuda_ok(cudaGetLastError(), "analysis launch");
}

void DacEngine::synthesize(const float* latent, const std::vector<int>& frames, float* pcm)
{
    require(synthesis_, "synthesis on an analysis model");
    if (!exact_synthesis_ && tensor_ready_)
        synthesize_tensor(latent, frames, pcm);
    else
        synthesize_exact(latent, frames, pcm);
}

void DacEngine::tc_conv(int index, const float* x_hi, const float* x_lo, long long in_rows,
                        int in_scale, const float* residual, float* raw, int alpha, float* hi,
                        float* lo, const unsigned char* valid)
{
    const auto& c = convs_[static_cast<std::size_t>(index)];
    dev::TcConvGeometry g{};
    g.rows = in_rows;
    g.cin = static_cast<int>(c.spec.input_channels);
    g.cout = static_cast<int>(c.spec.output_channels);
    g.taps = c.tc_taps;
    g.phases = c.tc_phases;
    g.out_stride = c.tc_phases;
    g.tap_step = c.tc_step;
    for (int r = 0; r < 8; ++r)
        g.row_shift[r] = c.tc_shift[r];
    g.in_rows = in_rows;
    g.out_rows = in_rows * c.tc_phases;
    g.out_scale = in_scale * c.tc_phases;
    const dev::TcConvEpilogue e{c.bias.as<float>(), residual, raw,
                                alpha >= 0 ? alphas_[static_cast<std::size_t>(alpha)].as<float>() : nullptr,
                                alpha >= 0 ? alpha_inverses_[static_cast<std::size_t>(alpha)].as<float>()
                                           : nullptr,
                                hi, lo, valid, error_word()};
    const dev::TcConvOperands op{x_hi, x_lo, c.tc_hi.as<float>(), c.tc_lo.as<float>()};
    // Useful MACs: valid output rows x cout x cin x taps per output.
    const double macs = static_cast<double>(tc_valid_latent_) * g.out_scale * g.cout * g.cin * g.taps;
    KernelTimer::Scope timing("conv_tc", stream_, 2.0 * macs);
    cuda_ok(dev::tc_conv(op, g, e, stream_), "tensor-core convolution");
}

void DacEngine::synthesize_tensor(const float* latent, const std::vector<int>& frames, float* pcm)
{
    // Padded latent rows: G zero rows before, between and after the windows.
    // At every stage the layout is this one scaled by the cumulative
    // upsampling, so gaps grow to >= 32 rows, wider than any tap reach (27).
    constexpr int G = 4;
    const std::size_t count = frames.size();
    std::vector<long long> base(count);
    long long r0 = G, total = 0;
    for (std::size_t q = 0; q < count; ++q)
    {
        require(frames[q] > 0, "synthesis window without frames");
        base[q] = r0;
        r0 += frames[q] + G;
        total += frames[q];
    }
    std::vector<unsigned char> valid(static_cast<std::size_t>(r0), 0);
    std::vector<long long> row_map(static_cast<std::size_t>(total));
    long long k = 0;
    for (std::size_t q = 0; q < count; ++q)
        for (int f = 0; f < frames[q]; ++f)
        {
            valid[static_cast<std::size_t>(base[q] + f)] = 1;
            row_map[static_cast<std::size_t>(k++)] = base[q] + f;
        }
    auto* d_valid = ws_.get<unsigned char>("tc_valid", valid.size());
    auto* d_map = ws_.get<long long>("tc_map", row_map.size());
    cuda_ok(cudaMemcpyAsync(d_valid, valid.data(), valid.size(), cudaMemcpyHostToDevice, stream_), "H2D");
    cuda_ok(cudaMemcpyAsync(d_map, row_map.data(), row_map.size() * sizeof(long long),
                            cudaMemcpyHostToDevice, stream_),
            "H2D");
    const std::size_t widest = static_cast<std::size_t>(r0) * 49152;
    float* a = ws_.get<float>("tc_a", widest);
    float* p[2][2] = {{ws_.get<float>("tc_p0h", widest), ws_.get<float>("tc_p0l", widest)},
                      {ws_.get<float>("tc_p1h", widest), ws_.get<float>("tc_p1l", widest)}};
    tc_valid_latent_ = total;
    const std::size_t latent_bytes = static_cast<std::size_t>(r0) * 1024 * sizeof(float);
    cuda_ok(cudaMemsetAsync(p[0][0], 0, latent_bytes, stream_), "memset");
    cuda_ok(cudaMemsetAsync(p[0][1], 0, latent_bytes, stream_), "memset");
    dev::pad_split_rows(latent, total, 1024, d_map, p[0][0], p[0][1], stream_);

    int cur = 0;
    long long rows = r0;
    int scale = 1;
    // Entry convolution; its epilogue applies stage 0's first Snake.
    tc_conv(0, p[cur][0], p[cur][1], rows, scale, nullptr, nullptr, 0, p[1 - cur][0], p[1 - cur][1], d_valid);
    cur ^= 1;
    for (int stage = 0; stage < 4; ++stage)
    {
        const int up = 1 + stage * 7;
        tc_conv(up, p[cur][0], p[cur][1], rows, scale, nullptr, a, stage * 7 + 1, p[1 - cur][0],
                p[1 - cur][1], d_valid);
        cur ^= 1;
        rows *= convs_[static_cast<std::size_t>(up)].tc_phases;
        scale *= convs_[static_cast<std::size_t>(up)].tc_phases;
        for (int unit = 0; unit < 3; ++unit)
        {
            const int conv_index = up + 1 + unit * 2;
            const int first_alpha = stage * 7 + 1 + unit * 2;
            tc_conv(conv_index, p[cur][0], p[cur][1], rows, scale, nullptr, nullptr, first_alpha + 1,
                    p[1 - cur][0], p[1 - cur][1], d_valid);
            cur ^= 1;
            const bool exit_next = stage == 3 && unit == 2;
            const int next_alpha = unit < 2 ? first_alpha + 2 : (stage < 3 ? (stage + 1) * 7 : 28);
            // Residual sum kept only while another residual unit of the stage reads it.
            tc_conv(conv_index + 1, p[cur][0], p[cur][1], rows, scale, a, unit < 2 ? a : nullptr,
                    next_alpha, p[1 - cur][0], exit_next ? nullptr : p[1 - cur][1], d_valid);
            cur ^= 1;
        }
    }
    // Exit convolution to PCM on the exact kernel, reading Snake(28) rows of
    // the padded layout.
    std::vector<int> in_frames(count), out_frames;
    std::vector<long long> offsets(count);
    for (std::size_t q = 0; q < count; ++q)
    {
        in_frames[q] = frames[q] * scale;
        offsets[q] = base[q] * scale;
    }
    conv(29, p[cur][0], pcm, nullptr, in_frames, out_frames, &offsets);
    cuda_ok(cudaGetLastError(), "synthesis launch");
}

void DacEngine::synthesize_exact(const float* latent, const std::vector<int>& frames, float* pcm)
{
    long long total = 0;
    for (int v : frames)
        total += v;
    // Widest activation: 1536 x n at entry, 768 x 8n after stage 0 ... = 6144n;
    // the last stage holds 96 x 512n = 49152n floats.
    const std::size_t biggest = static_cast<std::size_t>(total) * 49152;
    auto* a = ws_.get<float>("a", biggest);
    auto* t1 = ws_.get<float>("t1", biggest);
    auto* t2 = ws_.get<float>("t2", biggest);
    std::vector<int> cur = frames, f1;
    conv(0, latent, a, nullptr, cur, f1);
    cur = f1;
    for (int stage = 0; stage < 4; ++stage)
    {
        long long n = 0;
        for (int v : cur)
            n += v;
        snake(stage * 7, a, t1, n);
        conv(1 + stage * 7, t1, a, nullptr, cur, f1);
        cur = f1;
        n = 0;
        for (int v : cur)
            n += v;
        for (int unit = 0; unit < 3; ++unit)
        {
            const int base = 1 + stage * 7 + 1 + unit * 2;
            const int alpha = stage * 7 + 1 + unit * 2;
            snake(alpha, a, t1, n);
            conv(base, t1, t2, nullptr, cur, f1);
            snake(alpha + 1, t2, t1, n);
            conv(base + 1, t1, a, a, cur, f1);
        }
    }
    long long n = 0;
    for (int v : cur)
        n += v;
    snake(28, a, t1, n);
    conv(29, t1, pcm, nullptr, cur, f1);
    cuda_ok(cudaGetLastError(), "synthesis launch");
}

// ----------------------------------------------------------------- RVQ ----
RvqEngine::RvqEngine(const std::vector<PreparedRvqBook>& books, cudaStream_t stream)
    : books_(static_cast<int>(books.size())), stream_(stream), error_(sizeof(unsigned))
{
    std::vector<dev::RvqBookDevice> table;
    for (const auto& b : books)
    {
        const auto up = [&](const std::vector<float>& v)
        {
            storage_.push_back(upload(v, stream));
            return storage_.back().as<float>();
        };
        dev::RvqBookDevice d;
        d.input_weights = up(b.input_weights);
        d.input_bias = up(b.input_bias);
        d.search = up(b.search);
        d.codebook = up(b.codebook);
        d.output_weights = up(b.output_weights);
        d.output_bias = up(b.output_bias);
        table.push_back(d);
    }
    table_ = upload(table, stream);
    cuda_ok(cudaMemsetAsync(error_.as<void>(), 0, 4, stream), "memset");
    cuda_ok(cudaStreamSynchronize(stream), "RVQ upload");
}

void RvqEngine::encode(const float* latent, int frames, int books, std::uint16_t* tokens, int stride)
{
    KernelTimer::Scope timing("rvq_encode", stream_, static_cast<double>(frames) * books * 2.0 * (8192 + 8192 + 8192));
    require(books > 0 && books <= books_, "stream and prepared RVQ codebooks do not match");
    dev::rvq_encode(latent, frames, table_.as<dev::RvqBookDevice>(), books, tokens, stride,
                    error_word(), stream_);
}

void RvqEngine::encode_margins(const float* latent, int frames, int books, std::uint16_t* tokens, int stride,
                               float margin, unsigned char* uncertain)
{
    KernelTimer::Scope timing("rvq_encode", stream_, static_cast<double>(frames) * books * 2.0 * (8192 + 8192 + 8192));
    require(books > 0 && books <= books_, "stream and prepared RVQ codebooks do not match");
    dev::rvq_encode_margins(latent, frames, table_.as<dev::RvqBookDevice>(), books, tokens, stride, margin,
                            uncertain, error_word(), stream_);
}

void RvqEngine::decode(const std::uint16_t* tokens, int stride, int frames, int books, float* latent)
{
    require(books > 0 && books <= books_, "stream and prepared RVQ codebooks do not match");
    dev::rvq_decode(tokens, stride, frames, table_.as<dev::RvqBookDevice>(), books, latent, stream_);
}
} // namespace tsacb
