// C ABI: one tensor-core (3xTF32 tcgen05) convolution over a single sequence,
// for kernel-level accuracy tests and microbenchmarks.  The codec's decoder
// drives the same kernel through DacEngine on its padded multi-window layout;
// this entry point builds that layout for one sequence around the caller's
// tensors (it allocates and frees device memory, so it is not for hot loops).
#include "cuda_util.cuh"
#include "host/snake_inverse.hpp"
#include "host/tf32_split.hpp"
#include "kernels/tc_conv.cuh"

#include <cstring>
#include <vector>

namespace
{
struct DeviceBlock
{
    void* p = nullptr;
    explicit DeviceBlock(size_t bytes)
    {
        tsacb::cuda_check(cudaMalloc(&p, bytes ? bytes : 1), "cudaMalloc");
    }
    ~DeviceBlock()
    {
        if (p)
            cudaFree(p);
    }
    template <class T> T* as() const
    {
        return static_cast<T*>(p);
    }
};

} // namespace

extern "C"
{
int tsac_cuda_conv1d_tensor(const float* x, size_t frames, const float* weights, const float* bias,
                            const float* residual, const float* alpha, float* y, size_t cin,
                            size_t cout, size_t kernel, size_t stride, size_t padding,
                            size_t dilation, int transposed, unsigned* error_word, void* stream)
{
    return tsacb::guarded(
        [&]
        {
            using namespace tsacb;
            require_device();
            require(x && weights && bias && y && error_word, "null argument");
            require(frames > 0 && frames <= (1u << 24), "convolution frames out of range");
            require(dev::tc_conv_supported(static_cast<int>(cin), static_cast<int>(cout)),
                    "tensor-core convolution needs cin % 32 == 0 and cout a multiple of 128 or 96");
            const auto s = static_cast<cudaStream_t>(stream);
            dev::TcConvGeometry g{};
            int gap;
            if (!transposed)
            {
                require(stride == 1 && 2 * padding == (kernel - 1) * dilation && kernel <= 16,
                        "tensor-core convolution needs stride 1 and 'same' padding");
                g.taps = static_cast<int>(kernel);
                g.phases = 1;
                g.tap_step = static_cast<int>(dilation);
                g.row_shift[0] = -static_cast<int>(padding);
                gap = static_cast<int>(padding) + 1;
            }
            else
            {
                require(dilation == 1 && kernel == 2 * stride && 2 * padding == stride && stride <= 8,
                        "tensor-core transposed convolution needs kernel 2s and padding s/2");
                g.taps = 2;
                g.phases = static_cast<int>(stride);
                g.tap_step = -1;
                for (int r = 0; r < g.phases; ++r)
                    g.row_shift[r] = (r + static_cast<int>(padding)) / g.phases;
                gap = 2;
            }
            const long long in_rows = static_cast<long long>(frames) + 2 * gap;
            g.rows = in_rows;
            g.cin = static_cast<int>(cin);
            g.cout = static_cast<int>(cout);
            g.out_stride = g.phases;
            g.in_rows = in_rows;
            g.out_rows = in_rows * g.phases;
            g.out_scale = g.phases;

            // Weights [tap][cin][cout] -> slices [slice][cout][cin], head/tail.
            std::vector<float> w(kernel * cin * cout), t;
            cuda_check(cudaMemcpyAsync(w.data(), weights, w.size() * 4, cudaMemcpyDeviceToHost, s), "D2H");
            cuda_check(cudaStreamSynchronize(s), "conv weights");
            const int slices = g.taps * g.phases;
            t.resize(static_cast<size_t>(slices) * cout * cin);
            for (int sl = 0; sl < slices; ++sl)
            {
                int tap = sl;
                if (transposed)
                {
                    const int r = sl / 2, j = sl % 2;
                    tap = (r + static_cast<int>(padding)) % g.phases + j * g.phases;
                }
                for (size_t o = 0; o < cout; ++o)
                    for (size_t i = 0; i < cin; ++i)
                        t[(static_cast<size_t>(sl) * cout + o) * cin + i] = w[(tap * cin + i) * cout + o];
            }
            std::vector<float> whi, wlo;
            split_tf32(t, whi, wlo);
            DeviceBlock d_whi(whi.size() * 4), d_wlo(wlo.size() * 4);
            cuda_check(cudaMemcpyAsync(d_whi.p, whi.data(), whi.size() * 4, cudaMemcpyHostToDevice, s), "H2D");
            cuda_check(cudaMemcpyAsync(d_wlo.p, wlo.data(), wlo.size() * 4, cudaMemcpyHostToDevice, s), "H2D");

            // Input rows [gap, gap + frames) of the padded layout, zeros around.
            std::vector<long long> map(frames);
            for (size_t f = 0; f < frames; ++f)
                map[f] = gap + static_cast<long long>(f);
            std::vector<unsigned char> valid(static_cast<size_t>(in_rows), 0);
            for (size_t f = 0; f < frames; ++f)
                valid[gap + f] = 1;
            DeviceBlock d_map(map.size() * 8), d_valid(valid.size());
            cuda_check(cudaMemcpyAsync(d_map.p, map.data(), map.size() * 8, cudaMemcpyHostToDevice, s), "H2D");
            cuda_check(cudaMemcpyAsync(d_valid.p, valid.data(), valid.size(), cudaMemcpyHostToDevice, s), "H2D");
            const size_t in_bytes = static_cast<size_t>(in_rows) * cin * 4;
            DeviceBlock xhi(in_bytes), xlo(in_bytes);
            cuda_check(cudaMemsetAsync(xhi.p, 0, in_bytes, s), "memset");
            cuda_check(cudaMemsetAsync(xlo.p, 0, in_bytes, s), "memset");
            dev::pad_split_rows(x, static_cast<long long>(frames), static_cast<int>(cin),
                                d_map.as<long long>(), xhi.as<float>(), xlo.as<float>(), s);

            const size_t out_bytes = static_cast<size_t>(g.out_rows) * cout * 4;
            const size_t first = static_cast<size_t>(gap) * g.phases * cout;
            const size_t count = frames * g.phases * cout;
            DeviceBlock out(out_bytes), res(residual ? out_bytes : 0);
            if (residual)
                cuda_check(cudaMemcpyAsync(res.as<float>() + first, residual, count * 4,
                                           cudaMemcpyDeviceToDevice, s),
                           "D2D");
            // The kernel reads bias / alpha in 16-byte loads: aligned copies.
            DeviceBlock d_bias(cout * 4), d_alpha(alpha ? cout * 4 : 0);
            cuda_check(cudaMemcpyAsync(d_bias.p, bias, cout * 4, cudaMemcpyDeviceToDevice, s), "D2D");
            if (alpha)
                cuda_check(cudaMemcpyAsync(d_alpha.p, alpha, cout * 4, cudaMemcpyDeviceToDevice, s), "D2D");
            DeviceBlock d_inverse(alpha ? cout * 4 : 0);
            if (alpha)
            {
                std::vector<float> a(cout);
                cuda_check(cudaMemcpyAsync(a.data(), alpha, cout * 4, cudaMemcpyDeviceToHost, s), "D2H");
                cuda_check(cudaStreamSynchronize(s), "alpha");
                const auto inverse = tsacb::snake_inverse(a);
                cuda_check(cudaMemcpyAsync(d_inverse.p, inverse.data(), cout * 4, cudaMemcpyHostToDevice, s),
                           "H2D");
            }
            const dev::TcConvEpilogue e{d_bias.as<float>(), residual ? res.as<float>() : nullptr,
                                        alpha ? nullptr : out.as<float>(), alpha ? d_alpha.as<float>() : nullptr,
                                        alpha ? d_inverse.as<float>() : nullptr,
                                        alpha ? out.as<float>() : nullptr, nullptr,
                                        d_valid.as<unsigned char>(), error_word};
            const dev::TcConvOperands op{xhi.as<float>(), xlo.as<float>(), d_whi.as<float>(),
                                         d_wlo.as<float>()};
            cuda_check(dev::tc_conv(op, g, e, s), "tensor-core convolution");
            cuda_check(cudaMemcpyAsync(y, out.as<float>() + first, count * 4, cudaMemcpyDeviceToDevice, s),
                       "D2D");
            cuda_check(cudaStreamSynchronize(s), "tensor-core convolution");
        });
}
}
