// DAC analysis (encoder) / synthesis (decoder) and the residual VQ on the
// device, over batches of independent windows.
//
// DacAnalysis::apply / DacSynthesis::apply (src/common/analysis.tpp:169-214,
// src/common/synthesis.tpp:168-213) evaluate one window at a time with zero
// padding at the window edges; here every window of a call (all chunks of all
// recordings) is one "sequence" of a single launch per layer.
#pragma once
#include "device.hpp"
#include "models.hpp"
#include "kernels/dac.cuh"

namespace tsacb
{
struct DeviceConv
{
    Conv1dSpec spec;
    DeviceBuffer weights; // [tap][in][out]
    DeviceBuffer bias;
    // Tensor-core synthesis operands (empty when the shape stays on the exact
    // kernels): [slice][out][in] TF32 head and fp32 tail; see tc_conv.cuh.
    DeviceBuffer tc_hi, tc_lo;
    int tc_taps = 0, tc_phases = 0, tc_step = 0;
    int tc_shift[8] = {};
};

class DacEngine
{
public:
    DacEngine(const PreparedDac& dac, cudaStream_t stream);
    unsigned channels() const
    {
        return channels_;
    }
    // Analysis: window w reads frames[w]*512 PCM rows [C] starting at row
    // offsets[w] of `pcm` -> latent [sum of frames][1024] (windows in order).
    // fast: fused multiply-add convolutions (the certified fast analysis;
    // latents differ from the reference's in the last bits).
    void analyze(const float* pcm, const std::vector<long long>& offsets,
                 const std::vector<int>& frames, float* latent, bool fast = false);
    // Synthesis: latent windows [sum of frames][1024] -> pcm [sum frames*512][C].
    // Tensor-core mode (the default) runs the wide convolutions as 3xTF32
    // tcgen05 GEMMs (PCM within tolerance of the reference); exact mode keeps
    // the reference's serial arithmetic (PCM bit-identical).
    void synthesize(const float* latent, const std::vector<int>& frames, float* pcm);
    void set_exact_synthesis(bool exact)
    {
        exact_synthesis_ = exact;
    }
    bool exact_synthesis() const
    {
        return exact_synthesis_;
    }
    unsigned* error_word() const
    {
        return error_.as<unsigned>();
    }
    void check_errors(const char* what);

private:
    struct Layout; // per-layer sequence tables for one window set
    // y (raw result, or null) and optionally act = Snake(alpha)(result).
    void conv(int index, const float* x, float* y, const float* residual,
              const std::vector<int>& in_frames, std::vector<int>& out_frames,
              const std::vector<long long>* in_offsets = nullptr, int alpha = -1,
              float* act = nullptr);
    void snake(int index, const float* x, float* y, long long frames);
    void synthesize_exact(const float* latent, const std::vector<int>& frames, float* pcm);
    void synthesize_tensor(const float* latent, const std::vector<int>& frames, float* pcm);
    void tc_conv(int index, const float* x_hi, const float* x_lo, long long in_rows, int in_scale,
                 const float* residual, float* raw, int alpha, float* hi, float* lo,
                 const unsigned char* valid);

    bool synthesis_;
    bool exact_synthesis_ = false;
    bool fast_analysis_ = false; // set for the duration of a fast analyze()
    bool tensor_ready_ = true; // every wide synthesis convolution has tensor operands
    long long tc_valid_latent_ = 0;
    unsigned channels_;
    std::vector<DeviceConv> convs_;
    std::vector<DeviceBuffer> alphas_;
    std::vector<DeviceBuffer> alpha_inverses_; // synthesis: 1 / (alpha + eps) per Snake
    std::vector<int> alpha_width_;
    cudaStream_t stream_;
    Workspace ws_;
    DeviceBuffer error_;
};

class RvqEngine
{
public:
    RvqEngine(const std::vector<PreparedRvqBook>& books, cudaStream_t stream);
    // latent [frames][1024] (consumed as residual) -> tokens [frames][stride], books 0..count-1.
    void encode(const float* latent, int frames, int books, std::uint16_t* tokens, int stride);
    // encode, flagging uncertain[f] = 1 for frames where any book's winning
    // similarity leads the runner-up by less than `margin`.
    void encode_margins(const float* latent, int frames, int books, std::uint16_t* tokens, int stride,
                        float margin, unsigned char* uncertain);
    void decode(const std::uint16_t* tokens, int stride, int frames, int books, float* latent);
    unsigned* error_word() const
    {
        return error_.as<unsigned>();
    }

private:
    std::vector<DeviceBuffer> storage_;
    DeviceBuffer table_; // RvqBookDevice[books]
    int books_ = 0;
    cudaStream_t stream_;
    DeviceBuffer error_;
};
} // namespace tsacb
