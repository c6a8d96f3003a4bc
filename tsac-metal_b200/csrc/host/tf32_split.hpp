// Host-side TF32 head/tail split of weights for the tensor-core convolution:
// hi = nearest TF32 of w (ties away from zero), lo = nearest TF32 of w - hi;
// the device applies the same rule to activations (tc_conv.cu).
#pragma once
#include <cmath>
#include <cstdint>
#include <cstring>
#include <vector>

namespace tsacb
{
inline float tf32_round(float x)
{
    std::uint32_t bits;
    std::memcpy(&bits, &x, 4);
    std::uint32_t r = (bits + 0x1000u) & 0xffffe000u;
    float out;
    std::memcpy(&out, &r, 4);
    if (std::isinf(out) && !std::isinf(x))
    {
        r = bits & 0xffffe000u;
        std::memcpy(&out, &r, 4);
    }
    return out;
}

inline void split_tf32(const std::vector<float>& w, std::vector<float>& hi, std::vector<float>& lo)
{
    hi.resize(w.size());
    lo.resize(w.size());
    for (std::size_t i = 0; i < w.size(); ++i)
    {
        hi[i] = tf32_round(w[i]);
        lo[i] = tf32_round(w[i] - hi[i]);
    }
}
} // namespace tsacb
