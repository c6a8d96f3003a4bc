// 1 / (alpha + eps) per channel: the Snake divisor of the tensor-core
// synthesis epilogue as a reciprocal (eps 0x3089705f, the reference's Snake
// epsilon, src/weights/normalization.hpp:9).
#pragma once
#include <cstdint>
#include <cstring>
#include <vector>

namespace tsacb
{
inline std::vector<float> snake_inverse(const std::vector<float>& alpha)
{
    float eps;
    const std::uint32_t bits = 0x3089705fu;
    std::memcpy(&eps, &bits, sizeof(eps));
    std::vector<float> inverse(alpha.size());
    for (std::size_t i = 0; i < alpha.size(); ++i)
        inverse[i] = 1.0f / (alpha[i] + eps);
    return inverse;
}
} // namespace tsacb
