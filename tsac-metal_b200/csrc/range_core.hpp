// Binary range-coder arithmetic and the 1024-symbol bisection walk, shared by
// the host coder (csrc/host/format.cpp) and the device decoder
// (csrc/kernels/range_decode.cu), so that both decode with one definition.
//
// The stream contract these restate (reference project paths):
//   24-bit range, initial range 0xff0000, split = (range * p0) >> 15,
//   renormalise by whole bytes while range < 0xff01     src/format/range.cpp:14-157
//   bisection coding of a 1024-entry alphabet, each
//   node's decision with conditional_q15 of (left mass,
//   path mass), right mass = path mass - left          src/format/categorical.cpp:76-142
//
// Because the alphabet is a power of two, every bisection node splits its
// range in half exactly, so the walk is a loop over the 10 bits of the symbol,
// most significant first; the heap of left-child masses (node i's children at
// 2i+1 and 2i+2) is indexed by the path taken so far.
#pragma once
#include <cstdint>

#if defined(__CUDACC__)
#define TSACB_RANGE_FN __host__ __device__ __forceinline__
#else
#define TSACB_RANGE_FN inline
#endif

namespace tsacb::range
{
constexpr std::uint32_t initial_range = 0xff0000u;
constexpr std::uint32_t renormalise_below = 0xff01u;
constexpr unsigned symbol_bits = 10;
constexpr unsigned bisection_nodes = 1023;

// Width of the zero branch of a decision with Q15 zero-probability p0.
TSACB_RANGE_FN std::uint32_t zero_width(std::uint32_t range, std::uint32_t p0)
{
    return static_cast<std::uint32_t>((static_cast<std::uint64_t>(range) * p0) >> 15);
}

// A decoder's interval: the code's offset inside the current range.
struct DecodeWindow
{
    std::uint32_t range = initial_range;
    std::uint32_t code = 0;
};

// One binary decision.  source.next_byte() yields the following payload byte
// (0 once the payload is exhausted).  Returns the bit, or -1 when the code has
// left its interval (a corrupt payload); the window is then no longer
// meaningful.
template <class Source>
TSACB_RANGE_FN int decide(DecodeWindow& w, std::uint32_t p0, Source& source)
{
    const std::uint32_t zero = zero_width(w.range, p0);
    const int bit = w.code >= zero;
    if (bit)
    {
        w.code -= zero;
        w.range -= zero;
    }
    else
    {
        w.range = zero;
    }
    // range >= 1 after any split, so at most three byte shifts restore it.
    while (w.range < renormalise_below)
    {
        w.range <<= 8;
        w.code = (w.code << 8) | source.next_byte();
    }
    return w.code < w.range ? bit : -1;
}

// Walks the bisection heap of one symbol.  `Math` supplies q15(left, mass)
// (conditional_q15) and sub(a, b) (the flushed subtraction of the right
// mass) in the caller's arithmetic; step.node(p0, bit_index) makes the
// decision of the node (decoding: returns the decoded bit or -1; encoding:
// codes the known bit and returns it).  Returns the symbol, or -1 if a step
// failed.
template <class Math, class Step>
TSACB_RANGE_FN int walk_bisection(const float* left_masses, Step& step)
{
    unsigned node = 0, symbol = 0;
    float mass = 1.0f;
#if defined(__CUDA_ARCH__)
#pragma unroll 1
#endif
    for (int bit_index = symbol_bits - 1; bit_index >= 0; --bit_index)
    {
        const float left = left_masses[node];
        const int bit = step.node(Math::q15(left, mass), bit_index);
        if (bit < 0)
        {
            return -1;
        }
        symbol |= static_cast<unsigned>(bit) << bit_index;
        mass = bit ? Math::sub(mass, left) : left;
        node = 2 * node + 1 + static_cast<unsigned>(bit);
    }
    return static_cast<int>(symbol);
}
} // namespace tsacb::range
