/*
 * CPU restatement of the TSAC hot-path arithmetic (see oracle.h) —
 * TEST INFRASTRUCTURE ONLY, never the product.
 *
 * Compiled with -ffp-contract=off: every `a * b + c` rounds twice, and fma()
 * is the C99 correctly rounded fused multiply-add.  `volatile` temporaries pin
 * the rounding boundaries exactly as the reference writes them.
 */
#include "oracle.h"

#include <math.h>
#include <string.h>

uint16_t oracle_bf16(float x) /* src/common/numeric/bf16.hpp:9-13 */
{
    uint32_t b;
    memcpy(&b, &x, 4);
    return (uint16_t)((b + 0x7fffu + ((b >> 16) & 1u)) >> 16);
}

float oracle_float(uint16_t x) /* src/common/numeric/bf16.hpp:15-18 */
{
    uint32_t b = (uint32_t)x << 16;
    float f;
    memcpy(&f, &b, 4);
    return f;
}

static uint32_t bits_of(float x)
{
    uint32_t b;
    memcpy(&b, &x, 4);
    return b;
}

static float from_bits(uint32_t b)
{
    float f;
    memcpy(&f, &b, 4);
    return f;
}

float oracle_flush(float x) /* src/common/numeric/float_math.hpp:33-37 */
{
    uint32_t b = bits_of(x);
    return (b & 0x7f800000u) == 0 ? from_bits(b & 0x80000000u) : x;
}

static float add_f(float x, float y) /* float_math.hpp:39-43 */
{
    volatile float v = oracle_flush(x) + oracle_flush(y);
    return oracle_flush(v);
}

static float sub_f(float x, float y) /* float_math.hpp:45-49 */
{
    volatile float v = oracle_flush(x) - oracle_flush(y);
    return oracle_flush(v);
}

static float mul_f(float x, float y) /* float_math.hpp:51-55 */
{
    volatile float v = oracle_flush(x) * oracle_flush(y);
    return oracle_flush(v);
}

static float div_f(float x, float y) /* float_math.hpp:57-61 */
{
    volatile float v = oracle_flush(x) / oracle_flush(y);
    return oracle_flush(v);
}

float oracle_exp(float z) /* src/common/numeric/probability.hpp:14-33 */
{
    z = 87.0f < z ? 87.0f : z;
    z = -88.0f > z ? -88.0f : z;
    volatile float exponent = z * 0x1.715476p+0f;
    const float e = exponent;
    const int32_t n = isfinite(e) ? (int32_t)nearbyintf(e) : INT32_MIN;
    z = fmaf((float)n, -0x1.630000p-1f, z);
    z = fmaf((float)n, 0x1.bd0106p-13f, z);
    float p = fmaf(0x1.a01a02p-13f, z, 0x1.6c16c2p-10f);
    p = fmaf(p, z, 0x1.111112p-7f);
    p = fmaf(p, z, 0x1.555556p-5f);
    p = fmaf(p, z, 0x1.555556p-3f);
    volatile float square = z * z;
    p = fmaf(p, z, 0.5f);
    z = fmaf(p, square, z);
    volatile float plus_one = z + 1.0f;
    return from_bits(bits_of(plus_one) + ((uint32_t)n << 23));
}

static float pair_sum(const float* x, size_t count, size_t width) /* categorical.cpp:17-30 */
{
    float v[64];
    for (size_t i = 0; i < 64; ++i)
        v[i] = i < count ? x[i] : 0.0f;
    while (width > 1)
    {
        width /= 2;
        for (size_t i = 0; i < width; ++i)
            v[i] = add_f(v[2 * i], v[2 * i + 1]);
    }
    return v[0];
}

float oracle_probability_sum(const float* x, size_t n) /* categorical.cpp:44-74 */
{
    if (n <= 8)
        return pair_sum(x, n, 8);
    float partial[64] = {0};
    size_t blocks = 0;
    for (size_t offset = 0; offset < n;)
    {
        const size_t count = n - offset < 64 ? n - offset : 64;
        float value = pair_sum(x + offset, count, 64);
        ++blocks;
        const size_t level = (size_t)__builtin_ctzll(blocks);
        for (size_t i = 0; i < level; ++i)
        {
            value = add_f(value, partial[i]);
            partial[i] = 0;
        }
        partial[level] = value;
        offset += count;
    }
    float value = partial[0];
    const size_t width = 64 - (size_t)__builtin_clzll(blocks);
    for (size_t i = 1; i < width; ++i)
        value = add_f(value, partial[i]);
    return value;
}

uint16_t oracle_conditional_q15(float left, float mass) /* categorical.cpp:76-89 */
{
    const float value = div_f(mul_f(left, 32768.0f), mass);
    if (!isfinite(value) || value >= 0x1p63f || value < -0x1p63f)
        return 1;
    const int64_t integer = (int64_t)nearbyintf(value);
    const int32_t low = (int32_t)(uint32_t)integer;
    return (uint16_t)(low < 1 ? 1 : (low > 32767 ? 32767 : low));
}

void oracle_bf8l(const float* x, size_t n, int8_t* q, uint16_t* scales) /* scalar/probability.cpp:16-40 */
{
    for (size_t offset = 0; offset < n; offset += 256)
    {
        float maximum = 0;
        for (size_t i = 0; i < 256; ++i)
        {
            const float a = fabsf(oracle_flush(x[offset + i]));
            maximum = maximum < a ? a : maximum;
        }
        float d = div_f(maximum, 127.0f);
        d = d < 1e-35f ? 1e-35f : d;
        const uint16_t s = oracle_bf16(d);
        scales[offset / 256] = s;
        const float reciprocal = div_f(1.0f, oracle_float(s));
        for (size_t i = 0; i < 256; ++i)
        {
            float r = nearbyintf(mul_f(x[offset + i], reciprocal));
            r = r < -128.0f ? -128.0f : (127.0f < r ? 127.0f : r);
            q[offset + i] = (int8_t)r;
        }
    }
}

void oracle_linear(const int8_t* w, const float* w_scales, const float* bias, size_t k, size_t n,
                   const uint16_t* x, size_t m, uint16_t* y)
{
    /* packed_linear.tpp:85-123 + scalar/packed_linear.cpp:8-30 (R4 tiling is
     * layout-only, so the canonical [n][k] order is read directly). */
    float xf[8192];
    int8_t xq[8192];
    uint16_t xs[32];
    for (size_t c = 0; c < m; ++c)
    {
        for (size_t i = 0; i < k; ++i)
            xf[i] = oracle_float(x[c * k + i]);
        oracle_bf8l(xf, k, xq, xs);
        for (size_t o = 0; o < n; ++o)
        {
            float sum = 0;
            for (size_t b = 0; b < k / 256; ++b)
            {
                int32_t dot = 0;
                for (size_t i = 0; i < 256; ++i)
                    dot += (int32_t)w[o * k + b * 256 + i] * xq[b * 256 + i];
                volatile float scale = w_scales[b * n + o] * oracle_float(xs[b]);
                sum = fmaf((float)dot, scale, sum);
            }
            volatile float out = sum + bias[o];
            y[c * n + o] = oracle_bf16(out);
        }
    }
}

void oracle_layer_norm(const uint16_t* x, const uint16_t* gain, const uint16_t* bias, size_t n,
                       uint16_t* y) /* src/common/probability.cpp:138-169 */
{
    float values[4096], squares[4096];
    for (size_t i = 0; i < n; ++i)
    {
        values[i] = oracle_float(x[i]);
        squares[i] = values[i] * values[i];
    }
    volatile float reciprocal = 1.0f / (float)n;
    volatile float mean = oracle_probability_sum(values, n) * reciprocal;
    float variance = fmaf(oracle_probability_sum(squares, n), reciprocal, 0.0f);
    variance = fmaf(mean, -mean, variance);
    variance += 1e-5f;
    volatile float inverse = 1.0f / sqrtf(variance);
    volatile float offset = -mean * inverse;
    for (size_t i = 0; i < n; ++i)
    {
        const float normalized = fmaf(values[i], inverse, offset);
        y[i] = oracle_bf16(fmaf(normalized, oracle_float(gain[i]), oracle_float(bias[i])));
    }
}

void oracle_rotary(const uint16_t* x, const uint16_t* c, size_t n, uint16_t* y) /* probability.cpp:24-43 */
{
    for (size_t i = 0; i < n; i += 2)
    {
        const float real = oracle_float(x[i]), imaginary = oracle_float(x[i + 1]);
        const float cosine = oracle_float(c[i]), sine = oracle_float(c[i + 1]);
        volatile float imaginary_sine = imaginary * sine;
        volatile float real_sine = real * sine;
        const uint16_t a = oracle_bf16(fmaf(real, cosine, -imaginary_sine));
        const uint16_t b = oracle_bf16(fmaf(imaginary, cosine, real_sine));
        y[i] = a;
        y[i + 1] = b;
    }
}

uint16_t oracle_gelu(uint16_t value) /* src/common/probability.cpp:45-63 */
{
    const float x = oracle_float(value);
    volatile float cubic = 0x1.2444f2p-5f * x;
    float z = fmaf(cubic, x, 0x1.988454p-1f);
    z = z * x;
    volatile float half = x * 0.5f;
    z = z * -2.0f;
    const float exponential = oracle_exp(z);
    volatile float denominator = exponential + 1.0f;
    volatile float sigmoid = 2.0f / denominator;
    volatile float tanh_ = sigmoid - 1.0f;
    volatile float plus = tanh_ + 1.0f;
    volatile float result = half * plus;
    return oracle_bf16(result);
}

void oracle_softmax(const uint16_t* x, size_t n, uint16_t* y) /* probability.cpp:96-122 */
{
    float e[4096] = {0};
    float maximum = -INFINITY;
    for (size_t i = 0; i < n; ++i)
    {
        const float v = oracle_float(x[i]);
        maximum = maximum < v ? v : maximum;
    }
    for (size_t i = 0; i < n; ++i)
    {
        volatile float shifted = oracle_float(x[i]) - maximum;
        e[i] = oracle_exp(shifted);
    }
    const float total = oracle_probability_sum(e, n);
    volatile float reciprocal = 1.0f / total;
    for (size_t i = 0; i < n; ++i)
    {
        volatile float scaled = e[i] * reciprocal;
        y[i] = oracle_bf16(scaled);
    }
}

void oracle_attention(const uint16_t* q, const uint16_t* keys, const uint16_t* values,
                      size_t heads, size_t hw, size_t time, int prefill, uint16_t* y)
{
    /* src/scalar/attention.cpp:12-131 (row-major keys) */
    const size_t width = heads * hw;
    const int round_values = time > 64 || prefill;
    const float scale = 0.0883883461356163f;
    float scores[64], numerator[4096];
    for (size_t head = 0; head < heads; ++head)
    {
        float running = -INFINITY, total = 0;
        for (size_t j = 0; j < hw; ++j)
            numerator[j] = 0;
        for (size_t start = 0; start < time; start += 64)
        {
            const size_t count = time - start < 64 ? time - start : 64;
            float maximum = -INFINITY;
            for (size_t t = 0; t < count; ++t)
            {
                float dot = 0;
                for (size_t j = 0; j < hw; ++j)
                    dot = fmaf(oracle_float(q[head * hw + j]),
                               oracle_float(keys[(start + t) * width + head * hw + j]), dot);
                volatile float s = dot * scale;
                scores[t] = s;
                maximum = maximum < scores[t] ? scores[t] : maximum;
            }
            for (size_t t = 0; t < count; ++t)
            {
                volatile float shifted = scores[t] - maximum;
                scores[t] = oracle_exp(shifted);
            }
            volatile float difference = maximum - running;
            const float factor = oracle_exp(-fabsf(difference));
            const float old_scale = running > maximum ? 1.0f : factor;
            const float new_scale = running > maximum ? factor : 1.0f;
            volatile float old_total = total * old_scale;
            total = fmaf(oracle_probability_sum(scores, count), new_scale, old_total);
            for (size_t j = 0; j < hw; ++j)
            {
                float sum = 0;
                for (size_t t = 0; t < count; ++t)
                    sum = fmaf(oracle_float(values[(start + t) * width + head * hw + j]),
                               scores[t], sum);
                if (round_values)
                    sum = oracle_float(oracle_bf16(sum));
                volatile float old = numerator[j] * old_scale;
                numerator[j] = fmaf(sum, new_scale, old);
            }
            running = running < maximum ? maximum : running;
        }
        volatile float reciprocal = 1.0f / total;
        for (size_t j = 0; j < hw; ++j)
        {
            volatile float out = numerator[j] * reciprocal;
            y[head * hw + j] = oracle_bf16(out);
        }
    }
}

size_t oracle_conv1d(size_t in, size_t out, size_t k, size_t stride, size_t padding,
                     size_t dilation, int transposed, const float* w, const float* bias,
                     const float* x, size_t frames, float* y)
{
    /* scalar/dsp.cpp:11-51 with geometry from src/common/dsp.tpp:141-178 */
    const size_t span = (k - 1) * dilation + 1;
    const size_t out_frames =
        transposed ? (frames - 1) * stride + span - 2 * padding : (frames + 2 * padding - span) / stride + 1;
    for (size_t f = 0; f < out_frames; ++f)
    {
        for (size_t o = 0; o < out; ++o)
        {
            float sum = 0;
            for (size_t tap = 0; tap < k; ++tap)
            {
                size_t source;
                if (!transposed)
                {
                    const size_t position = f * stride + tap * dilation;
                    if (position < padding)
                        continue;
                    source = position - padding;
                }
                else
                {
                    const size_t position = f + padding, offset = tap * dilation;
                    if (position < offset || (position - offset) % stride)
                        continue;
                    source = (position - offset) / stride;
                }
                if (source >= frames)
                    continue;
                for (size_t i = 0; i < in; ++i)
                {
                    const float wv = transposed ? w[o + tap * out + i * out * k] : w[i + tap * in + o * in * k];
                    volatile float product = x[source * in + i] * wv;
                    sum = sum + product;
                }
            }
            y[f * out + o] = sum + bias[o];
        }
    }
    return out_frames;
}

static float sine_squared(float phase) /* scalar/dsp.cpp:55-91 */
{
    const float reduced = phase * from_bits(0x3f22f983);
    const double lower = floor((double)reduced);
    const double fraction = (double)reduced - lower;
    const double nearest =
        lower + ((fraction > 0.5 || (fraction == 0.5 && fmod(lower, 2.0) != 0)) ? 1.0 : 0.0);
    const float quadrant = (float)nearest;
    const int32_t q = nearest >= -2147483648.0 && nearest < 2147483648.0 ? (int32_t)nearest : INT32_MIN;
    float x = fmaf(quadrant, from_bits(0xbfc90000), phase);
    x = fmaf(quadrant, from_bits(0xb9fdaa22), x);
    volatile float x2 = x * x;
    float value;
    if ((q & 1) == 0)
    {
        float p = fmaf(from_bits(0xb94ca1f9), x2, from_bits(0x3c08839e));
        p = fmaf(p, x2, from_bits(0xbe2aaaa3));
        volatile float cube = x * x2;
        value = fmaf(cube, p, x);
    }
    else
    {
        float p = fmaf(from_bits(0x37ccf5ce), x2, from_bits(0xbab6061a));
        p = fmaf(p, x2, from_bits(0x3d2aaaa5));
        p = fmaf(p, x2, from_bits(0xbf000000));
        value = fmaf(p, x2, 1.0f);
    }
    volatile float squared = value * value;
    return squared;
}

void oracle_snake(const float* x, size_t channels, size_t frames, const float* alpha, float* y)
{
    /* scalar/dsp.cpp:93-119; epsilon bits from src/weights/normalization.hpp:9 */
    const float epsilon = from_bits(0x3089705f);
    for (size_t f = 0; f < frames; ++f)
    {
        for (size_t c = 0; c < channels; ++c)
        {
            const size_t i = f * channels + c;
            volatile float phase = alpha[c] * x[i];
            const float s = sine_squared(phase);
            volatile float denominator = alpha[c] + epsilon;
            volatile float ratio = s / denominator;
            y[i] = x[i] + ratio;
        }
    }
}

uint16_t oracle_rvq_nearest(const float* input, const float* vectors) /* rvq.cpp:126-146 */
{
    const float epsilon = from_bits(0x2b8cbccc);
    float squares[8], query[8];
    for (int i = 0; i < 8; ++i)
        squares[i] = input[i] * input[i];
    for (int width = 8; width > 1; width /= 2)
        for (int i = 0; i < width / 2; ++i)
            squares[i] = squares[2 * i] + squares[2 * i + 1];
    volatile float mean = squares[0] * 0.125f;
    volatile float rms = sqrtf(mean + epsilon);
    volatile float inverse_rms = 1.0f / rms;
    volatile float inverse_width = 1.0f / sqrtf(8.0f);
    for (int i = 0; i < 8; ++i)
    {
        volatile float normalized = input[i] * inverse_rms;
        query[i] = normalized * inverse_width;
    }
    float best = -INFINITY;
    uint16_t selected = 0;
    for (int index = 0; index < 1024; ++index)
    {
        float similarity = 0;
        for (int i = 0; i < 8; ++i)
            similarity = fmaf(vectors[index * 8 + i], query[i], similarity);
        if (similarity > best)
        {
            best = similarity;
            selected = (uint16_t)index;
        }
    }
    return selected;
}

void oracle_rvq_project(uint16_t index, const float* codebook, const float* weights,
                        const float* bias, float* out) /* weights/preparation.cpp:95-114 */
{
    for (size_t j = 0; j < 1024; ++j)
    {
        float sum = 0;
        for (size_t i = 0; i < 8; ++i)
            sum = fmaf(weights[j * 8 + i], codebook[(size_t)index * 8 + i], sum);
        out[j] = sum + bias[j];
    }
}

/* Bisection path of encode_categorical (src/format/categorical.cpp:91-117):
 * the Q15 probability of a zero bit and the bit taken at each of the
 * ceil(log2 n) nodes on the way to `symbol`.  Returns the node count. */
size_t oracle_categorical_path(const float* p, size_t n, size_t symbol, uint16_t* q15,
                               uint8_t* bits)
{
    size_t base = 0, count = n, nodes = 0;
    float mass = 1;
    while (count > 1)
    {
        const size_t half = count / 2;
        const float left = oracle_probability_sum(p + base, half);
        const int bit = symbol >= base + half;
        q15[nodes] = oracle_conditional_q15(left, mass);
        bits[nodes] = (uint8_t)bit;
        ++nodes;
        if (bit)
        {
            base += half;
            count -= half;
            mass = sub_f(mass, left);
        }
        else
        {
            count = half;
            mass = left;
        }
    }
    return nodes;
}

/* Left-child masses of the 1023 bisection nodes of each 1024-entry row, heap
 * order (node i's children at 2i+1, 2i+2): node (depth d, index k) covers the
 * aligned range [k*w, (k+1)*w) with w = 1024 >> d, and its left mass is
 * probability_sum over the first half of that range, as encode_categorical
 * sums it (src/format/categorical.cpp:91-117). */
void oracle_bisection_masses(const float* p, size_t rows, float* out)
{
    for (size_t r = 0; r < rows; ++r)
    {
        const float* row = p + r * 1024;
        float* heap = out + r * 1023;
        for (unsigned depth = 0; depth < 10; ++depth)
        {
            const size_t width = (size_t)1024 >> depth;
            for (size_t k = 0; k < ((size_t)1 << depth); ++k)
                heap[((size_t)1 << depth) - 1 + k] = oracle_probability_sum(row + k * width, width / 2);
        }
    }
}
