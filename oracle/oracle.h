/*
 * CPU restatement of the TSAC hot-path arithmetic — TEST INFRASTRUCTURE ONLY.
 *
 * This is the checker the CUDA kernels are compared against.  Only tests/,
 * __graft_entry__.smoke() and bench.py's CPU-baseline leg may load it; the
 * product path never calls it.  Each function cites the reference file:line
 * whose arithmetic it restates.  It is pinned (tests/test_oracle.py) against
 * the reference's own known-answer tests (the attention checksum
 * 15737425383056432415 of tests/attention.cpp:103, the exhaustive BF16 rule of
 * tests/numeric.cpp:60-76, the BF8L and convolution KATs of tests/scalar.cpp)
 * and against the reference scalar path itself built under oracle/_ref.
 */
#ifndef TSAC_ORACLE_H
#define TSAC_ORACLE_H
#include <stddef.h>
#include <stdint.h>

uint16_t oracle_bf16(float x);
float oracle_float(uint16_t x);
float oracle_flush(float x);
float oracle_exp(float z);
float oracle_probability_sum(const float* x, size_t n);
void oracle_bisection_masses(const float* p, size_t rows, float* out);
uint16_t oracle_conditional_q15(float left, float mass);

void oracle_bf8l(const float* x, size_t n, int8_t* q, uint16_t* scales);
/* weights canonical int8 [n][k]; x bf16 [m][k]; y bf16 [m][n]. */
void oracle_linear(const int8_t* w, const float* w_scales, const float* bias, size_t k, size_t n,
                   const uint16_t* x, size_t m, uint16_t* y);
void oracle_layer_norm(const uint16_t* x, const uint16_t* gain, const uint16_t* bias, size_t n,
                       uint16_t* y);
void oracle_rotary(const uint16_t* x, const uint16_t* coefficients, size_t n, uint16_t* y);
uint16_t oracle_gelu(uint16_t x);
void oracle_softmax(const uint16_t* x, size_t n, uint16_t* y);
/* keys/values row-major [time][heads*head_width] bf16. */
void oracle_attention(const uint16_t* q, const uint16_t* keys, const uint16_t* values,
                      size_t heads, size_t head_width, size_t time, int prefill, uint16_t* y);

/* ordinary: w [out][k][in]; transposed: w [in][k][out]; x [frames][in]. */
size_t oracle_conv1d(size_t in, size_t out, size_t k, size_t stride, size_t padding,
                     size_t dilation, int transposed, const float* w, const float* bias,
                     const float* x, size_t frames, float* y);
void oracle_snake(const float* x, size_t channels, size_t frames, const float* alpha, float* y);
uint16_t oracle_rvq_nearest(const float* projected8, const float* search);
size_t oracle_categorical_path(const float* p, size_t n, size_t symbol, uint16_t* q15,
                               uint8_t* bits);
void oracle_rvq_project(uint16_t index, const float* codebook, const float* weights,
                        const float* bias, float* out);
#endif
