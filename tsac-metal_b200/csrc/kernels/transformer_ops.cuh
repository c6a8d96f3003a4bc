// Launch interface of the Transformer's row-wise kernels (everything except
// the quantized linear layers, which live in qlinear.cuh).
//
// Rows: the unit of batching.  A row is one (lane, position) of the temporal
// stack or one (frame, book) of the codebook stack; all rows of a launch are
// independent except through the K/V cache, which attention reads by slot.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

#include "kernels/row_meta.hpp"

namespace tsacb::dev
{
// out[r][0:1024] = sum over j < count[r] of E[j][tokens[offset[r] + j]] with
// bf16 adds in book order (first term copied); count 0 gives zeros.  With yq
// non-null the rows are also BF8L-quantized into yq [rows][1024] and
// yscale [rows][4] (qlinear_quantize's result, nonfinite values flagged in
// error_word).
void embed_sum(const std::uint16_t* embeddings, const std::uint16_t* tokens, const int* offsets,
               const int* counts, int rows, std::uint16_t* out, cudaStream_t stream,
               std::int8_t* yq = nullptr, float* yscale = nullptr, unsigned* error_word = nullptr);

// LayerNorm(512) per row; writes bf16 output and/or BF8L-quantized output.
void layer_norm(const std::uint16_t* x, const std::uint16_t* gain, const std::uint16_t* bias,
                int rows, std::uint16_t* y, std::int8_t* yq, float* yscale, unsigned* error_word,
                cudaStream_t stream);

// qkv [rows][1536] -> query [rows][512] and cache K/V [slot][512], with
// rotary on query and key when meta.rotary >= 0 (coefficients [1024][128]).
void rotary_scatter(const std::uint16_t* qkv, const RowMeta* meta, const std::uint16_t* rotations,
                    int rows, std::uint16_t* query, std::uint16_t* cache_k, std::uint16_t* cache_v,
                    cudaStream_t stream);

// Causal attention over the cache, 4 heads x 128, 64-key blocks merged in order.
// `partials` scratch: rows * 4 heads * 16 blocks * 130 floats.  With yq
// non-null and every history within one 64-key block (max_time <= 64), the
// output goes BF8L-quantized to yq [rows][512] and yscale [rows][2] instead
// of bf16 to `out` (qlinear_quantize's result; nonfinite values flagged in
// error_word), and the call returns true; otherwise it writes `out` and
// returns false.  sequence_rows: rows come in runs of consecutive positions
// of one sequence (a causal prefill, a context replay), so several rows can
// share each staged key block.
bool attention(const std::uint16_t* query, const RowMeta* meta, const std::uint16_t* cache_k,
               const std::uint16_t* cache_v, int rows, int max_time, float* partials,
               std::uint16_t* out, cudaStream_t stream, std::int8_t* yq = nullptr,
               float* yscale = nullptr, unsigned* error_word = nullptr, bool sequence_rows = false);
size_t attention_partials_bytes(int rows, int max_time);

// out[r] = bf16(src[source_row[r]] + positions[book[r]]) (512 wide).
void add_positions(const std::uint16_t* src, const int* source_row, const int* book,
                   const std::uint16_t* positions, int rows, std::uint16_t* out,
                   cudaStream_t stream);

// Softmax(1024) per row.  Writes any of: bf16 probabilities, float
// probabilities, and the 1023-node subtree mass tree (node i of a heap:
// children 2i+1, 2i+2; node value = FTZ pair sum of its range).
void softmax_tree(const std::uint16_t* logits, int rows, std::uint16_t* probs_bf16,
                  float* probs_f32, float* tree, unsigned* error_word, cudaStream_t stream);

// For known tokens: the Q15 zero-probability of the 10 bisection nodes on the
// path to token[r] (conditional_q15 with the reference's mass recurrence).
void categorical_path_q15(const float* tree, const std::uint16_t* token, const int* token_index,
                          int rows, std::uint16_t* q15, cudaStream_t stream);

// dst row dst_index[j] = src row src_index[j], j < rows (512-wide bf16 rows).
void scatter_rows(const std::uint16_t* src, const int* src_index, const int* dst_index, int rows,
                  std::uint16_t* dst, cudaStream_t stream);

// 65536-entry bf16 GELU table computed on the device.
void build_gelu_table(std::uint16_t* table, cudaStream_t stream);
} // namespace tsacb::dev
