// GPU TokenPredictor: the two-stack probability model on the device.
//
// Replaces CpuTransformer + TransformerPredictor (src/common/cpu_transformer.tpp,
// src/common/transformer.cpp) behind the TokenPredictor seam
// (src/format/entropy.hpp:12-26).  Work is organised in rows (see
// kernels/transformer_ops.cuh); a row's K/V lives in a cache slot and its
// attention reads the slots of its own sequence.
//
// Encode (known tokens): the whole recording is evaluated as one layer-wise
// causal prefill per lane, exactly reproducing the per-step schedule of
// TransformerPredictor::prepare (1024-position context, reset and replay of
// the last 256 frames with replay rounding), and emits for every symbol the
// Q15 probabilities of the bisection nodes on the path to its token.
//
// Decode: one (step, book) at a time for all lanes of all recordings in the
// batch, entirely on the device: each step's rows are set up from a device
// step clock, the model emits each row's bisection masses, and the device
// range decoders write the symbols into the batch token array that the next
// step's embeddings read.  Each step shape is a CUDA graph captured once, so
// the host only enqueues graph launches and synchronises once per batch.
#pragma once
#include "device.hpp"
#include "kernels/row_meta.hpp"
#include "format.hpp"
#include "models.hpp"

#include <map>
#include <memory>
#include <tuple>

namespace tsacb
{
struct DeviceLinear
{
    DeviceBuffer weights, scales, bias;
    int input = 0, output = 0;
};

struct DeviceTransformer
{
    unsigned channels = 0, books = 0;
    std::vector<DeviceLinear> projections; // 63, contract order
    std::vector<DeviceBuffer> norm_gain, norm_bias; // 32
    DeviceBuffer positions, rotations, embeddings, gelu;

    DeviceTransformer(const PreparedTransformer& t, cudaStream_t stream);
};

class TransformerEngine
{
public:
    TransformerEngine(std::shared_ptr<const DeviceTransformer> model, cudaStream_t stream);
    ~TransformerEngine();

    // Known-token evaluation of whole recordings (encode).
    // tokens: [frames][groups][books] of each recording; outputs per recording
    // q15[symbol][10] indexed by token offset, and optionally the float
    // probabilities [symbol][1024] (token-offset order).
    void predict_known(const Header& header, std::span<const std::uint16_t> tokens,
                       std::uint16_t* q15, float* probabilities);

    // --- decode: the whole token loop of a batch of normal streams on the GPU
    // payloads[r]: recording r's range-coded payload (headers[r].payload_bytes);
    // tokens[r] receives its tokens [frame][group][book].  Runs every (step,
    // book) of every lane as device work (the probability model, the bisection
    // masses and the range decoders), with one host synchronisation at the end.
    void decode_streams(const std::vector<Header>& headers, const std::vector<ByteView>& payloads,
                        std::vector<std::vector<std::uint16_t>>& tokens);

    unsigned* error_word() const
    {
        return error_.as<unsigned>();
    }
    void check_errors();

private:
    // residual_stride: elements per residual row (-1: the output width; 0: one
    // residual row added to every row).
    void run_linear(int projection, const std::int8_t* xq, const float* xs, int rows,
                    std::uint16_t* y, const std::uint16_t* residual, bool gelu,
                    int residual_stride = -1);
    // bf16 input: BF8L pass into xq / xs (scratch of rows x K), then the linear.
    void run_linear_bf16(int projection, const std::uint16_t* x, int rows, std::uint16_t* y,
                         const std::uint16_t* residual, bool gelu, std::int8_t* xq, float* xs);
    // QKV projection + rotary + K/V cache scatter (fused where it fits; else
    // through `qkv` scratch [rows][1536] and the rotary kernel).
    void run_qkv(int projection, const std::int8_t* xq, const float* xs, int rows,
                 const dev::RowMeta* meta, std::uint16_t* query, std::uint16_t* cache_k,
                 std::uint16_t* cache_v, std::uint16_t* qkv);
    void quantize(const std::uint16_t* x, int rows, int k, std::int8_t* xq, float* xs);
    // One (step, book) of the decode loop for the rows of one shape.
    void enqueue_decode_step(const int* row_lane, const int* row_begin, int rows, int book, int per_lane);
    void run_stack(Workspace& ws, bool temporal, int rows, std::uint16_t* h,
                   const void* meta_device, int max_time, std::uint16_t* cache_k,
                   std::uint16_t* cache_v, std::size_t cache_layer_stride,
                   std::uint16_t* final_out, std::int8_t* final_q, float* final_s,
                   bool sequence_rows = false);

    std::shared_ptr<const DeviceTransformer> model_;
    cudaStream_t stream_;
    Workspace ws_;
    DeviceBuffer error_;

    struct DecodeState;
    std::unique_ptr<DecodeState> decode_;
};
} // namespace tsacb
