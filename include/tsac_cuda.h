/*
 * tsac_cuda.h — C ABI of the B200-native TSAC inference hot path.
 *
 * This is the drop-in boundary for skimmilk/tsac-metal's analyzer plug-in
 * point.  The reference has no FFI of its own (it is C++ end to end); the
 * entry points below are the ones its `AudioAnalyzer` seam would bind
 * (include/tsac/audio_analyzer.hpp:30-37) plus the per-stage and per-kernel
 * calls a backend implements behind it.  Each declaration names the
 * reference interface it replaces (path:line within the reference project).
 *
 * Conventions
 *  - Every function returns 0 (TSAC_CUDA_OK) or a nonzero status; the
 *    message of the last failure on the calling thread is returned by
 *    tsac_cuda_last_error().  A C++ caller maps nonzero codes to tsac::Error
 *    (include/tsac/types.hpp:15-18).
 *  - Plain pointers and sizes only.  Pointers documented as "device" are
 *    CUDA device addresses; "host" are ordinary CPU memory.  `stream` is a
 *    cudaStream_t passed as void* (NULL = legacy default stream).
 *  - Context calls are synchronous: GPU work is complete on return, matching
 *    the AudioAnalyzer contract (include/tsac/audio_analyzer.hpp:24-29).
 *    Kernel-level calls only enqueue on `stream`.
 *  - bf16 values are uint16_t bit patterns.  No entry point falls back to the
 *    CPU: without a usable CUDA device they fail with TSAC_CUDA_ERROR_DEVICE.
 */
#ifndef TSAC_CUDA_H
#define TSAC_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum tsac_cuda_status_code
{
    TSAC_CUDA_OK = 0,
    TSAC_CUDA_ERROR = 1,        /* validation / format error (tsac::Error) */
    TSAC_CUDA_ERROR_DEVICE = 2, /* CUDA runtime error or no device */
    TSAC_CUDA_ERROR_NUMERIC = 3 /* device error word: nonfinite value */
};

/* Message of the last failure on this thread ("" if none). */
const char* tsac_cuda_last_error(void);
/* Releases any buffer returned through an out-pointer by this library. */
void tsac_cuda_free(void* pointer);

/* ---- model package tooling (host only, no GPU needed) ------------------ */

/* Writes seeded random-init originals dac_{mono,stereo}_q8.bin and
 * tsac_{mono,stereo}_q8.bin (libnc container, the input format the
 * reference packer parses: src/weights/source_model.cpp:104-178). */
int tsac_cuda_write_seeded_sources(const char* directory, uint64_t seed);

/* Packs four originals into the 20-file `.weights` package plus
 * adapter_offsets.hpp; byte-identical to the reference packer
 * `tsac-pack-models INPUT OUTPUT ID TRANSFORMER` (src/weights/pack_main.cpp:733-787). */
int tsac_cuda_pack_models(const char* input_directory, const char* output_directory,
                          const char* pack_id, int include_transformer);

/* ---- analyzer context (one per AudioAnalyzer instance and device) ------ */

typedef struct tsac_cuda_context tsac_cuda_context;

/* EncodeOptions (include/tsac/audio_analyzer.hpp:16-22). */
typedef struct tsac_cuda_encode_options
{
    int method;             /* 0 = fast (10-bit fields), 1 = normal (Transformer + range coder) */
    unsigned codebooks;     /* 0 = model maximum (12 joint stereo, 9 otherwise) */
    int separate_channels;  /* nonzero: code a stereo input as two mono groups */
    int entropy_batch;      /* 0 = automatic (select_entropy_batch), else 1..65535 */
} tsac_cuda_encode_options;

/* Binds a model package directory (the reference's ModelDirectory: 20
 * `.weights` files + adapter_offsets.hpp, include/tsac/model_directory.hpp:15-25)
 * to CUDA device `device`.  Prepared device weights are created on first use
 * and kept for later calls.  A context is used by one thread at a time;
 * separate contexts are independent (AUDIO_API.md:81-118). */
int tsac_cuda_context_create(const char* package_directory, int device, tsac_cuda_context** out);
void tsac_cuda_context_destroy(tsac_cuda_context* context);

/* Policy limits (tsac::Limits, include/tsac/types.hpp:20-31), checked
 * before any allocation exactly where the reference checks them: input and
 * padded PCM elements, symbols, decoded PCM bytes and elements, stream size.
 * A new context uses the reference's defaults. */
typedef struct tsac_cuda_limits
{
    size_t file_bytes, symbols, pcm_bytes, cache_bytes, tensor_elements, tensors, metadata_bytes,
        name_bytes;
} tsac_cuda_limits;
int tsac_cuda_set_limits(tsac_cuda_context* context, const tsac_cuda_limits* limits);

/* Decoder synthesis arithmetic of a context.  0 (the default): the wide DAC
 * decoder convolutions run on the tensor cores in 3xTF32 (decoded PCM within
 * 1e-4 * (1 + max(|a|, |b|)) of the reference, the reference's own pipeline
 * tolerance, tests/metal_optimized.cpp:741-745).  Nonzero: the reference's
 * serial fp32 order on CUDA cores (decoded PCM bit-identical).  Streams are
 * unaffected either way. */
int tsac_cuda_set_exact_synthesis(tsac_cuda_context* context, int exact);

/* Certified fast analysis (the encoder's DAC analysis; streams stay
 * byte-identical to the reference's).  margin 0 (the default): the exact
 * analysis, the reference's serial arithmetic (analysis.tpp:169-214 with
 * scalar::Conv1d, src/scalar/dsp.cpp:11-51).  margin > 0: the analysis
 * convolutions use fused multiply-adds (one rounding per term), every RVQ
 * decision reports by how much the winning similarity leads the runner-up
 * (similarities lie in [-1, 1]), and every frame with a decision whose lead
 * is below `margin` is recomputed exactly on the 17-frame sub-window its
 * latent depends on, so its tokens are the reference's; the margin must
 * exceed the fast path's largest similarity error (see DESIGN).  Also makes
 * tsac_cuda_dac_analysis return the fast latents.  margin in [0, 2]. */
int tsac_cuda_set_fast_analysis(tsac_cuda_context* context, float margin);
/* Cumulative counts since the context was created: central frames the fast
 * analysis coded, frames it flagged as uncertain, and frames the exact
 * recomputation evaluated (sub-windows included). */
int tsac_cuda_fast_analysis_stats(tsac_cuda_context* context, uint64_t* frames, uint64_t* uncertain,
                                  uint64_t* recomputed_frames);

/* Host worker budget of a context (the reference CLI's -T, src/cli.cpp:66-68,
 * passed to AppleArmAnalyzer, src/codec.cpp:117-120, which accepts 1-256,
 * src/apple-arm/audio_analyzer.cpp:93): range encoding of a batch's
 * recordings uses at most `threads` host threads (decoding runs its range
 * decoders on the GPU).  0 (the default): all hardware threads.  More than
 * 256 is TSAC_CUDA_ERROR. */
int tsac_cuda_set_host_threads(tsac_cuda_context* context, unsigned threads);

/* AudioAnalyzer::encode (include/tsac/audio_analyzer.hpp:33-34) for a host
 * PCM view [channel, sample] with the given strides (in floats, as
 * tsac::PcmView's layout_stride).  *out (free with tsac_cuda_free) receives the
 * .tsac stream; *symbol_bits (nullable) the payload bit position before
 * termination (the sum an EntropyObserver's after_symbol would report). */
int tsac_cuda_encode(tsac_cuda_context* context, const float* pcm, size_t channels,
                     size_t samples, ptrdiff_t channel_stride, ptrdiff_t sample_stride,
                     const tsac_cuda_encode_options* options, uint8_t** out, size_t* out_bytes,
                     size_t* symbol_bits);

/* tsac_cuda_encode plus the per-codebook totals an EntropyObserver would
 * accumulate from after_symbol (include/tsac/observer.hpp:12-16; the bits of a
 * symbol are the range encoder's bit-position difference,
 * src/format/entropy.cpp:93-98): codebook_bits[b] for b < codebooks (entries
 * past the stream's codebook count are 0; all 0 for fast streams). */
int tsac_cuda_encode_observed(tsac_cuda_context* context, const float* pcm, size_t channels,
                              size_t samples, ptrdiff_t channel_stride, ptrdiff_t sample_stride,
                              const tsac_cuda_encode_options* options, uint8_t** out,
                              size_t* out_bytes, uint64_t* codebook_bits, size_t codebooks);

/* tsac_cuda_encode plus every symbol's bits in entropy order
 * (visit_entropy_positions, src/format/entropy.cpp:26-55): the value an
 * EntropyObserver's after_symbol receives for it while encoding
 * (src/format/entropy.cpp:93-98).  *symbol_bits (free with tsac_cuda_free)
 * holds *symbols values, the stream's symbol count; fast streams have none
 * (NULL, 0: fast coding emits no entropy callbacks). */
int tsac_cuda_encode_symbol_bits(tsac_cuda_context* context, const float* pcm, size_t channels,
                                 size_t samples, ptrdiff_t channel_stride, ptrdiff_t sample_stride,
                                 const tsac_cuda_encode_options* options, uint8_t** out,
                                 size_t* out_bytes, uint32_t** symbol_bits, size_t* symbols);

/* AudioAnalyzer::decode (include/tsac/audio_analyzer.hpp:35): stream ->
 * interleaved float PCM [sample][channel], padding retained. */
int tsac_cuda_decode(tsac_cuda_context* context, const uint8_t* stream, size_t bytes,
                     float** out, size_t* samples, unsigned* channels);

/* Batched forms: `count` independent interleaved recordings per call (the
 * throughput path: all recordings share each GPU launch). */
int tsac_cuda_encode_batch(tsac_cuda_context* context, size_t count, const float* const* pcm,
                           const size_t* channels, const size_t* samples,
                           const tsac_cuda_encode_options* options, uint8_t** out,
                           size_t* out_bytes);
int tsac_cuda_decode_batch(tsac_cuda_context* context, size_t count,
                           const uint8_t* const* streams, const size_t* bytes, float** out,
                           size_t* samples, unsigned* channels);

/* HBM-resident forms of the batched calls: PCM inputs are device pointers
 * (interleaved [sample][channel] floats); decoded PCM is written to
 * caller-allocated device buffers of channels x samples_per_channel floats
 * (sizes from tsac_cuda_stream_info).  Streams stay host byte buffers. */
int tsac_cuda_encode_batch_device(tsac_cuda_context* context, size_t count,
                                  const float* const* pcm_device, const size_t* channels,
                                  const size_t* samples, const tsac_cuda_encode_options* options,
                                  uint8_t** out, size_t* out_bytes);
int tsac_cuda_decode_batch_device(tsac_cuda_context* context, size_t count,
                                  const uint8_t* const* streams, const size_t* bytes,
                                  float* const* pcm_device);

/* parse_header (src/format/container.cpp:43-80): channels, padded samples per
 * channel and symbol count of a stream, without decoding it. */
int tsac_cuda_stream_info(const uint8_t* stream, size_t bytes, unsigned* channels,
                          size_t* samples_per_channel, size_t* symbols);

/* Header fields of a .tsac stream (parse_header, src/format/container.cpp:43-80). */
typedef struct tsac_cuda_stream_header
{
    unsigned method;         /* 0 fast, 1 normal */
    unsigned model_channels; /* 1 or 2 */
    unsigned groups;         /* channel groups (separate channels / mono layouts) */
    unsigned codebooks;
    uint64_t frames;         /* 512-sample frames */
    unsigned batch;          /* entropy batch (lanes) */
} tsac_cuda_stream_header;
int tsac_cuda_stream_header_info(const uint8_t* stream, size_t bytes, tsac_cuda_stream_header* out);

/* unpack_fast (src/format/container.hpp:28, src/format/container.cpp): the
 * 10-bit token fields of a fast-method stream, after the header and CRC
 * checks.  Host-only; *tokens is malloc'd, release with tsac_cuda_free. */
int tsac_cuda_unpack_fast(const uint8_t* stream, size_t bytes, uint16_t** tokens, size_t* count);

/* token_crc32 (src/format/container.hpp:32): the CRC-32 (polynomial
 * 0x04c11db7) that a normal stream's header carries over its token indices. */
uint32_t tsac_cuda_token_crc32(const uint16_t* tokens, size_t count);

/* ---- pipeline stages (host buffers; synchronous) ----------------------- */

/* Encoder front end: padding, 400-frame chunks with 8/9 context, DAC analysis
 * and RVQ (detail::analyze_audio, src/common/audio_pipeline.hpp:36-61) ->
 * tokens [frame][group][book]. */
int tsac_cuda_analyze_tokens(tsac_cuda_context* context, const float* interleaved_pcm,
                             size_t channels, size_t samples,
                             const tsac_cuda_encode_options* options, uint16_t** tokens,
                             size_t* count);

/* DacAnalysis::apply (src/common/analysis.tpp:169-214) of one window:
 * pcm [pcm_frames][channels] (pcm_frames a multiple of 512) -> latent [pcm_frames/512][1024]. */
int tsac_cuda_dac_analysis(tsac_cuda_context* context, unsigned channels, const float* pcm,
                           size_t pcm_frames, float* latent);

/* DacSynthesis::apply (src/common/synthesis.tpp:168-213) of one window:
 * latent [frames][1024] -> pcm [frames*512][channels]. */
int tsac_cuda_dac_synthesis(tsac_cuda_context* context, unsigned channels, const float* latent,
                            size_t frames, float* pcm);

/* RvqEncoder::encode (src/common/rvq.tpp:59-95) of one group: latent
 * [frames][1024] -> tokens [frames][books]; RvqDecoder::decode
 * (src/common/rvq.cpp:76-120) the inverse reconstruction. */
int tsac_cuda_rvq_encode(tsac_cuda_context* context, unsigned channels, unsigned books,
                         const float* latent, size_t frames, uint16_t* tokens);
int tsac_cuda_rvq_decode(tsac_cuda_context* context, unsigned channels, unsigned books,
                         const uint16_t* tokens, size_t frames, float* latent);

/* TokenPredictor over known tokens (TransformerPredictor + CpuTransformer,
 * src/common/transformer.cpp:59-166, src/common/cpu_transformer.tpp:317-385):
 * for tokens [frame][group][book], writes per symbol (token-offset order) the
 * float probabilities [1024] (nullable) and the Q15 zero-probabilities of the
 * 10 bisection nodes on the path to the symbol's token (nullable,
 * encode_categorical, src/format/categorical.cpp:91-117). */
int tsac_cuda_transformer_probabilities(tsac_cuda_context* context, unsigned channels,
                                        unsigned groups, unsigned books, size_t frames,
                                        unsigned batch, const uint16_t* tokens,
                                        float* probabilities, uint16_t* q15);

/* pack_normal (src/format/entropy.cpp:57-123) for known tokens [frame][group][book]
 * with the GPU predictor and the host range coder: the normal-mode stream. */
int tsac_cuda_pack_normal(tsac_cuda_context* context, unsigned channels, unsigned groups,
                          unsigned books, size_t frames, unsigned batch, const uint16_t* tokens,
                          uint8_t** out, size_t* out_bytes);

/* ---- instrumentation --------------------------------------------------- */

/* Enables (nonzero) or disables per-kernel-family timing: each launch family
 * (conv_exact, conv_transposed, snake, qlinear_gemv, qlinear_gemm, attention,
 * rvq_encode, ...) is bracketed by CUDA events on its stream; resets totals. */
int tsac_cuda_kernel_timing(int enable);
/* JSON {family: {"launches": n, "ms": total, "work": algorithmic FLOPs or bytes}}
 * accumulated since the last tsac_cuda_kernel_timing call (free with tsac_cuda_free). */
int tsac_cuda_kernel_stats(char** json);

/* Kernels this library has launched in this process so far (every device and
 * thread; a decode-step graph launch adds its kernel nodes). */
uint64_t tsac_cuda_launch_count(void);

/* ---- kernel-level entry points (device pointers, enqueue on `stream`) -- */

/* Scratch bytes tsac_cuda_qlinear needs for m columns of k inputs (the BF8L
 * quantized activations: int8 [m][k] then f32 scales [m][k/256]). */
size_t tsac_cuda_qlinear_scratch_bytes(size_t m, size_t k);

/* Quantized linear projection, y = bf16(W x + bias) [+ residual]:
 * PackedLinear::apply_into (src/common/packed_linear.tpp:85-123) = scalar::bf8l
 * (src/scalar/probability.cpp:16-40) + Kernels::linear_column per column
 * (src/scalar/packed_linear.cpp:8-30).
 *   weights       device int8 [n][k] canonical row-major (the package's
 *                 transformer-source plane; no R4 re-tiling)
 *   weight_scales device f32 [k/256][n];  bias device f32 [n]
 *   x             device bf16 [m][k];     y device bf16 [m][n]
 *   residual      device bf16 [m][n] or NULL: y = bf16(residual + y)
 *                 (probability_add_bf16, src/common/probability.cpp:7-12)
 *   scratch       device, >= tsac_cuda_qlinear_scratch_bytes(m, k)
 *   error_word    device unsigned or NULL; bit 1 set on nonfinite input
 *                 (the reference throws "BF8L activations must be finite").
 * k: multiple of 256 up to 8192; n: multiple of 64; buffers 16-byte aligned. */
int tsac_cuda_qlinear(const int8_t* weights, const float* weight_scales, const float* bias,
                      size_t k, size_t n, const uint16_t* x, size_t m, const uint16_t* residual,
                      uint16_t* y, void* scratch, size_t scratch_bytes, unsigned* error_word,
                      void* stream);

/* tsac_cuda_qlinear for callers that cannot allocate device memory: for
 * example a service that reserves all of its GPU memory at start-up and then
 * forbids cudaMalloc, or a real-time audio thread that must not wait on the
 * driver's allocator.  This entry point has no counterpart in the reference.
 * It allocates nothing: its scratch is a fixed 1 MiB + 16 KiB array in the
 * library's device image, present on every GPU that loads the library until the
 * process exits.  Limit: m * k <= tsac_cuda_qlinear_noalloc_max_elements()
 * (1,048,576, e.g. 256 columns of 4096 inputs); larger calls fail with
 * TSAC_CUDA_ERROR.  The first call on a device looks up the array's device
 * address (cudaGetSymbolAddress) and should come before any stream capture.
 * That address belongs to the device's primary context, so do not use this
 * entry point on a device after cudaDeviceReset in the same process.
 * All calls share the array, so calls that overlap on the GPU race; serialise
 * them.  Other arguments and results are those of tsac_cuda_qlinear. */
size_t tsac_cuda_qlinear_noalloc_max_elements(void);
int tsac_cuda_qlinear_noalloc(const int8_t* weights, const float* weight_scales,
                              const float* bias, size_t k, size_t n, const uint16_t* x, size_t m,
                              const uint16_t* residual, uint16_t* y, unsigned* error_word,
                              void* stream);

/* Measurement helper (no reference counterpart): the FP32 issue rate of the
 * current device for the exact convolution's instruction pair, a separately
 * rounded multiply then an add, as operations (multiplies + adds) per second.
 * Runs 16 independent recurrences per thread on 8 x 256-thread CTAs per SM
 * for `iterations` steps, timed with CUDA events on `stream` after one
 * warm-up launch; *milliseconds (nullable) receives the timed launch's
 * duration.  Allocates a small sink buffer.  Synchronous. */
int tsac_cuda_fp32_issue_rate(int iterations, double* ops_per_second, double* milliseconds, void* stream);

/* Causal attention of the probability model, 4 heads x 128 over bf16 keys
 * and values: scalar::Attention / attention_bf16_into
 * (src/scalar/attention.cpp:12-131), per head 64-key blocks merged in order,
 * value sums bf16-rounded when `round` is set (the reference's
 * `time > 64 || prefill`, :128).
 *   query      device bf16 [rows][512]
 *   rows_meta  device int32 [rows][5]: (slot, base, time, rotary, round);
 *              row r attends to keys/values [base, base + time) (slot and
 *              rotary are unused here)
 *   keys, values device bf16 [positions][512]; out device bf16 [rows][512]
 *   max_time   >= every row's time (at most 4,194,240)
 *   scratch    device, >= tsac_cuda_attention_scratch_bytes(rows, max_time)
 *              (may be NULL when max_time <= 64)
 * Asynchronous on `stream`. */
size_t tsac_cuda_attention_scratch_bytes(size_t rows, size_t max_time);
int tsac_cuda_attention(const uint16_t* query, const int* rows_meta, const uint16_t* keys,
                        const uint16_t* values, size_t rows, size_t max_time, uint16_t* out,
                        void* scratch, size_t scratch_bytes, void* stream);

/* Scratch bytes tsac_cuda_conv1d needs (its per-launch tile table). */
size_t tsac_cuda_conv1d_scratch_bytes(size_t out_frames, int stride, int transposed);

/* One exact-order convolution: scalar::Conv1d::sample (src/scalar/dsp.cpp:11-35)
 * for every output, with the geometry of src/common/dsp.tpp:141-178.
 *   x        device f32 [frames][cin]
 *   weights  device f32 [kernel][cin][cout] (tap, input, output; the
 *            reference stores [cout][kernel][cin] ordinary, [cin][kernel][cout]
 *            transposed — the same values re-laid)
 *   bias     device f32 [cout]; residual device f32 [out_frames][cout] or NULL
 *            (y = residual + conv, the residual-unit add of src/common/analysis.tpp:59-66)
 *   y        device f32 [out_frames][cout]
 * Transposed convolutions require dilation 1.  Synchronous on `stream`. */
int tsac_cuda_conv1d(const float* x, size_t frames, const float* weights, const float* bias,
                     const float* residual, float* y, size_t cin, size_t cout, size_t kernel,
                     size_t stride, size_t padding, size_t dilation, int transposed,
                     void* scratch, size_t scratch_bytes, unsigned* error_word, void* stream);

/* The decoder's tensor-core convolution (3xTF32 tcgen05 implicit GEMM, the
 * kernel DAC synthesis runs) on one sequence, for accuracy tests and
 * microbenchmarks; arguments as tsac_cuda_conv1d.  Ordinary convolutions need
 * stride 1 and 'same' padding (2 padding = (kernel - 1) dilation); transposed
 * ones kernel 2 stride and padding stride / 2.  cin % 32 == 0; cout a multiple
 * of 128 or 96.  alpha (device f32 [cout]) or NULL: y = Snake(conv).
 * Allocates and frees device memory per call.  Synchronous on `stream`. */
int tsac_cuda_conv1d_tensor(const float* x, size_t frames, const float* weights, const float* bias,
                            const float* residual, const float* alpha, float* y, size_t cin,
                            size_t cout, size_t kernel, size_t stride, size_t padding,
                            size_t dilation, int transposed, unsigned* error_word, void* stream);

/* DAC Snake, y = x + sin^2(alpha x) / (alpha + eps) with the captured
 * polynomial (scalar_snake_frames, src/scalar/dsp.cpp:93-119); x, y device
 * f32 [frames][channels], alpha device f32 [channels]. */
int tsac_cuda_snake(const float* x, size_t channels, size_t frames, const float* alpha, float* y,
                    unsigned* error_word, void* stream);

/* Range decoding of normal-stream symbols on the device, the optional
 * GPU-resident alternative to the host decoders (the reference's Metal
 * range_decode, src/metal/probability/range.metal:12-77: one serialized
 * RangeDecoder per stream, src/format/range.cpp:118-157, walking the
 * bisection heap of decode_categorical, src/format/categorical.cpp:119-142).
 * Payload s of `streams` is bytes[offsets[s], offsets[s] + sizes[s]); bytes,
 * offsets, sizes, cursors (tsac_cuda_range_cursor_bytes() each) are device
 * memory.  tsac_cuda_range_start reads each payload's first three bytes;
 * tsac_cuda_range_decode then decodes `count` symbols: row r belongs to stream
 * rows[r] (device int32), a stream's rows in increasing r, its left-child
 * masses masses[r][1023] (device f32, the softmax tree's heap), symbol to
 * symbols[r] (device u16).  The cursors carry each decoder across calls.  A
 * stream whose code leaves its interval stops (cursor status 1, symbols 0)
 * and ORs 2 (the range-error bit) into *error_word (nullable).  Asynchronous
 * on `stream`. */
size_t tsac_cuda_range_cursor_bytes(void);
int tsac_cuda_range_start(const uint8_t* bytes, const uint64_t* offsets, const uint64_t* sizes,
                          void* cursors, size_t streams, unsigned* error_word, void* stream);
int tsac_cuda_range_decode(const uint8_t* bytes, const uint64_t* offsets, const uint64_t* sizes,
                           void* cursors, size_t streams, const int* rows, size_t count,
                           const float* masses, uint16_t* symbols, unsigned* error_word, void* stream);

/* Host range coding over given bisection masses (host memory, [count][1023]
 * heap order), the coder the decode loop runs: tsac_cuda_range_encode_tree
 * codes count symbols (encode_categorical's 10 decisions each) into *out
 * (free with tsac_cuda_free); tsac_cuda_range_decode_tree decodes them back.
 * Host only; for round-trip tests of either decoder. */
int tsac_cuda_range_encode_tree(const float* masses, const uint16_t* symbols, size_t count,
                                uint8_t** out, size_t* out_bytes);
int tsac_cuda_range_decode_tree(const uint8_t* bytes, size_t size, const float* masses, size_t count,
                                uint16_t* symbols);

#ifdef __cplusplus
}
#endif

#endif /* TSAC_CUDA_H */
