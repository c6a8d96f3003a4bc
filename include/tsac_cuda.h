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

#ifdef __cplusplus
}
#endif

#endif /* TSAC_CUDA_H */
