/*
 * Shared plain-C types of the dranzer-b200 C ABI (dz_host.h, dz_cuda.h).
 * No C++ or CUDA types cross this boundary: plain pointers, sizes and status codes.
 */
#ifndef DZ_TYPES_H
#define DZ_TYPES_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes: 0 or negative. Mapping to the reference's dranzer_status_t
 * (src/include/dranzer.h:30-41): DZ_E_INVALID -> DRANZER_INVALID_ARGUMENT,
 * DZ_E_IO -> DRANZER_IO_ERROR, DZ_E_FORMAT -> DRANZER_FORMAT_ERROR,
 * DZ_E_CHECKSUM -> DRANZER_CHECKSUM_ERROR, DZ_E_NOMEM -> DRANZER_OUT_OF_MEMORY,
 * DZ_E_UNSUPPORTED -> DRANZER_UNSUPPORTED, DZ_E_DEVICE / DZ_E_TIMEOUT ->
 * DRANZER_MODEL_ERROR, DZ_E_NOT_BUNDLE -> DRANZER_FORMAT_ERROR. */
enum {
    DZ_OK = 0,
    DZ_E_INVALID = -1,
    DZ_E_IO = -2,
    DZ_E_FORMAT = -3,
    DZ_E_CHECKSUM = -4,
    DZ_E_NOMEM = -5,
    DZ_E_UNSUPPORTED = -6,
    DZ_E_DEVICE = -7,
    DZ_E_TIMEOUT = -8,
    DZ_E_NOT_BUNDLE = -9
};

/* Quantization granularity, src/include/core/quantize.h:41-56. */
enum { DZ_GRAN_TENSOR = 0, DZ_GRAN_ROW = 1, DZ_GRAN_COLUMN = 2 };

/* Parameter kinds, src/include/core/model_params.h:20-38. */
enum { DZ_KIND_PROJECTION = 0, DZ_KIND_EMBEDDING = 1, DZ_KIND_BIAS = 2, DZ_KIND_NORM = 3 };

/* Model shape: the six bundle header dimensions (src/core/bundle.c:452-458)
 * minus the derived parameter count, plus the v3 architecture flags
 * (src/include/core/model_types.h:26-36). */
typedef struct {
    size_t vocab_size;
    size_t embedding_dim;
    size_t num_heads;
    size_t num_layers;
    size_t max_seq_len;
    uint32_t architecture_flags;
} dz_model_desc_t;

/* One parameter tensor in model_param_tensors() order
 * (src/core/model_params.c:39-103). Either `f32` (bits == 0) or `scales` +
 * `packed` in the reference's storage form: codes biased by qmax, packed
 * least-significant bit first at bit offset i*bits of the row-major k x n
 * tensor (src/core/quantize.c:213-270). */
typedef struct {
    uint32_t kind;
    size_t rows;
    size_t cols;
    int bits;
    int granularity;
    const float *scales;
    size_t scale_count;
    const uint8_t *packed;
    size_t packed_size;
    const float *f32;
} dz_tensor_blob_t;

#ifdef __cplusplus
}
#endif

#endif
