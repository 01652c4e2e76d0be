/*
 * dranzer-b200 host library (plain C): the quantizer, the code-retaining
 * bundle loader/writer and the host-side tables the CUDA path consumes.
 * Compiled into dranzer_b200/libdz_cuda.so beside the CUDA shim; none of these
 * functions touch a GPU.
 */
#ifndef DZ_HOST_H
#define DZ_HOST_H

#include "dz_types.h"

#ifdef __cplusplus
extern "C" {
#endif

/* ---- RNG: src/core/rng.c:18-57 (stream constants src/include/core/rng.h:51-54). */
#define DZ_RNG_STREAM_INIT     UINT64_C(0x9e3779b97f4a7c15)
#define DZ_RNG_STREAM_DROPOUT  UINT64_C(0xbf58476d1ce4e5b9)
#define DZ_RNG_STREAM_SAMPLING UINT64_C(0x94d049bb133111eb)
#define DZ_RNG_STREAM_TESTING  UINT64_C(0x2545f4914f6cdd1d)

uint64_t dz_rng_stream(uint64_t seed, uint64_t stream);   /* replaces dranzer_rng_stream */
uint64_t dz_rng_next(uint64_t *state);                    /* replaces dranzer_rng_next */
double dz_rng_unit(uint64_t *state);                      /* replaces dranzer_rng_unit */

/* Synthetic inputs: N(0, sd) by Box-Muller over two dz_rng_unit() draws
 * (u1 floored at 2^-53); prompt ids by dz_rng_next() % vocab with rejection. */
void dz_synth_gaussian(uint64_t *state, float *out, size_t count, double sd);
void dz_synth_prompt_ids(uint64_t *state, uint32_t *out, size_t count, uint32_t vocab,
                         const uint32_t *excluded, size_t n_excluded);

/* ---- Quantizer. Same contract, arguments and -1 returns as
 * quantized_scale_count / quantized_packed_size / quantize_pack /
 * quantize_unpack (src/include/core/quantize.h:129-140). Codes and scale bit
 * patterns are identical to the reference build's (scale = peak * fl(1/qmax),
 * the reciprocal multiply its -ffast-math build compiles peak/qmax to). */
int dz_quantized_scale_count(size_t rows, size_t cols, int granularity, size_t *out_count);
int dz_quantized_packed_size(size_t value_count, int bits, size_t *out_size);
int dz_quantize_pack(const float *src, size_t rows, size_t cols, int bits, int granularity,
                     float *scales, size_t scales_count, uint8_t *packed, size_t packed_size);
int dz_quantize_unpack(const float *scales, size_t scales_count, const uint8_t *packed,
                       size_t packed_size, size_t rows, size_t cols, int bits, int granularity,
                       float *dst);

/* Error of one simulated quantization, quant_error_t
 * (src/include/core/quantize.h:58-80): the same fields in the same order. */
typedef struct {
    size_t count;
    float max_abs_error;
    double rms_error;
    double rms_relative;
    double original_rms;
    size_t clipped;
    size_t levels_used;
} dz_quant_error_t;

/* quantize_dequantize_into / quantize_dequantize (src/core/quantize.c:
 * 54-174, src/include/core/quantize.h:88-115): the symmetric grid applied
 * and mapped straight back, dst = scale * clamp(round_half_away(x * inverse),
 * +-qmax) per group with scale = peak / qmax and inverse = qmax / peak; an
 * all-zero group is copied through. Small negatives become -0.0, as in the
 * reference (round_half_away is ceilf there). Same -1 returns (null
 * pointers, empty tensor, bits outside 2..16, bad granularity). The error
 * statistics accumulate in double in the reference's order. */
int dz_quantize_dequantize_into(const float *src, float *dst, size_t rows, size_t cols, int bits,
                                int granularity, dz_quant_error_t *error_out);
int dz_quantize_dequantize(float *values, size_t rows, size_t cols, int bits, int granularity,
                           dz_quant_error_t *error_out);

/* Rows [start, start + count) (axis 0) or columns (axis 1) of a quantized
 * rows x cols matrix as a quantized matrix of its own: the same codes (the
 * reference's layout, INT4 nibbles LSB-first with a zero pad nibble) and the
 * scales of the kept rows / columns (COLUMN scales follow a column slice and
 * stay whole for a row slice, ROW scales the other way round, TENSOR keeps
 * its one scale). Exact: a slice of a matrix quantized per column (or row)
 * is what quantize_pack gives for that slice of the float matrix. Used to
 * shard projections across tensor-parallel ranks; no counterpart in the
 * reference. scales_out / packed_out hold dz_quantized_scale_count /
 * dz_quantized_packed_size of the slice. */
int dz_quantized_slice(const float *scales, size_t scales_count, const uint8_t *packed, size_t packed_size,
                       size_t rows, size_t cols, int bits, int granularity, int axis, size_t start,
                       size_t count, float *scales_out, uint8_t *packed_out);

/* ---- Sinusoidal positions, compute_positional_encoding (src/core/tensor_ops.c:227-248):
 * PE[pos][i] = sin/cos(pos / 10000^(2i/d)), even i -> sin, odd i -> cos. */
int dz_positional_encoding(float *out, size_t rows, size_t dim);

/* ---- FNV-1a, dranzer_fnv1a (src/core/fingerprint.c:14-20). */
uint64_t dz_fnv1a(uint64_t running, const void *data, size_t size);

/* ---- Bundles (docs/model-bundle.md; src/core/bundle.c).
 *
 * dz_bundle_open parses a v1/v3 float32 or v2/v3 quantized bundle with every
 * check model_bundle_load (src/core/bundle.c:523-833) applies - magic,
 * header checksum, shape validity, file size, weight checksum, tensor records,
 * canonical codes (no code above 2*qmax, zero padding, finite non-negative
 * scales), tokenizer checksum, footer - but RETAINS the packed codes and
 * scales instead of unpacking them to fp32 (src/core/bundle.c:748). The file
 * is memory-mapped; tensor blobs point into it until dz_bundle_close. */
typedef struct dz_bundle dz_bundle_t;

typedef struct {
    uint32_t format_version;
    uint32_t numeric;          /* 1 float32, 2 quantized */
    int bits;                  /* 0 for float32 bundles */
    int granularity;
    uint32_t policy_flags;     /* 1 embeddings, 2 biases+norms */
    uint64_t train_window;
    uint64_t seed;
    uint64_t input_fingerprint;
    uint64_t input_bytes;
    uint32_t training_steps;
    uint32_t loss_bits;
    uint64_t total_param_count;
    uint64_t values_quantized;
    uint64_t scales_stored;
} dz_bundle_info_t;

int dz_bundle_open(const char *path, dz_bundle_t **out);
void dz_bundle_close(dz_bundle_t *bundle);
int dz_bundle_desc(const dz_bundle_t *bundle, dz_model_desc_t *out);
int dz_bundle_info(const dz_bundle_t *bundle, dz_bundle_info_t *out);
size_t dz_bundle_tensor_count(const dz_bundle_t *bundle);
int dz_bundle_tensor(const dz_bundle_t *bundle, size_t index, dz_tensor_blob_t *out);
const dz_tensor_blob_t *dz_bundle_tensors(const dz_bundle_t *bundle);
/* Raw tokenizer payload (the reference's portable BPE blob), borrowed. */
const uint8_t *dz_bundle_tokenizer(const dz_bundle_t *bundle, size_t *size);

/* Number of tensors and their shapes/kinds for a model description, in
 * model_param_tensors() order. `out` may be NULL to count. */
size_t dz_model_tensor_layout(const dz_model_desc_t *desc, dz_tensor_blob_t *out, size_t capacity);
size_t dz_model_param_count(const dz_model_desc_t *desc);

/* Writer with the byte layout of model_bundle_save_quantized
 * (src/core/bundle.c:280-501): `params` is the flat float32 parameter vector
 * in the reference's layout (src/core/model.c:38-67,213-228); projections are
 * quantized (the default policy, src/core/model_quantize.c:19-28), everything
 * else stored as float32. The output is byte-identical to the reference
 * writer's for the same parameters, metadata and tokenizer payload. */
typedef struct {
    uint64_t train_window;
    uint64_t seed;
    uint64_t input_fingerprint;
    uint64_t input_bytes;
    uint32_t training_steps;
    uint32_t loss_bits;
} dz_bundle_meta_t;

int dz_bundle_save_quantized(const char *path, const dz_model_desc_t *desc, const float *params,
                             int bits, int granularity, const dz_bundle_meta_t *meta,
                             const uint8_t *tokenizer, size_t tokenizer_size);

/* The 32-byte portable tokenizer payload of a frozen, merge-free
 * special-token encoder with `max_vocab` ids
 * (libs/src/byte_pair_encoding.c:573-616). */
int dz_tokenizer_minimal(uint64_t max_vocab, uint8_t out[32]);

#ifdef __cplusplus
}
#endif

#endif
