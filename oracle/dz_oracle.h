/*
 * Oracle: a CPU restatement of DRANZER's quantized-weight inference path.
 *
 * TEST INFRASTRUCTURE ONLY. This library is the checker that tests/,
 * __graft_entry__.smoke() and bench.py's cpu_baseline leg compare the CUDA
 * path against. The product (dranzer_b200/) never links, loads or calls it.
 *
 * Every function restates a reference function and cites it (paths relative to
 * the DRANZER source tree). It is compiled with strict IEEE flags (no
 * -ffast-math, no FP contraction), so its arithmetic is the plain C semantics
 * of the reference's source text. Parity pins: tests/golden/ holds vectors
 * produced by the reference's own sources (oracle/_ref, built by
 * oracle/Makefile) and the RNG literals of src/tests/core/test_rng.c; the
 * oracle is checked against all of them in tests/test_oracle_golden.py.
 */
#ifndef DZ_ORACLE_H
#define DZ_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#define OR_STREAM_INIT     UINT64_C(0x9e3779b97f4a7c15)
#define OR_STREAM_DROPOUT  UINT64_C(0xbf58476d1ce4e5b9)
#define OR_STREAM_SAMPLING UINT64_C(0x94d049bb133111eb)
#define OR_STREAM_TESTING  UINT64_C(0x2545f4914f6cdd1d)

/* src/core/rng.c:18-57 */
uint64_t or_rng_stream(uint64_t seed, uint64_t stream);
uint64_t or_rng_next(uint64_t *state);
double or_rng_unit(uint64_t *state);

/* Synthetic-input generator shared by harness, oracle and product. */
void or_fill_gaussian(uint64_t *state, float *out, size_t count, double sd);
void or_prompt_ids(uint64_t *state, uint32_t *out, size_t count, uint32_t vocab,
                   const uint32_t *excluded, size_t n_excluded);

/* src/core/quantize.c:183-303. granularity: 0 tensor, 1 row, 2 column. */
size_t or_scale_count(size_t rows, size_t cols, int granularity);
size_t or_packed_size(size_t values, int bits);
int or_quantize_pack(const float *src, size_t rows, size_t cols, int bits, int granularity,
                     float *scales, uint8_t *packed);
int or_quantize_unpack(const float *scales, const uint8_t *packed, size_t rows, size_t cols,
                       int bits, int granularity, float *dst);

/* src/core/quantized_matmul.c:253-295: C[m x n] = A[m x k] . deq(W[k x n]). */
int or_matmul_quantized(const float *A, size_t m, size_t k, size_t n,
                        const float *scales, const uint8_t *packed, int bits, int granularity,
                        float *C);

/* src/core/tensor_ops.c:227-260 */
void or_positional_encoding(float *out, size_t rows, size_t dim);
void or_positional_encoding_at(float *out, size_t position, size_t dim);

/* A decoder with the reference's flat parameter layout (src/core/model.c:38-67,
 * 213-228): token_emb[V x d], output_proj[d x V], output_bias[V], then per layer
 * Wq,Wk,Wv,Wo[d x d], ln_gamma_attn[d], ln_beta_attn[d], W1[d x 4d], b1[4d],
 * W2[4d x d], b2[d], ln_gamma_ffn[d], ln_beta_ffn[d]. */
typedef struct or_model or_model_t;
typedef struct or_cache or_cache_t;

size_t or_model_param_count(size_t vocab, size_t dim, size_t layers);
/* With the architecture bits of src/include/core/model_types.h:26-36 (1 tied
 * embeddings, 2 RoPE, 4 RMSNorm, 8 GELU, 16 SwiGLU): the tensors of
 * src/core/model_params.c:39-103 for those bits, and the forward of
 * src/core/transformer.c:755-858 with rope_rotate (:24-54), rms_normalize
 * (src/core/tensor_ops.c:173-179), gelu / silu (:17-40) and the tied head
 * (src/core/lm_head.c:21-46). */
size_t or_model_param_count_arch(size_t vocab, size_t dim, size_t layers, uint32_t flags);
or_model_t *or_model_create_arch(size_t vocab, size_t dim, size_t heads, size_t layers,
                                 size_t max_seq, uint32_t flags, const float *params);
or_model_t *or_model_create(size_t vocab, size_t dim, size_t heads, size_t layers,
                            size_t max_seq, const float *params);
void or_model_free(or_model_t *m);
or_cache_t *or_cache_create(const or_model_t *m, size_t capacity);
void or_cache_reset(or_cache_t *c);
void or_cache_free(or_cache_t *c);
/* src/core/transformer.c:755-858 */
int or_forward_token(const or_model_t *m, or_cache_t *c, uint32_t token, float *logits);
int or_forward_masked(const or_model_t *m, const uint32_t *ids, size_t T, const uint8_t *padding,
                      const uint8_t *attention, float *logits);

/* src/cli/sampling.c:38-207. strategy: 0 greedy, 1 top-k, 2 top-p. */
uint32_t or_sample_next_token(float *logits, size_t vocab, int strategy, float temperature,
                              size_t top_k, float top_p, uint64_t *rng_state);

/* The decode loop of src/cli/generation.c:231-295 (see ref_harness.c:rh_generate
 * for the exact contract; identical arguments). */
int or_generate(const or_model_t *m, or_cache_t *c, const uint32_t *prompts, size_t n_seq,
                size_t prompt_len, size_t n_new, int strategy, float temperature,
                size_t top_k, float top_p, const uint64_t *seeds,
                const uint32_t *masked, size_t n_masked,
                uint32_t *out_tokens, float *out_logits);

/* generation_decode_with_options (src/cli/generation.c:198-308) with its
 * controls; see dz_oracle.c for the contract. */
int or_generate_ex(const or_model_t *m, or_cache_t *c, const uint32_t *prompts, size_t n_seq,
                   size_t prompt_len, size_t n_new, int strategy, float temperature, size_t top_k,
                   float top_p, const uint64_t *seeds, float penalty, uint32_t eos_id, size_t min_new,
                   uint32_t mask_from, const uint32_t *masked, size_t n_masked, const uint32_t *stop_tokens,
                   const size_t *stop_lengths, size_t n_stops, uint32_t *out_tokens, uint32_t *results,
                   float *out_logits);

/* src/core/fingerprint.c:14-20 */
uint64_t or_fnv1a(uint64_t running, const void *data, size_t size);

#endif
