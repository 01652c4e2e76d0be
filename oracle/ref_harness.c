/*
 * Harness around the reference's own C sources (test infrastructure only).
 *
 * Compiled by oracle/Makefile (`make -C oracle ref`) together with the
 * reference's core objects into oracle/_ref/libdzref.so. Every function here
 * drives the reference's public or core API unchanged; nothing of the
 * reference is re-implemented. Used to generate tests/golden/ fixtures and as
 * the CPU baseline ("kind": "reference") beside the GPU numbers.
 *
 * Synthetic inputs follow one generator shared with the product and the
 * oracle: dranzer_rng_stream(seed, DRANZER_RNG_STREAM_TESTING), one value per
 * two dranzer_rng_unit() draws through Box-Muller (u1 floored at 2^-53),
 * w = (float)(sd * sqrt(-2 ln u1) * cos(2 pi u2)).
 */

#include "core/bundle.h"
#include "core/model.h"
#include "core/model_params.h"
#include "core/model_quantize.h"
#include "core/quantize.h"
#include "core/quantized_matmul.h"
#include "core/rng.h"
#include "core/transformer.h"
#include "cli/sampling.h"
#include "cli/generation.h"
#include "byte_pair_encoding.h"
#include <float.h>
#include <math.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>
#include <omp.h>

#define RH_TWO_PI 6.283185307179586476925286766559

float rh_gaussian(uint64_t *state, double sd) {
    double u1 = dranzer_rng_unit(state);
    if (u1 < 1.0 / 9007199254740992.0) u1 = 1.0 / 9007199254740992.0;
    double u2 = dranzer_rng_unit(state);
    return (float)(sd * sqrt(-2.0 * log(u1)) * cos(RH_TWO_PI * u2));
}

/* The xorshift state update is linear over GF(2), so the state n draws
 * ahead is the update's n-th power (a 64 x 64 bit matrix, held as the images
 * of the basis vectors) applied to the state. Long fills are cut into pieces
 * started from their own jumped states and generated in parallel; values and
 * final state equal one sequential pass. */
typedef struct { uint64_t col[64]; } rh_gf2_map;

static uint64_t rh_gf2_apply(const rh_gf2_map *m, uint64_t x) {
    uint64_t y = 0;
    for (int j = 0; j < 64; j++)
        if ((x >> j) & 1) y ^= m->col[j];
    return y;
}

static void rh_gf2_compose(rh_gf2_map *out, const rh_gf2_map *a, const rh_gf2_map *b) {
    rh_gf2_map t;
    for (int j = 0; j < 64; j++) t.col[j] = rh_gf2_apply(a, b->col[j]);
    *out = t;
}

static uint64_t rh_rng_jump(uint64_t state, uint64_t n) {
    if (n == 0) return state;
    rh_gf2_map step, acc;
    for (int j = 0; j < 64; j++) {
        uint64_t x = UINT64_C(1) << j;
        x ^= x >> 12;
        x ^= x << 25;
        x ^= x >> 27;
        step.col[j] = x;
        acc.col[j] = UINT64_C(1) << j;
    }
    while (n) {
        if (n & 1) rh_gf2_compose(&acc, &step, &acc);
        rh_gf2_compose(&step, &step, &step);
        n >>= 1;
    }
    return rh_gf2_apply(&acc, state ? state : UINT64_C(0x9e3779b97f4a7c15));
}

/* Same values and final state as rh_gaussian called count times. */
void rh_fill_gaussian(uint64_t *state, float *out, size_t count, double sd) {
    const size_t piece = (size_t)1 << 22;
    const long long parts = (long long)((count + piece - 1) / piece);
    const uint64_t s0 = *state;
#pragma omp parallel for schedule(dynamic, 1)
    for (long long t = 0; t < parts; t++) {
        const size_t lo = (size_t)t * piece, hi = lo + piece < count ? lo + piece : count;
        uint64_t st = rh_rng_jump(s0, 2 * (uint64_t)lo);
        for (size_t i = lo; i < hi; i++) out[i] = rh_gaussian(&st, sd);
    }
    *state = rh_rng_jump(s0, 2 * (uint64_t)count);
}

/* Parameter count of a model of this shape and architecture, as
 * model_new lays it out (src/core/model.c:37-72, 120-124): embeddings (and
 * the untied output projection), output bias, then per layer 4 d^2, the
 * norms (beta only for LayerNorm), W_ff1 + b_ff1, the SwiGLU gate branch,
 * W_ff2 + b_ff2. */
size_t rh_arch_param_count(size_t vocab, size_t dim, size_t layers, uint32_t flags) {
    const size_t F = 4 * dim, norms = (flags & MODEL_ARCH_RMSNORM) ? dim : 2 * dim;
    size_t per = 4 * dim * dim + 2 * norms + dim * F + F + F * dim + dim;
    if (flags & MODEL_ARCH_SWIGLU) per += dim * F + F;
    return vocab * dim * ((flags & MODEL_ARCH_TIED_EMBEDDINGS) ? 1 : 2) + vocab + layers * per;
}

/* Build a model over a parameter buffer of our own (no initialisation pass),
 * fill it with N(0, 0.02) for embeddings/projections (model_param_tensors
 * order), 1/0 for norm gamma/beta and 0 for biases, then write a quantized
 * bundle with the reference's own writer (projections only, per the default
 * policy). */
int rh_build_bundle_arch(const char *path, size_t vocab, size_t dim, size_t heads,
                         size_t layers, size_t max_seq, uint64_t weight_seed,
                         int bits, int granularity, uint32_t flags) {
    neural_model_t model = {0};
    const size_t total = rh_arch_param_count(vocab, dim, layers, flags);
    float *params = calloc(total, sizeof(float));
    if (!params) return -2;
    if (model_new_external_parameters_architecture(&model, vocab, dim, heads, layers, max_seq, flags,
                                                   params) != MODEL_SUCCESS) {
        free(params);
        return -1;
    }
    if (model.total_param_count != total) {
        model_free(&model);
        free(params);
        return -4;
    }
    size_t count = model_param_tensor_count(&model);
    param_tensor_t *tensors = calloc(count, sizeof(*tensors));
    if (!tensors) { model_free(&model); free(params); return -2; }
    model_param_tensors(&model, tensors, count);
    uint64_t state = dranzer_rng_stream(weight_seed, DRANZER_RNG_STREAM_TESTING);
    for (size_t t = 0; t < count; t++) {
        size_t n = tensors[t].rows * tensors[t].cols;
        switch (tensors[t].kind) {
            case PARAM_KIND_PROJECTION:
            case PARAM_KIND_EMBEDDING:
                rh_fill_gaussian(&state, tensors[t].values, n, 0.02);
                break;
            case PARAM_KIND_NORM:
                for (size_t i = 0; i < n; i++)
                    tensors[t].values[i] = strstr(tensors[t].name, "ln_gamma") != NULL ? 1.0f : 0.0f;
                break;
            default:
                memset(tensors[t].values, 0, n * sizeof(float));
        }
    }
    free(tensors);

    bpe_encoder_t encoder = {0};
    if (bpe_encoder_new_with_special_tokens(&encoder, vocab) != BPE_SUCCESS ||
        bpe_encoder_freeze(&encoder) != BPE_SUCCESS) {
        model_free(&model);
        free(params);
        return -3;
    }
    model_bundle_metadata_t meta = {0};
    meta.train_window = max_seq;
    meta.seed = weight_seed;
    model_quant_config_t config;
    model_quantize_default_config(&config);
    config.bits = bits;
    config.granularity = (quant_granularity_t)granularity;
    bundle_errors_t rc = model_bundle_save_quantized(&model, &encoder, &meta, &config, NULL, path);
    bpe_encoder_free(&encoder);
    model_free(&model);
    free(params);
    return rc == BUNDLE_SUCCESS ? 0 : -10 - (int)rc;
}

int rh_build_bundle(const char *path, size_t vocab, size_t dim, size_t heads,
                    size_t layers, size_t max_seq, uint64_t weight_seed,
                    int bits, int granularity) {
    return rh_build_bundle_arch(path, vocab, dim, heads, layers, max_seq, weight_seed, bits,
                                granularity, 0);
}

typedef struct {
    neural_model_t model;
    bpe_encoder_t *encoder;
    model_kv_cache_t cache;
} rh_session_t;

void *rh_load(const char *path) {
    rh_session_t *s = calloc(1, sizeof(*s));
    if (!s) return NULL;
    model_bundle_metadata_t meta;
    if (model_bundle_load(&s->model, &s->encoder, &meta, path) != BUNDLE_SUCCESS ||
        model_kv_cache_init(&s->cache, &s->model) != MODEL_SUCCESS) {
        free(s);
        return NULL;
    }
    return s;
}

void rh_free(void *handle) {
    rh_session_t *s = handle;
    if (!s) return;
    model_kv_cache_free(&s->cache);
    if (s->encoder) { bpe_encoder_free(s->encoder); free(s->encoder); }
    model_free(&s->model);
    free(s);
}

size_t rh_param_count(void *handle) { return ((rh_session_t *)handle)->model.total_param_count; }
const void *rh_model(void *handle) { return &((rh_session_t *)handle)->model; }
const float *rh_params(void *handle) { return ((rh_session_t *)handle)->model.params; }
void rh_reset(void *handle) { model_kv_cache_reset(&((rh_session_t *)handle)->cache); }

int rh_forward_token(void *handle, uint32_t token, float *logits) {
    rh_session_t *s = handle;
    return model_forward_token(&s->model, &s->cache, token, logits) == MODEL_SUCCESS ? 0 : -1;
}

/* model_forward_masked (src/core/transformer.c:527-576) on the loaded model:
 * the full-prefix forward of one sequence of seq_len ids with an optional
 * padding mask [seq_len] and attention mask [seq_len][seq_len] (either may be
 * NULL), logits of the last real position into `logits` [V]. Returns the
 * reference's model_errors_t. */
int rh_forward_masked(void *handle, const uint32_t *ids, size_t seq_len, const uint8_t *padding,
                      const uint8_t *attention, float *logits) {
    rh_session_t *s = handle;
    uint32_t *copy = malloc(seq_len * sizeof(*copy));
    if (!copy) return -1;
    memcpy(copy, ids, seq_len * sizeof(*copy));
    model_attention_mask_t mask = {padding, attention};
    const int rc = (int)model_forward_masked(&s->model, copy, seq_len,
                                             (padding || attention) ? &mask : NULL, logits);
    free(copy);
    return rc;
}

/* The decode loop of generation_decode_with_options (src/cli/generation.c:
 * 231-295) with the tokenizer treated as fully trained (vocab_size == V):
 * control ids `masked` are set to -FLT_MAX before each draw, repetition
 * penalty 1.0 (a no-op), no stop sequences. Sequences run one after another,
 * as the reference does. `out_tokens` is [n_seq][n_new]; `out_logits`, when not
 * NULL, receives the raw logits each draw was taken from, [n_seq][n_new][V]. */
int rh_generate(void *handle, const uint32_t *prompts, size_t n_seq,
                size_t prompt_len, size_t n_new, int strategy,
                float temperature, size_t top_k, float top_p,
                const uint64_t *seeds, const uint32_t *masked, size_t n_masked,
                uint32_t *out_tokens, float *out_logits) {
    rh_session_t *s = handle;
    const size_t vocab = s->model.vocab_size;
    float *logits = s->model.ws_logits;
    for (size_t q = 0; q < n_seq; q++) {
        model_kv_cache_reset(&s->cache);
        for (size_t i = 0; i < prompt_len; i++) {
            if (model_forward_token(&s->model, &s->cache, prompts[q * prompt_len + i],
                                    logits) != MODEL_SUCCESS) return -1;
        }
        uint64_t rng = seeds ? dranzer_rng_stream(seeds[q], DRANZER_RNG_STREAM_SAMPLING) : 0;
        for (size_t i = 0; i < n_new; i++) {
            for (size_t m = 0; m < n_masked; m++)
                if (masked[m] < vocab) logits[masked[m]] = -FLT_MAX;
            if (out_logits) memcpy(out_logits + (q * n_new + i) * vocab, logits, vocab * sizeof(float));
            uint32_t next = sample_next_token(logits, vocab, (sampling_strategy_t)strategy,
                                              temperature, top_k, top_p,
                                              seeds ? &rng : NULL);
            out_tokens[q * n_new + i] = next;
            if (i + 1 < n_new &&
                model_forward_token(&s->model, &s->cache, next, logits) != MODEL_SUCCESS)
                return -2;
        }
    }
    return 0;
}

/* The reference's own generation loop, generation_decode_with_options
 * (src/cli/generation.c:198-308), per sequence with its controls: sampling
 * strategy, repetition penalty, minimum new tokens and stop sequences
 * (token ids, concatenated, with their lengths), the bundle's tokenizer for
 * control masking and EOS. out_tokens [n_seq][n_new] receives the drawn
 * tokens (UINT32_MAX after the end); results [n_seq][5] = new_count,
 * emitted_count, stopped_on_eos, stopped_on_stop_sequence,
 * stop_sequence_index (UINT32_MAX when none). Returns the first non-zero
 * generation_errors_t, or 0. */
int rh_generate_ex(void *handle, const uint32_t *prompts, size_t n_seq, size_t prompt_len,
                   size_t n_new, int strategy, float temperature, size_t top_k, float top_p,
                   const uint64_t *seeds, float penalty, size_t min_new,
                   const uint32_t *stop_tokens, const size_t *stop_lengths, size_t n_stops,
                   uint32_t *out_tokens, uint32_t *results) {
    rh_session_t *s = handle;
    generation_stop_sequence_t stops[16];
    if (n_stops > 16) return -100;
    size_t off = 0;
    for (size_t i = 0; i < n_stops; i++) {
        stops[i].token_ids = stop_tokens + off;
        stops[i].token_count = stop_lengths[i];
        off += stop_lengths[i];
    }
    uint32_t *seq = malloc((prompt_len + n_new) * sizeof(uint32_t));
    if (!seq) return -101;
    for (size_t q = 0; q < n_seq; q++) {
        memcpy(seq, prompts + q * prompt_len, prompt_len * sizeof(uint32_t));
        uint64_t rng = seeds ? dranzer_rng_stream(seeds[q], DRANZER_RNG_STREAM_SAMPLING) : 0;
        generation_options_t opt;
        generation_options_init(&opt);
        opt.strategy = (sampling_strategy_t)strategy;
        opt.temperature = temperature;
        opt.top_k = top_k;
        opt.top_p = top_p;
        opt.repetition_penalty = penalty;
        opt.minimum_new_tokens = min_new;
        opt.sequence_capacity = prompt_len + n_new;
        opt.stop_sequences = n_stops ? stops : NULL;
        opt.stop_sequence_count = n_stops;
        opt.rng_state = seeds ? &rng : NULL;
        generation_result_t res;
        generation_errors_t rc = generation_decode_with_options(&s->model, s->encoder, seq, prompt_len,
                                                                n_new, &opt, &res);
        if (rc != GENERATION_SUCCESS) { free(seq); return (int)rc; }
        for (size_t i = 0; i < n_new; i++)
            out_tokens[q * n_new + i] = i < res.new_count ? seq[prompt_len + i] : UINT32_MAX;
        uint32_t *r = results + 5 * q;
        r[0] = (uint32_t)res.new_count;
        r[1] = (uint32_t)res.emitted_count;
        r[2] = (uint32_t)res.stopped_on_eos;
        r[3] = (uint32_t)res.stopped_on_stop_sequence;
        r[4] = res.stop_sequence_index == SIZE_MAX ? UINT32_MAX : (uint32_t)res.stop_sequence_index;
    }
    free(seq);
    return 0;
}

/* The tokenizer's assigned vocabulary size (ids at or above it are masked
 * by generation_mask_control_logits, src/cli/generation.c:43-45). */
size_t rh_tokenizer_vocab(void *handle) { return ((rh_session_t *)handle)->encoder->vocab_size; }

/* Quantized weight matrix through the reference's encoder and INT8/INT4
 * matmul (src/core/quantized_matmul.c). */
void *rh_qmat_encode(const float *values, size_t k, size_t n, int bits, int granularity) {
    quantized_weight_matrix_t *q = calloc(1, sizeof(*q));
    if (!q) return NULL;
    if (quantized_weight_matrix_encode(q, values, k, n, bits,
                                       (quant_granularity_t)granularity) != 0) {
        free(q);
        return NULL;
    }
    return q;
}

const float *rh_qmat_scales(void *h, size_t *count) {
    quantized_weight_matrix_t *q = h;
    *count = q->scale_count;
    return q->scales;
}

const uint8_t *rh_qmat_packed(void *h, size_t *size) {
    quantized_weight_matrix_t *q = h;
    *size = q->packed_size;
    return q->packed;
}

int rh_qmat_matmul(void *h, const float *a, float *c, size_t m) {
    quantized_weight_matrix_t *q = h;
    return matmul_quantized_weight(a, q, c, m, q->rows, 0);
}

void rh_qmat_free(void *h) {
    quantized_weight_matrix_free(h);
    free(h);
}

double rh_now(void) {
    struct timespec ts;
    clock_gettime(CLOCK_MONOTONIC, &ts);
    return (double)ts.tv_sec + 1e-9 * (double)ts.tv_nsec;
}

/* Threads the reference's OpenMP regions use from the calling thread on. */
void rh_set_omp_threads(int n) { omp_set_num_threads(n); }
