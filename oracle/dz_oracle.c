/*
 * Oracle: CPU restatement of DRANZER's quantized-weight inference path.
 * TEST INFRASTRUCTURE ONLY - see dz_oracle.h. Only tests/, smoke() and
 * bench.py's cpu_baseline leg load this library, always as the checker.
 */
#include "dz_oracle.h"

#include <float.h>
#include <math.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------ RNG */

/* src/core/rng.c:18-23 (SplitMix64 finaliser). */
static uint64_t or_splitmix64(uint64_t x) {
    x += UINT64_C(0x9e3779b97f4a7c15);
    x = (x ^ (x >> 30)) * UINT64_C(0xbf58476d1ce4e5b9);
    x = (x ^ (x >> 27)) * UINT64_C(0x94d049bb133111eb);
    return x ^ (x >> 31);
}

/* src/core/rng.c:25-33 */
uint64_t or_rng_stream(uint64_t seed, uint64_t stream) {
    uint64_t state = or_splitmix64(seed ^ or_splitmix64(stream));
    return state ? state : UINT64_C(0x9e3779b97f4a7c15);
}

/* src/core/rng.c:35-44: xorshift64* (12, 25, 27). */
uint64_t or_rng_next(uint64_t *state) {
    uint64_t x = *state ? *state : UINT64_C(0x9e3779b97f4a7c15);
    x ^= x >> 12;
    x ^= x << 25;
    x ^= x >> 27;
    *state = x;
    return x * UINT64_C(2685821657736338717);
}

/* src/core/rng.c:46-52: top 53 bits over 2^53. */
double or_rng_unit(uint64_t *state) {
    return (double)(or_rng_next(state) >> 11) * (1.0 / 9007199254740992.0);
}

/* The xorshift state update is linear over GF(2), so the state n draws
 * ahead is the update's n-th power (a 64 x 64 bit matrix, held as the images
 * of the basis vectors) applied to the state. Long fills are cut into pieces
 * started from their own jumped states and generated in parallel; values and
 * final state equal one sequential pass. */
typedef struct { uint64_t col[64]; } or_gf2_map;

static uint64_t or_gf2_apply(const or_gf2_map *m, uint64_t x) {
    uint64_t y = 0;
    for (int j = 0; j < 64; j++)
        if ((x >> j) & 1) y ^= m->col[j];
    return y;
}

static void or_gf2_compose(or_gf2_map *out, const or_gf2_map *a, const or_gf2_map *b) {
    or_gf2_map t;
    for (int j = 0; j < 64; j++) t.col[j] = or_gf2_apply(a, b->col[j]);
    *out = t;
}

static uint64_t or_rng_jump(uint64_t state, uint64_t n) {
    if (n == 0) return state;
    or_gf2_map step, acc;
    for (int j = 0; j < 64; j++) {
        uint64_t x = UINT64_C(1) << j;
        x ^= x >> 12;
        x ^= x << 25;
        x ^= x >> 27;
        step.col[j] = x;
        acc.col[j] = UINT64_C(1) << j;
    }
    while (n) {
        if (n & 1) or_gf2_compose(&acc, &step, &acc);
        or_gf2_compose(&step, &step, &step);
        n >>= 1;
    }
    return or_gf2_apply(&acc, state ? state : UINT64_C(0x9e3779b97f4a7c15));
}

static void or_gaussian_run(uint64_t state, float *out, size_t count, double sd) {
    const double two_pi = 6.283185307179586476925286766559;
    for (size_t i = 0; i < count; i++) {
        double u1 = or_rng_unit(&state);
        if (u1 < 1.0 / 9007199254740992.0) u1 = 1.0 / 9007199254740992.0;
        double u2 = or_rng_unit(&state);
        out[i] = (float)(sd * sqrt(-2.0 * log(u1)) * cos(two_pi * u2));
    }
}

void or_fill_gaussian(uint64_t *state, float *out, size_t count, double sd) {
    const size_t piece = (size_t)1 << 22;
    const long long parts = (long long)((count + piece - 1) / piece);
    const uint64_t s0 = *state;
#pragma omp parallel for schedule(dynamic, 1)
    for (long long t = 0; t < parts; t++) {
        const size_t lo = (size_t)t * piece, hi = lo + piece < count ? lo + piece : count;
        or_gaussian_run(or_rng_jump(s0, 2 * (uint64_t)lo), out + lo, hi - lo, sd);
    }
    *state = or_rng_jump(s0, 2 * (uint64_t)count);
}

void or_prompt_ids(uint64_t *state, uint32_t *out, size_t count, uint32_t vocab,
                   const uint32_t *excluded, size_t n_excluded) {
    for (size_t i = 0; i < count;) {
        uint32_t id = (uint32_t)(or_rng_next(state) % vocab);
        int skip = 0;
        for (size_t e = 0; e < n_excluded; e++) skip |= (id == excluded[e]);
        if (!skip) out[i++] = id;
    }
}

/* -------------------------------------------------------- quantization */

/* src/core/quantize.c:21-23 */
static int or_qmax(int bits) { return (1 << (bits - 1)) - 1; }

/* src/core/quantize.c:48-50 */
static float or_round_half_away(float v) {
    return (v >= 0.0f) ? floorf(v + 0.5f) : ceilf(v - 0.5f);
}

/* src/core/quantize.c:183-197 */
size_t or_scale_count(size_t rows, size_t cols, int granularity) {
    return granularity == 0 ? 1 : granularity == 1 ? rows : cols;
}

/* src/core/quantize.c:199-204 */
size_t or_packed_size(size_t values, int bits) {
    return (values * (size_t)bits + 7) / 8;
}

/* src/core/quantize.c:206-211 */
static size_t or_scale_index(size_t i, size_t cols, int granularity) {
    if (granularity == 1) return i / cols;
    if (granularity == 2) return i % cols;
    return 0;
}

static int or_finite(float v) {
    uint32_t b;
    memcpy(&b, &v, 4);
    return (b & 0x7f800000u) != 0x7f800000u;
}

/* src/core/quantize.c:235-270: two passes (per-group peak |w|, then codes
 * level+qmax packed LSB-first at bit offset i*bits), then scale = peak/qmax. */
int or_quantize_pack(const float *src, size_t rows, size_t cols, int bits, int granularity,
                     float *scales, uint8_t *packed) {
    if (!src || !scales || !packed || rows == 0 || cols == 0 || bits < 2 || bits > 16 ||
        granularity < 0 || granularity > 2) return -1;
    const size_t total = rows * cols;
    const int qmax = or_qmax(bits);
    const size_t ns = or_scale_count(rows, cols, granularity);
    memset(scales, 0, ns * sizeof(float));
    memset(packed, 0, or_packed_size(total, bits));
    for (size_t i = 0; i < total; i++) {
        if (!or_finite(src[i])) return -1;
        size_t g = or_scale_index(i, cols, granularity);
        float mag = fabsf(src[i]);
        if (mag > scales[g]) scales[g] = mag;
    }
    for (size_t i = 0; i < total; i++) {
        const float peak = scales[or_scale_index(i, cols, granularity)];
        float level = 0.0f;
        if (peak > 0.0f) {
            const float inverse = (float)qmax / peak;
            const float scaled = src[i] * inverse;
            /* A subnormal peak makes qmax/peak overflow to +inf and a zero
             * weight then gives 0 * inf = NaN, which passes both clamps; the
             * reference's (int)level of it is INT_MIN on x86, whose low `bits`
             * bits after + qmax are qmax: the zero level. Restated explicitly
             * (pinned by tests/golden/quant.npz). */
            level = (scaled != scaled) ? 0.0f : or_round_half_away(scaled);
        }
        if (level > (float)qmax) level = (float)qmax;
        if (level < -(float)qmax) level = -(float)qmax;
        uint32_t code = (uint32_t)((int)level + qmax);
        size_t bit0 = i * (size_t)bits;
        for (int b = 0; b < bits; b++) {
            if (code & (UINT32_C(1) << b)) {
                size_t pos = bit0 + (size_t)b;
                packed[pos / 8] |= (uint8_t)(1u << (pos % 8));
            }
        }
    }
    /* quantize.c:265-267: scales[g] /= qmax, a true division (the reference
     * compiles quantize.c without -ffast-math, src/Makefile:259-268). */
    for (size_t g = 0; g < ns; g++) {
        if (scales[g] > 0.0f) scales[g] = scales[g] / (float)qmax;
    }
    return 0;
}

/* src/core/quantize.c:272-303: canonical decode; rejects non-finite or
 * negative scales, codes above 2*qmax and non-zero padding bits. */
int or_quantize_unpack(const float *scales, const uint8_t *packed, size_t rows, size_t cols,
                       int bits, int granularity, float *dst) {
    if (!scales || !packed || !dst || rows == 0 || cols == 0 || bits < 2 || bits > 16 ||
        granularity < 0 || granularity > 2) return -1;
    const size_t ns = or_scale_count(rows, cols, granularity);
    for (size_t g = 0; g < ns; g++)
        if (!or_finite(scales[g]) || scales[g] < 0.0f) return -1;
    const size_t total = rows * cols;
    const int qmax = or_qmax(bits);
    for (size_t i = 0; i < total; i++) {
        uint32_t code = 0;
        size_t bit0 = i * (size_t)bits;
        for (int b = 0; b < bits; b++) {
            size_t pos = bit0 + (size_t)b;
            if (packed[pos / 8] & (1u << (pos % 8))) code |= UINT32_C(1) << b;
        }
        if (code > (uint32_t)(2 * qmax)) return -1;
        dst[i] = scales[or_scale_index(i, cols, granularity)] * (float)((int)code - qmax);
    }
    size_t used = total * (size_t)bits;
    if (used % 8 != 0) {
        uint8_t mask = (uint8_t)(0xFFu << (used % 8));
        if (packed[or_packed_size(total, bits) - 1] & mask) return -1;
    }
    return 0;
}

/* ------------------------------------------------------------- matmul */

/* src/core/quantized_matmul.c:67-96: one decoded weight, level * scale. */
static float or_weight(const float *scales, const uint8_t *packed, int bits, int granularity,
                       size_t n, size_t row, size_t col) {
    size_t index = row * n + col;
    int qmax = bits == 8 ? 127 : 7;
    uint32_t code;
    if (bits == 8) {
        code = packed[index];
    } else {
        uint8_t byte = packed[index / 2];
        code = (index & 1u) ? (uint32_t)(byte >> 4) : (uint32_t)(byte & 0x0f);
    }
    float scale = granularity == 1 ? scales[row] : granularity == 2 ? scales[col] : scales[0];
    return (float)((int)code - qmax) * scale;
}

/* src/core/quantized_matmul.c:253-295 with its AVX rungs' arithmetic: the
 * weight is decoded to fp32 (level * scale) and accumulated with a fused
 * multiply-add in ascending k. */
int or_matmul_quantized(const float *A, size_t m, size_t k, size_t n,
                        const float *scales, const uint8_t *packed, int bits, int granularity,
                        float *C) {
    if (!A || !C || !scales || !packed || m == 0 || k == 0 || n == 0 ||
        (bits != 4 && bits != 8)) return -1;
    #pragma omp parallel for schedule(static)
    for (size_t j = 0; j < n; j++) {
        for (size_t i = 0; i < m; i++) {
            float sum = 0.0f;
            for (size_t l = 0; l < k; l++)
                sum = fmaf(A[i * k + l], or_weight(scales, packed, bits, granularity, n, l, j), sum);
            C[i * n + j] = sum;
        }
    }
    return 0;
}

/* -------------------------------------------------------- tensor ops */

/* src/core/tensor_ops.c:227-248 */
void or_positional_encoding(float *out, size_t rows, size_t dim) {
    for (size_t pos = 0; pos < rows; pos++) or_positional_encoding_at(out + pos * dim, pos, dim);
}

/* src/core/tensor_ops.c:250-260. The source computes the inverse frequency
 * as 1.0f / powf(10000.0f, x); the reference's -ffast-math build folds
 * 1/pow(C, x) into exp(-x * ln C), which is what its tables hold (pinned by
 * tests/golden/pe.npz to 1 ulp), so that is the form restated here. */
void or_positional_encoding_at(float *out, size_t position, size_t dim) {
    const float ln_base = logf(10000.0f);
    for (size_t i = 0; i < dim; i++) {
        float scale = expf(-((2.0f * (float)i) / (float)dim) * ln_base);
        float angle = (float)position * scale;
        out[i] = (i % 2 == 0) ? sinf(angle) : cosf(angle);
    }
}

/* src/core/tensor_ops.c:55-76 */
static void or_softmax(float *v, size_t n) {
    if (n == 0) return;
    float mx = v[0];
    for (size_t i = 1; i < n; i++) if (v[i] > mx) mx = v[i];
    float sum = 0.0f;
    for (size_t i = 0; i < n; i++) { v[i] = expf(v[i] - mx); sum += v[i]; }
    if (sum > 0) {
        float inv = 1.0f / sum;
        for (size_t i = 0; i < n; i++) v[i] *= inv;
    }
}

/* src/core/tensor_ops.c:88-111 (layer_normalize -> layer_norm_internal). */
static void or_layer_norm(const float *in, float *out, size_t n, const float *gamma,
                          const float *beta, float eps) {
    float mean = 0.0f;
    for (size_t i = 0; i < n; i++) mean += in[i];
    mean /= (float)n;
    float var = 0.0f;
    for (size_t i = 0; i < n; i++) { float d = in[i] - mean; var += d * d; }
    var /= (float)n;
    float sd = sqrtf(var + eps);
    for (size_t i = 0; i < n; i++) out[i] = gamma[i] * ((in[i] - mean) / sd) + beta[i];
}

/* src/core/tensor_ops.c:173-179 */
static void or_rms_norm(const float *in, float *out, size_t n, const float *gamma, float eps) {
    float ms = 0.0f;
    for (size_t i = 0; i < n; i++) ms += in[i] * in[i];
    float rms = sqrtf(ms / (float)n + eps);
    for (size_t i = 0; i < n; i++) out[i] = gamma[i] * in[i] / rms;
}

/* src/core/tensor_ops.c:17-20 */
static float or_gelu(float x) { return 0.5f * x * (1.0f + erff(x * 0.70710678118654752440f)); }

/* src/core/tensor_ops.c:29-40 */
static float or_silu(float x) {
    float sg;
    if (x >= 0.0f) {
        float z = expf(-x);
        sg = 1.0f / (1.0f + z);
    } else {
        float z = expf(x);
        sg = z / (1.0f + z);
    }
    return x * sg;
}

/* src/core/transformer.c:24-54 (rope_rotate, forward): each head's pairs
 * (2p, 2p + 1) rotated by position * 10000^(-2p / head_dim), the angle and
 * its cosine and sine in double. */
static void or_rope(float *v, size_t dim, size_t heads, size_t position) {
    const size_t hd = dim / heads;
    for (size_t h = 0; h < heads; h++) {
        float *x = v + h * hd;
        for (size_t p = 0; p < hd / 2; p++) {
            const double angle = (double)position * pow(10000.0, -(double)(2 * p) / (double)hd);
            const float c = (float)cos(angle), s = (float)sin(angle);
            const float a = x[2 * p], b = x[2 * p + 1];
            x[2 * p] = a * c - b * s;
            x[2 * p + 1] = a * s + b * c;
        }
    }
}

/* C[n] = a[k] . B[k x n], fp32 fused accumulation in ascending k. */
static void or_matvec(const float *a, const float *B, float *c, size_t k, size_t n) {
    for (size_t j = 0; j < n; j++) c[j] = 0.0f;
    for (size_t l = 0; l < k; l++) {
        const float al = a[l];
        const float *row = B + l * n;
        for (size_t j = 0; j < n; j++) c[j] = fmaf(al, row[j], c[j]);
    }
}

/* -------------------------------------------------------------- model */

typedef struct {
    const float *wq, *wk, *wv, *wo, *g1, *be1, *w1, *b1, *wg, *bg, *w2, *b2, *g2, *be2;
} or_layer_t;

#define OR_TIED 1u
#define OR_ROPE 2u
#define OR_RMSNORM 4u
#define OR_GELU 8u
#define OR_SWIGLU 16u

struct or_model {
    size_t vocab, dim, heads, layers, max_seq;
    uint32_t flags;
    float *params;
    const float *emb, *out_proj, *out_bias;
    or_layer_t *layer;
    float *pe;
};

struct or_cache {
    const or_model_t *m;
    size_t capacity, length, start, total;
    float *keys, *values; /* [layers][capacity][dim] */
    float *hidden, *attn_norm, *query, *concat, *attn_raw, *ff, *gate, *ff_raw, *scores, *pe_row;
};

/* src/core/model.c:107-124 parameter count. */
size_t or_model_param_count_arch(size_t vocab, size_t dim, size_t layers, uint32_t flags) {
    const size_t per = ((flags & OR_SWIGLU) ? 16 : 12) * dim * dim +
                       (((flags & OR_RMSNORM) ? 7 : 9) + ((flags & OR_SWIGLU) ? 4 : 0)) * dim;
    return ((flags & OR_TIED) ? 1 : 2) * vocab * dim + vocab + layers * per;
}

size_t or_model_param_count(size_t vocab, size_t dim, size_t layers) {
    return or_model_param_count_arch(vocab, dim, layers, 0);
}

or_model_t *or_model_create(size_t vocab, size_t dim, size_t heads, size_t layers,
                            size_t max_seq, const float *params) {
    return or_model_create_arch(vocab, dim, heads, layers, max_seq, 0, params);
}

or_model_t *or_model_create_arch(size_t vocab, size_t dim, size_t heads, size_t layers,
                                 size_t max_seq, uint32_t flags, const float *params) {
    if (!params || vocab == 0 || dim == 0 || heads == 0 || dim % heads || layers == 0 ||
        max_seq == 0 || (flags & ~31u) || ((flags & OR_GELU) && (flags & OR_SWIGLU)) ||
        ((flags & OR_ROPE) && (dim / heads) % 2)) return NULL;
    or_model_t *m = calloc(1, sizeof(*m));
    m->flags = flags;
    size_t count = or_model_param_count_arch(vocab, dim, layers, flags);
    m->params = malloc(count * sizeof(float));
    m->layer = calloc(layers, sizeof(or_layer_t));
    m->pe = malloc(max_seq * dim * sizeof(float));
    if (!m->params || !m->layer || !m->pe) { or_model_free(m); return NULL; }
    memcpy(m->params, params, count * sizeof(float));
    m->vocab = vocab; m->dim = dim; m->heads = heads; m->layers = layers; m->max_seq = max_seq;
    /* src/core/model.c:38-67,213-228; src/core/model_params.c:39-103 */
    const float *p = m->params;
    const size_t F = 4 * dim;
    const int rms = (flags & OR_RMSNORM) != 0;
    m->emb = p; p += vocab * dim;
    if (!(flags & OR_TIED)) { m->out_proj = p; p += dim * vocab; }
    m->out_bias = p; p += vocab;
    for (size_t l = 0; l < layers; l++) {
        or_layer_t *L = &m->layer[l];
        L->wq = p; p += dim * dim;
        L->wk = p; p += dim * dim;
        L->wv = p; p += dim * dim;
        L->wo = p; p += dim * dim;
        L->g1 = p; p += dim;
        if (!rms) { L->be1 = p; p += dim; }
        L->w1 = p; p += dim * F;
        L->b1 = p; p += F;
        if (flags & OR_SWIGLU) {
            L->wg = p; p += dim * F;
            L->bg = p; p += F;
        }
        L->w2 = p; p += F * dim;
        L->b2 = p; p += dim;
        L->g2 = p; p += dim;
        if (!rms) { L->be2 = p; p += dim; }
    }
    or_positional_encoding(m->pe, max_seq, dim);
    return m;
}

void or_model_free(or_model_t *m) {
    if (!m) return;
    free(m->params); free(m->layer); free(m->pe); free(m);
}

or_cache_t *or_cache_create(const or_model_t *m, size_t capacity) {
    if (!m || capacity == 0 || capacity > m->max_seq) return NULL;
    or_cache_t *c = calloc(1, sizeof(*c));
    size_t d = m->dim;
    c->m = m;
    c->capacity = capacity;
    c->keys = malloc(m->layers * capacity * d * sizeof(float));
    c->values = malloc(m->layers * capacity * d * sizeof(float));
    c->hidden = malloc(d * sizeof(float));
    c->attn_norm = malloc(d * sizeof(float));
    c->query = malloc(d * sizeof(float));
    c->concat = malloc(d * sizeof(float));
    c->attn_raw = malloc(d * sizeof(float));
    c->ff = malloc(4 * d * sizeof(float));
    c->gate = malloc(4 * d * sizeof(float));
    c->ff_raw = malloc(d * sizeof(float));
    c->scores = malloc(m->heads * capacity * sizeof(float));
    c->pe_row = malloc(d * sizeof(float));
    return c;
}

void or_cache_reset(or_cache_t *c) { c->length = 0; c->start = 0; c->total = 0; }

void or_cache_free(or_cache_t *c) {
    if (!c) return;
    free(c->keys); free(c->values); free(c->hidden); free(c->attn_norm); free(c->query);
    free(c->concat); free(c->attn_raw); free(c->ff); free(c->gate); free(c->ff_raw); free(c->scores);
    free(c->pe_row); free(c);
}

/* src/core/transformer.c:755-858 (model_forward_token), with
 * attention_forward_token / attention_head_forward_token (:686-753). */
int or_forward_token(const or_model_t *m, or_cache_t *c, uint32_t token, float *logits) {
    const size_t d = m->dim, H = m->heads, hd = d / H, F = 4 * d, cap = c->capacity;
    const float eps = 1e-6f;
    size_t pos = c->total, slot, ctx;
    if (c->length < cap) {
        slot = (c->start + c->length) % cap;
        ctx = c->length + 1;
    } else {
        slot = c->start;
        c->start = (c->start + 1) % cap;
        ctx = cap;
    }
    const int rope = (m->flags & OR_ROPE) != 0, rms = (m->flags & OR_RMSNORM) != 0;
    const float *pe = NULL;
    if (!rope) {
        if (pos < m->max_seq) {
            pe = m->pe + pos * d;
        } else {
            or_positional_encoding_at(c->pe_row, pos, d);
            pe = c->pe_row;
        }
    }
    if (token >= m->vocab) token = 0;
    for (size_t i = 0; i < d; i++) c->hidden[i] = m->emb[token * d + i] + (pe ? pe[i] : 0.0f);

    for (size_t l = 0; l < m->layers; l++) {
        const or_layer_t *L = &m->layer[l];
        float *K = c->keys + l * cap * d, *V = c->values + l * cap * d;
        or_matvec(c->hidden, L->wq, c->query, d, d);
        or_matvec(c->hidden, L->wk, K + slot * d, d, d);
        or_matvec(c->hidden, L->wv, V + slot * d, d, d);
        if (rope) {
            or_rope(c->query, d, H, pos);
            or_rope(K + slot * d, d, H, pos);
        }
        for (size_t h = 0; h < H; h++) {
            float *sc = c->scores + h * cap;
            for (size_t j = 0; j < ctx; j++) {
                size_t phys = (c->start + j) % cap;
                float s = 0.0f;
                for (size_t e = 0; e < hd; e++)
                    s += c->query[h * hd + e] * K[phys * d + h * hd + e];
                sc[j] = s / sqrtf((float)hd);
            }
            or_softmax(sc, ctx);
            for (size_t e = 0; e < hd; e++) {
                float s = 0.0f;
                for (size_t j = 0; j < ctx; j++) {
                    size_t phys = (c->start + j) % cap;
                    s += sc[j] * V[phys * d + h * hd + e];
                }
                c->concat[h * hd + e] = s;
            }
        }
        or_matvec(c->concat, L->wo, c->attn_raw, d, d);
        for (size_t i = 0; i < d; i++) c->attn_raw[i] += c->hidden[i];
        if (rms) or_rms_norm(c->attn_raw, c->attn_norm, d, L->g1, eps);
        else or_layer_norm(c->attn_raw, c->attn_norm, d, L->g1, L->be1, eps);
        or_matvec(c->attn_norm, L->w1, c->ff, d, F);
        if (m->flags & OR_SWIGLU) or_matvec(c->attn_norm, L->wg, c->gate, d, F);
        for (size_t i = 0; i < F; i++) {
            float pre = c->ff[i] + L->b1[i];
            if (m->flags & OR_SWIGLU) c->ff[i] = or_silu(pre) * (c->gate[i] + L->bg[i]);
            else if (m->flags & OR_GELU) c->ff[i] = or_gelu(pre);
            else c->ff[i] = pre > 0.0f ? pre : 0.0f;
        }
        or_matvec(c->ff, L->w2, c->ff_raw, F, d);
        for (size_t i = 0; i < d; i++) c->ff_raw[i] += L->b2[i] + c->attn_norm[i];
        if (rms) or_rms_norm(c->ff_raw, c->hidden, d, L->g2, eps);
        else or_layer_norm(c->ff_raw, c->hidden, d, L->g2, L->be2, eps);
    }
    if (m->flags & OR_TIED) {
        /* src/core/lm_head.c:21-46: logits = hidden . token_embeddings^T */
        for (size_t v = 0; v < m->vocab; v++) {
            float s = 0.0f;
            for (size_t i = 0; i < d; i++) s += c->hidden[i] * m->emb[v * d + i];
            logits[v] = s;
        }
    } else {
        or_matvec(c->hidden, m->out_proj, logits, d, m->vocab);
    }
    for (size_t i = 0; i < m->vocab; i++) logits[i] += m->out_bias[i];
    if (c->length < cap) c->length++;
    c->total++;
    return 0;
}

/* src/core/tensor_ops.c:113-141 (layer_norm_forward_cached) for one row. */
static void or_layer_norm_rows(const float *in, float *out, size_t n, const float *gamma,
                               const float *beta, float eps) {
    float mean = 0.0f;
    for (size_t i = 0; i < n; i++) mean += in[i];
    mean /= (float)n;
    float var = 0.0f;
    for (size_t i = 0; i < n; i++) { float d = in[i] - mean; var += d * d; }
    var /= (float)n;
    float sd = sqrtf(var + eps);
    for (size_t i = 0; i < n; i++) out[i] = gamma[i] * ((in[i] - mean) / sd) + beta[i];
}

/* src/core/tensor_ops.c:181-200 (rms_norm_forward_cached) for one row:
 * gamma * (x / rms), the decode step's rms_normalize order differs. */
static void or_rms_norm_rows(const float *in, float *out, size_t n, const float *gamma, float eps) {
    float ms = 0.0f;
    for (size_t i = 0; i < n; i++) ms += in[i] * in[i];
    float rms = sqrtf(ms / (float)n + eps);
    for (size_t i = 0; i < n; i++) out[i] = gamma[i] * (in[i] / rms);
}

/* The masked full-prefix forward: model_forward_masked (src/core/
 * transformer.c:527-576) over model_forward_hidden_masked (:392-519),
 * prepare_attention_mask (:366-390), zero_padded_rows (:355-363),
 * multihead_attention_forward (:192-235) and attention_head_forward
 * (:73-190). One sequence of T ids, padding [T] and attention [T][T] either
 * NULL; logits of the last real position into `logits` [V]. Returns 0, or -1
 * for T == 0, T > max_seq_len or a padding mask without a real position. */
int or_forward_masked(const or_model_t *m, const uint32_t *ids, size_t T, const uint8_t *padding,
                      const uint8_t *attention, float *logits) {
    if (!m || !ids || !logits || T == 0 || T > m->max_seq) return -1;
    const size_t d = m->dim, H = m->heads, hd = d / H, F = 4 * d;
    const float eps = 1e-6f;
    size_t last = T - 1;
    if (padding) {
        int found = 0;
        for (size_t i = 0; i < T; i++) if (padding[i]) { last = i; found = 1; }
        if (!found) return -1;
    }
    const int rope = (m->flags & OR_ROPE) != 0, rms = (m->flags & OR_RMSNORM) != 0;
    const int masked = padding || attention;
    uint8_t *allowed = masked ? malloc(T * T) : NULL;
    float *h = malloc(T * d * sizeof(float)), *q = malloc(T * d * sizeof(float));
    float *k = malloc(T * d * sizeof(float)), *v = malloc(T * d * sizeof(float));
    float *concat = malloc(T * d * sizeof(float)), *raw = malloc(T * d * sizeof(float));
    float *x1 = malloc(T * d * sizeof(float)), *ff = malloc(T * F * sizeof(float));
    float *gate = malloc(T * F * sizeof(float)), *row = malloc(T * sizeof(float));
    int rc = 0;
    if ((masked && !allowed) || !h || !q || !k || !v || !concat || !raw || !x1 || !ff || !gate || !row) {
        rc = -1;
        goto done;
    }
    if (masked) {
        for (size_t i = 0; i < T; i++)
            for (size_t j = 0; j < T; j++) {
                const int qv = !padding || padding[i], kv = !padding || padding[j];
                const int custom = !attention || attention[i * T + j];
                allowed[i * T + j] = (uint8_t)(j <= i && qv && kv && custom);
            }
    }
    for (size_t i = 0; i < T; i++) {
        float *hr = h + i * d;
        if (padding && !padding[i]) { memset(hr, 0, d * sizeof(float)); continue; }
        uint32_t tok = ids[i] < m->vocab ? ids[i] : 0;
        for (size_t e = 0; e < d; e++) hr[e] = m->emb[tok * d + e] + (rope ? 0.0f : m->pe[i * d + e]);
    }
    const float denom = sqrtf((float)hd);
    for (size_t l = 0; l < m->layers; l++) {
        const or_layer_t *L = &m->layer[l];
        for (size_t i = 0; i < T; i++) {
            or_matvec(h + i * d, L->wq, q + i * d, d, d);
            or_matvec(h + i * d, L->wk, k + i * d, d, d);
            or_matvec(h + i * d, L->wv, v + i * d, d, d);
            if (rope) {
                or_rope(q + i * d, d, H, i);
                or_rope(k + i * d, d, H, i);
            }
        }
        memset(concat, 0, T * d * sizeof(float));
        for (size_t hh = 0; hh < H; hh++) {
            for (size_t i = 0; i < T; i++) {
                const float *qi = q + i * d + hh * hd;
                if (masked) {
                    /* scores on allowed edges only; a row with none stays zero */
                    size_t count = 0;
                    float mx = 0.0f;
                    for (size_t j = 0; j < T; j++) {
                        row[j] = 0.0f;
                        if (!allowed[i * T + j]) continue;
                        float sc = 0.0f;
                        for (size_t e = 0; e < hd; e++) sc += qi[e] * k[j * d + hh * hd + e];
                        row[j] = sc / denom;
                        if (count == 0 || row[j] > mx) mx = row[j];
                        count++;
                    }
                    if (count == 0) continue;
                    float sum = 0.0f;
                    for (size_t j = 0; j < T; j++) {
                        if (!allowed[i * T + j]) continue;
                        row[j] = expf(row[j] - mx);
                        sum += row[j];
                    }
                    if (sum > 0.0f) {
                        const float inv = 1.0f / sum;
                        for (size_t j = 0; j < T; j++) if (allowed[i * T + j]) row[j] *= inv;
                    }
                    for (size_t e = 0; e < hd; e++) {
                        float acc = 0.0f;
                        for (size_t j = 0; j < T; j++) {
                            if (!allowed[i * T + j]) continue;
                            acc += row[j] * v[j * d + hh * hd + e];
                        }
                        concat[i * d + hh * hd + e] = acc;
                    }
                } else {
                    for (size_t j = 0; j <= i; j++) {
                        float sc = 0.0f;
                        for (size_t e = 0; e < hd; e++) sc += qi[e] * k[j * d + hh * hd + e];
                        row[j] = sc / denom;
                    }
                    or_softmax(row, i + 1);
                    for (size_t e = 0; e < hd; e++) {
                        float acc = 0.0f;
                        for (size_t j = 0; j <= i; j++) acc += row[j] * v[j * d + hh * hd + e];
                        concat[i * d + hh * hd + e] = acc;
                    }
                }
            }
        }
        for (size_t i = 0; i < T; i++) {
            float *r = raw + i * d;
            or_matvec(concat + i * d, L->wo, r, d, d);
            for (size_t e = 0; e < d; e++) r[e] += h[i * d + e];
            if (rms) or_rms_norm_rows(r, x1 + i * d, d, L->g1, eps);
            else or_layer_norm_rows(r, x1 + i * d, d, L->g1, L->be1, eps);
            if (padding && !padding[i]) memset(x1 + i * d, 0, d * sizeof(float));
        }
        for (size_t i = 0; i < T; i++) {
            float *fr = ff + i * F, *gr = gate + i * F;
            or_matvec(x1 + i * d, L->w1, fr, d, F);
            if (m->flags & OR_SWIGLU) or_matvec(x1 + i * d, L->wg, gr, d, F);
            for (size_t e = 0; e < F; e++) {
                const float pre = fr[e] + L->b1[e];
                if (m->flags & OR_SWIGLU) fr[e] = or_silu(pre) * (gr[e] + L->bg[e]);
                else if (m->flags & OR_GELU) fr[e] = or_gelu(pre);
                else fr[e] = pre > 0.0f ? pre : 0.0f;
            }
            float *r = raw + i * d;
            or_matvec(fr, L->w2, r, F, d);
            for (size_t e = 0; e < d; e++) r[e] += L->b2[e];
            for (size_t e = 0; e < d; e++) r[e] += x1[i * d + e];
            if (rms) or_rms_norm_rows(r, h + i * d, d, L->g2, eps);
            else or_layer_norm_rows(r, h + i * d, d, L->g2, L->be2, eps);
            if (padding && !padding[i]) memset(h + i * d, 0, d * sizeof(float));
        }
    }
    {
        const float *hl = h + last * d;
        if (m->flags & OR_TIED) {
            for (size_t t = 0; t < m->vocab; t++) {
                float sc = 0.0f;
                for (size_t e = 0; e < d; e++) sc += hl[e] * m->emb[t * d + e];
                logits[t] = sc;
            }
        } else {
            or_matvec(hl, m->out_proj, logits, d, m->vocab);
        }
        for (size_t t = 0; t < m->vocab; t++) logits[t] += m->out_bias[t];
    }
done:
    free(allowed); free(h); free(q); free(k); free(v); free(concat); free(raw); free(x1);
    free(ff); free(gate); free(row);
    return rc;
}

/* ----------------------------------------------------------- sampling */

typedef struct { float prob; uint32_t idx; } or_pair_t;

/* Descending order with ties kept in index order. src/cli/sampling.c sorts with
 * qsort(compare_prob_desc); glibc's qsort is a stable merge sort for buffers
 * it can allocate, so equal logits keep ascending index order. */
static void or_sort_desc(or_pair_t *a, size_t n) {
    or_pair_t *tmp = malloc(n * sizeof(*tmp));
    for (size_t width = 1; width < n; width *= 2) {
        for (size_t lo = 0; lo < n; lo += 2 * width) {
            size_t mid = lo + width < n ? lo + width : n;
            size_t hi = lo + 2 * width < n ? lo + 2 * width : n;
            size_t i = lo, j = mid, o = lo;
            while (i < mid && j < hi) tmp[o++] = (a[j].prob > a[i].prob) ? a[j++] : a[i++];
            while (i < mid) tmp[o++] = a[i++];
            while (j < hi) tmp[o++] = a[j++];
        }
        memcpy(a, tmp, n * sizeof(*a));
    }
    free(tmp);
}

/* src/cli/sampling.c:38-53 */
static uint32_t or_greedy(const float *logits, size_t n) {
    uint32_t best = 0;
    float bv = logits[0];
    for (uint32_t i = 1; i < n; i++) if (logits[i] > bv) { bv = logits[i]; best = i; }
    return best;
}

/* src/cli/sampling.c:56-102 */
static uint32_t or_topk(const float *logits, size_t n, size_t k, uint64_t *rng) {
    if (k > n) k = n;
    or_pair_t *p = malloc(n * sizeof(*p));
    for (size_t i = 0; i < n; i++) { p[i].prob = logits[i]; p[i].idx = (uint32_t)i; }
    or_sort_desc(p, n);
    float best = p[0].prob, sum = 0.0f;
    for (size_t i = 0; i < k; i++) { float e = expf(p[i].prob - best); p[i].prob = e; sum += e; }
    float r = (float)or_rng_unit(rng) * sum, acc = 0.0f;
    uint32_t sel = p[0].idx;
    for (size_t i = 0; i < k; i++) {
        acc += p[i].prob;
        if (acc >= r) { sel = p[i].idx; break; }
    }
    free(p);
    return sel;
}

/* src/cli/sampling.c:105-177 */
static uint32_t or_topp(const float *logits, size_t n, float top_p, uint64_t *rng) {
    or_pair_t *p = malloc(n * sizeof(*p));
    float *e = malloc(n * sizeof(float));
    for (size_t i = 0; i < n; i++) { p[i].prob = logits[i]; p[i].idx = (uint32_t)i; }
    or_sort_desc(p, n);
    float mx = p[0].prob, sum_all = 0.0f;
    for (size_t i = 0; i < n; i++) { e[i] = expf(p[i].prob - mx); sum_all += e[i]; }
    float cum = 0.0f, inv = 1.0f / sum_all;
    size_t cand = n;
    for (size_t i = 0; i < n; i++) {
        cum += e[i] * inv;
        if (cum >= top_p) { cand = i + 1; break; }
    }
    float nsum = 0.0f;
    for (size_t i = 0; i < cand; i++) nsum += e[i];
    float r = (float)or_rng_unit(rng) * nsum, acc = 0.0f;
    uint32_t sel = p[0].idx;
    for (size_t i = 0; i < cand; i++) {
        acc += e[i];
        if (acc >= r) { sel = p[i].idx; break; }
    }
    free(p); free(e);
    return sel;
}

/* src/cli/sampling.c:179-207 */
uint32_t or_sample_next_token(float *logits, size_t vocab, int strategy, float temperature,
                              size_t top_k, float top_p, uint64_t *rng_state) {
    if (!logits || vocab == 0) return 0;
    if (strategy == 0 || temperature <= 0.0f || !rng_state) return or_greedy(logits, vocab);
    float inv_t = 1.0f / temperature;
    for (size_t i = 0; i < vocab; i++) logits[i] *= inv_t;
    if (strategy == 1) {
        if (top_k == 0) return or_greedy(logits, vocab);
        return or_topk(logits, vocab, top_k, rng_state);
    }
    if (strategy == 2) {
        if (top_p <= 0.0f || top_p > 1.0f) return or_greedy(logits, vocab);
        return or_topp(logits, vocab, top_p, rng_state);
    }
    return or_greedy(logits, vocab);
}

int or_generate(const or_model_t *m, or_cache_t *c, const uint32_t *prompts, size_t n_seq,
                size_t prompt_len, size_t n_new, int strategy, float temperature,
                size_t top_k, float top_p, const uint64_t *seeds,
                const uint32_t *masked, size_t n_masked,
                uint32_t *out_tokens, float *out_logits) {
    const size_t V = m->vocab;
    float *logits = malloc(V * sizeof(float));
    for (size_t q = 0; q < n_seq; q++) {
        or_cache_reset(c);
        for (size_t i = 0; i < prompt_len; i++)
            or_forward_token(m, c, prompts[q * prompt_len + i], logits);
        uint64_t rng = seeds ? or_rng_stream(seeds[q], OR_STREAM_SAMPLING) : 0;
        for (size_t i = 0; i < n_new; i++) {
            for (size_t k = 0; k < n_masked; k++)
                if (masked[k] < V) logits[masked[k]] = -FLT_MAX;
            if (out_logits) memcpy(out_logits + (q * n_new + i) * V, logits, V * sizeof(float));
            uint32_t next = or_sample_next_token(logits, V, strategy, temperature, top_k, top_p,
                                                 seeds ? &rng : NULL);
            out_tokens[q * n_new + i] = next;
            if (i + 1 < n_new) or_forward_token(m, c, next, logits);
        }
    }
    free(logits);
    return 0;
}

/* src/cli/generation.c:52-72: the sign-aware penalty, once per token id
 * present in sequence[0..count). */
static void or_repetition_penalty(float *logits, size_t vocab, const uint32_t *sequence, size_t count,
                                  float penalty) {
    if (penalty <= 1.0f) return;
    for (size_t i = 0; i < count; i++) {
        uint32_t id = sequence[i];
        if (id >= vocab) continue;
        int seen = 0;
        for (size_t j = 0; j < i; j++)
            if (sequence[j] == id) { seen = 1; break; }
        if (seen) continue;
        if (logits[id] < 0.0f) logits[id] *= penalty;
        else logits[id] /= penalty;
    }
}

/* The decode loop of generation_decode_with_options (src/cli/generation.c:
 * 198-308) with its controls: repetition penalty over prompt + generated ids,
 * control masking (the ids in `masked` and every id >= mask_from, :31-46),
 * EOS masked until min_new tokens are drawn (:250-254), a draw of EOS ends
 * the sequence (:262-269), and the generated tail matching a stop sequence
 * that starts at or after min_new ends it (:120-138, :271-280). results[5 *
 * q] = new_count, emitted_count, stopped_on_eos, stopped_on_stop_sequence,
 * stop_sequence_index (UINT32_MAX when none). Tokens after the end are
 * UINT32_MAX. out_logits, when not NULL, receives the logits of every draw
 * after penalty and masking ([n_seq][n_new][V]). */
int or_generate_ex(const or_model_t *m, or_cache_t *c, const uint32_t *prompts, size_t n_seq,
                   size_t prompt_len, size_t n_new, int strategy, float temperature, size_t top_k,
                   float top_p, const uint64_t *seeds, float penalty, uint32_t eos_id, size_t min_new,
                   uint32_t mask_from, const uint32_t *masked, size_t n_masked, const uint32_t *stop_tokens,
                   const size_t *stop_lengths, size_t n_stops, uint32_t *out_tokens, uint32_t *results,
                   float *out_logits) {
    const size_t V = m->vocab;
    float *logits = malloc(V * sizeof(float));
    uint32_t *seq = malloc((prompt_len + n_new) * sizeof(uint32_t));
    if (!logits || !seq) { free(logits); free(seq); return -1; }
    for (size_t q = 0; q < n_seq; q++) {
        or_cache_reset(c);
        memcpy(seq, prompts + q * prompt_len, prompt_len * sizeof(uint32_t));
        for (size_t i = 0; i < prompt_len; i++) or_forward_token(m, c, seq[i], logits);
        uint64_t rng = seeds ? or_rng_stream(seeds[q], OR_STREAM_SAMPLING) : 0;
        size_t total = prompt_len, new_count = 0, emitted = 0;
        uint32_t on_eos = 0, on_stop = 0, stop_index = UINT32_MAX;
        for (size_t i = 0; i < n_new; i++) out_tokens[q * n_new + i] = UINT32_MAX;
        int ended = 0;
        for (size_t i = 0; i < n_new && !ended; i++) {
            or_repetition_penalty(logits, V, seq, total, penalty);
            for (size_t k = 0; k < n_masked; k++)
                if (masked[k] < V) logits[masked[k]] = -FLT_MAX;
            for (size_t k = mask_from; k < V; k++) logits[k] = -FLT_MAX;
            if (new_count < min_new && eos_id < V) logits[eos_id] = -FLT_MAX;
            if (out_logits) memcpy(out_logits + (q * n_new + i) * V, logits, V * sizeof(float));
            uint32_t next = or_sample_next_token(logits, V, strategy, temperature, top_k, top_p,
                                                 seeds ? &rng : NULL);
            seq[total++] = next;
            new_count++;
            out_tokens[q * n_new + i] = next;
            if (next == eos_id) {
                emitted = new_count - 1;
                on_eos = 1;
                ended = 1;
                break;
            }
            const uint32_t *gen = seq + prompt_len;
            size_t off = 0;
            for (size_t s = 0; s < n_stops; s++) {
                const size_t len = stop_lengths[s];
                if (len <= new_count && new_count - len >= min_new &&
                    memcmp(gen + new_count - len, stop_tokens + off, len * sizeof(uint32_t)) == 0) {
                    emitted = new_count - len;
                    on_stop = 1;
                    stop_index = (uint32_t)s;
                    ended = 1;
                    break;
                }
                off += len;
            }
            if (ended) break;
            if (i + 1 < n_new) or_forward_token(m, c, next, logits);
        }
        if (!on_eos && !on_stop) emitted = new_count;
        uint32_t *r = results + 5 * q;
        r[0] = (uint32_t)new_count;
        r[1] = (uint32_t)emitted;
        r[2] = on_eos;
        r[3] = on_stop;
        r[4] = stop_index;
    }
    free(logits);
    free(seq);
    return 0;
}

/* src/core/fingerprint.c:14-20 */
uint64_t or_fnv1a(uint64_t running, const void *data, size_t size) {
    const uint8_t *b = data;
    for (size_t i = 0; i < size; i++) { running ^= b[i]; running *= UINT64_C(1099511628211); }
    return running;
}
