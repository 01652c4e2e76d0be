/*
 * dranzer-b200 host library: quantizer, code-retaining bundle loader/writer,
 * positional table, RNG and synthetic inputs. Plain C11, strict IEEE
 * (built without -ffast-math and without FP contraction).
 */
#define _GNU_SOURCE
#include "dz_host.h"

#include <errno.h>
#include <fcntl.h>
#include <math.h>
#include <pthread.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

/* ------------------------------------------------------------------ RNG */

static uint64_t splitmix64(uint64_t x) {
    x += UINT64_C(0x9e3779b97f4a7c15);
    x = (x ^ (x >> 30)) * UINT64_C(0xbf58476d1ce4e5b9);
    x = (x ^ (x >> 27)) * UINT64_C(0x94d049bb133111eb);
    return x ^ (x >> 31);
}

uint64_t dz_rng_stream(uint64_t seed, uint64_t stream) {
    uint64_t s = splitmix64(seed ^ splitmix64(stream));
    return s ? s : UINT64_C(0x9e3779b97f4a7c15);
}

uint64_t dz_rng_next(uint64_t *state) {
    uint64_t x = *state ? *state : UINT64_C(0x9e3779b97f4a7c15);
    x ^= x >> 12;
    x ^= x << 25;
    x ^= x >> 27;
    *state = x;
    return x * UINT64_C(2685821657736338717);
}

double dz_rng_unit(uint64_t *state) {
    return (double)(dz_rng_next(state) >> 11) * (1.0 / 9007199254740992.0);
}

/* The xorshift state update is linear over GF(2): the state n draws ahead is
 * a 64 x 64 bit matrix (the update's n-th power) applied to the state. A
 * matrix is held as the images of the 64 basis vectors. */
typedef struct { uint64_t col[64]; } gf2_map;

static uint64_t gf2_apply(const gf2_map *m, uint64_t x) {
    uint64_t y = 0;
    for (int j = 0; j < 64; j++)
        if ((x >> j) & 1) y ^= m->col[j];
    return y;
}

static void gf2_compose(gf2_map *out, const gf2_map *a, const gf2_map *b) {
    gf2_map t;
    for (int j = 0; j < 64; j++) t.col[j] = gf2_apply(a, b->col[j]);
    *out = t;
}

/* The state after n draws from `state`. */
static uint64_t rng_jump(uint64_t state, uint64_t n) {
    if (n == 0) return state;
    gf2_map step, acc;
    for (int j = 0; j < 64; j++) {
        uint64_t x = UINT64_C(1) << j;
        x ^= x >> 12;
        x ^= x << 25;
        x ^= x >> 27;
        step.col[j] = x;
        acc.col[j] = UINT64_C(1) << j;
    }
    while (n) {
        if (n & 1) gf2_compose(&acc, &step, &acc);
        gf2_compose(&step, &step, &step);
        n >>= 1;
    }
    return gf2_apply(&acc, state ? state : UINT64_C(0x9e3779b97f4a7c15));
}

static void gaussian_run(uint64_t state, float *out, size_t count, double sd) {
    const double two_pi = 6.283185307179586476925286766559;
    const double floor_u = 1.0 / 9007199254740992.0;
    for (size_t i = 0; i < count; i++) {
        double u1 = dz_rng_unit(&state);
        if (u1 < floor_u) u1 = floor_u;
        double u2 = dz_rng_unit(&state);
        out[i] = (float)(sd * sqrt(-2.0 * log(u1)) * cos(two_pi * u2));
    }
}

typedef struct { uint64_t state; float *out; size_t count; double sd; } gaussian_part;

static void *gaussian_thread(void *arg) {
    gaussian_part *p = (gaussian_part *)arg;
    gaussian_run(p->state, p->out, p->count, p->sd);
    return NULL;
}

/* One value per two draws (Box-Muller). Long fills are cut into pieces, each
 * started from the state that the draws before it leave (rng_jump), and run
 * on the host's cores; the values and the final state are those of one
 * sequential pass. */
void dz_synth_gaussian(uint64_t *state, float *out, size_t count, double sd) {
    enum { MAX_PARTS = 64 };
    const size_t min_part = (size_t)1 << 22;
    long cores = sysconf(_SC_NPROCESSORS_ONLN);
    size_t parts = count / min_part;
    if (parts > (size_t)(cores > 0 ? cores : 1)) parts = (size_t)(cores > 0 ? cores : 1);
    if (parts > MAX_PARTS) parts = MAX_PARTS;
    if (parts < 2) {
        gaussian_run(*state, out, count, sd);
        *state = rng_jump(*state, 2 * (uint64_t)count);
        return;
    }
    gaussian_part job[MAX_PARTS];
    pthread_t th[MAX_PARTS];
    int started[MAX_PARTS] = {0};
    const size_t per = (count + parts - 1) / parts;
    for (size_t t = 0; t < parts; t++) {
        const size_t lo = t * per < count ? t * per : count, hi = lo + per < count ? lo + per : count;
        job[t].state = rng_jump(*state, 2 * (uint64_t)lo);
        job[t].out = out + lo;
        job[t].count = hi - lo;
        job[t].sd = sd;
        started[t] = pthread_create(&th[t], NULL, gaussian_thread, &job[t]) == 0;
        if (!started[t]) gaussian_thread(&job[t]);
    }
    for (size_t t = 0; t < parts; t++)
        if (started[t]) pthread_join(th[t], NULL);
    *state = rng_jump(*state, 2 * (uint64_t)count);
}

void dz_synth_prompt_ids(uint64_t *state, uint32_t *out, size_t count, uint32_t vocab,
                         const uint32_t *excluded, size_t n_excluded) {
    size_t i = 0;
    while (i < count) {
        uint32_t id = (uint32_t)(dz_rng_next(state) % vocab);
        int rejected = 0;
        for (size_t e = 0; e < n_excluded; e++) rejected |= (excluded[e] == id);
        if (!rejected) out[i++] = id;
    }
}

/* -------------------------------------------------------------- FNV-1a */

uint64_t dz_fnv1a(uint64_t running, const void *data, size_t size) {
    const uint8_t *b = (const uint8_t *)data;
    for (size_t i = 0; i < size; i++) {
        running ^= b[i];
        running *= UINT64_C(1099511628211);
    }
    return running;
}

#define DZ_FNV_OFFSET UINT64_C(0xcbf29ce484222325)

/* -------------------------------------------------------- quantization */

static int valid_granularity(int g) { return g >= DZ_GRAN_TENSOR && g <= DZ_GRAN_COLUMN; }

int dz_quantized_scale_count(size_t rows, size_t cols, int granularity, size_t *out_count) {
    if (!out_count || rows == 0 || cols == 0 || !valid_granularity(granularity)) return -1;
    *out_count = granularity == DZ_GRAN_TENSOR ? 1 : granularity == DZ_GRAN_ROW ? rows : cols;
    return 0;
}

int dz_quantized_packed_size(size_t value_count, int bits, size_t *out_size) {
    if (!out_size || value_count == 0 || bits < 2 || bits > 16 ||
        value_count > (SIZE_MAX - 7) / (size_t)bits) return -1;
    *out_size = (value_count * (size_t)bits + 7) / 8;
    return 0;
}

static int finite_bits(float v) {
    uint32_t b;
    memcpy(&b, &v, sizeof(b));
    return (b & 0x7f800000u) != 0x7f800000u;
}

/* round half away from zero, written as the reference writes it
 * (src/core/quantize.c:48-50) so ties do not depend on the rounding mode. */
static inline float round_half_away(float v) {
    return (v >= 0.0f) ? floorf(v + 0.5f) : ceilf(v - 0.5f);
}

/* level = clamp(round_half_away(w * (qmax / peak)), +-qmax), code = level + qmax
 * (src/core/quantize.c:257-264). When the peak is subnormal, qmax / peak
 * overflows to +inf and a zero weight gives NaN, which passes both clamps; the
 * reference's (int) conversion of it yields INT_MIN on x86, whose low `bits`
 * bits after + qmax are qmax, i.e. the zero level, and so does this. */
static inline uint32_t quant_code(float w, float peak, int qmax) {
    float level = 0.0f;
    if (peak > 0.0f) {
        const float scaled = w * ((float)qmax / peak);
        level = (scaled != scaled) ? 0.0f : round_half_away(scaled);
    }
    if (level > (float)qmax) level = (float)qmax;
    if (level < -(float)qmax) level = -(float)qmax;
    return (uint32_t)((int)level + qmax);
}

int dz_quantize_pack(const float *src, size_t rows, size_t cols, int bits, int granularity,
                     float *scales, size_t scales_count, uint8_t *packed, size_t packed_size) {
    size_t need_scales = 0, need_bytes = 0;
    if (!src || !scales || !packed || rows == 0 || cols == 0 || bits < 2 || bits > 16 ||
        rows > SIZE_MAX / cols ||
        dz_quantized_scale_count(rows, cols, granularity, &need_scales) != 0 ||
        dz_quantized_packed_size(rows * cols, bits, &need_bytes) != 0 ||
        scales_count != need_scales || packed_size != need_bytes) return -1;
    const size_t total = rows * cols;
    const int qmax = (1 << (bits - 1)) - 1;
    memset(scales, 0, scales_count * sizeof(float));
    memset(packed, 0, packed_size);

    /* pass 1: per-group peak |w| (a max: independent of visiting order) */
    for (size_t i = 0; i < total; i++)
        if (!finite_bits(src[i])) return -1;
    if (granularity == DZ_GRAN_COLUMN) {
        for (size_t r = 0; r < rows; r++) {
            const float *row = src + r * cols;
            for (size_t c = 0; c < cols; c++) {
                float m = fabsf(row[c]);
                if (m > scales[c]) scales[c] = m;
            }
        }
    } else {
        for (size_t i = 0; i < total; i++) {
            size_t g = granularity == DZ_GRAN_ROW ? i / cols : 0;
            float m = fabsf(src[i]);
            if (m > scales[g]) scales[g] = m;
        }
    }

    /* pass 2: codes, LSB-first (src/core/quantize.c:213-221,257-264) */
    if (bits == 8) {
        for (size_t r = 0; r < rows; r++)
            for (size_t c = 0; c < cols; c++) {
                size_t i = r * cols + c;
                float peak = scales[granularity == DZ_GRAN_COLUMN ? c : granularity == DZ_GRAN_ROW ? r : 0];
                packed[i] = (uint8_t)quant_code(src[i], peak, qmax);
            }
    } else if (bits == 4) {
        for (size_t r = 0; r < rows; r++)
            for (size_t c = 0; c < cols; c++) {
                size_t i = r * cols + c;
                float peak = scales[granularity == DZ_GRAN_COLUMN ? c : granularity == DZ_GRAN_ROW ? r : 0];
                uint32_t code = quant_code(src[i], peak, qmax);
                packed[i >> 1] |= (uint8_t)(code << ((i & 1u) * 4));
            }
    } else {
        for (size_t i = 0; i < total; i++) {
            size_t g = granularity == DZ_GRAN_COLUMN ? i % cols : granularity == DZ_GRAN_ROW ? i / cols : 0;
            uint32_t code = quant_code(src[i], scales[g], qmax);
            size_t bit0 = i * (size_t)bits;
            for (int b = 0; b < bits; b++)
                if (code & (UINT32_C(1) << b))
                    packed[(bit0 + (size_t)b) >> 3] |= (uint8_t)(1u << ((bit0 + (size_t)b) & 7u));
        }
    }

    /* scale = peak / qmax, a true division (src/core/quantize.c:265-267; the
     * reference compiles its quantizer without -ffast-math, src/Makefile:
     * 259-268) */
    for (size_t g = 0; g < scales_count; g++)
        if (scales[g] > 0.0f) scales[g] = scales[g] / (float)qmax;
    return 0;
}

/* One group of quantize_dequantize_into (quantize_group, src/core/
 * quantize.c:54-116): values src[i * stride], i < count. The original is read
 * before the store so the in-place form measures against it. */
static void qdq_group(const float *src, float *dst, size_t count, size_t stride, int qmax, double *sse,
                      double *sso, float *max_abs, size_t *clipped, unsigned char *seen) {
    float peak = 0.0f;
    for (size_t i = 0; i < count; i++) {
        const float m = fabsf(src[i * stride]);
        if (m > peak) peak = m;
    }
    if (!(peak > 0.0f)) {   /* nothing to scale: copied through, the zero level used */
        for (size_t i = 0; i < count; i++) dst[i * stride] = src[i * stride];
        seen[qmax] = 1;
        return;
    }
    const float scale = peak / (float)qmax;
    const float inverse = (float)qmax / peak;
    for (size_t i = 0; i < count; i++) {
        const float original = src[i * stride];
        float level = round_half_away(original * inverse);
        if (level > (float)qmax) level = (float)qmax;
        if (level < -(float)qmax) level = -(float)qmax;
        const int index = (int)level;
        if (index == qmax || index == -qmax) (*clipped)++;
        seen[index + qmax] = 1;
        const float rec = scale * level;
        dst[i * stride] = rec;
        const double diff = (double)original - (double)rec;
        *sse += diff * diff;
        *sso += (double)original * (double)original;
        const float a = fabsf((float)diff);
        if (a > *max_abs) *max_abs = a;
    }
}

int dz_quantize_dequantize_into(const float *src, float *dst, size_t rows, size_t cols, int bits,
                                int granularity, dz_quant_error_t *error_out) {
    if (!src || !dst || rows == 0 || cols == 0 || bits < 2 || bits > 16 || !valid_granularity(granularity))
        return -1;
    const int qmax = (1 << (bits - 1)) - 1;
    const size_t total = rows * cols, levels = (size_t)(2 * qmax + 1);
    unsigned char seen[1 << 16];
    memset(seen, 0, levels);
    double sse = 0.0, sso = 0.0;
    float max_abs = 0.0f;
    size_t clipped = 0;
    if (granularity == DZ_GRAN_TENSOR) {
        qdq_group(src, dst, total, 1, qmax, &sse, &sso, &max_abs, &clipped, seen);
    } else if (granularity == DZ_GRAN_ROW) {
        for (size_t r = 0; r < rows; r++)
            qdq_group(src + r * cols, dst + r * cols, cols, 1, qmax, &sse, &sso, &max_abs, &clipped, seen);
    } else {
        for (size_t c = 0; c < cols; c++)
            qdq_group(src + c, dst + c, rows, cols, qmax, &sse, &sso, &max_abs, &clipped, seen);
    }
    if (error_out) {
        memset(error_out, 0, sizeof(*error_out));
        error_out->count = total;
        error_out->max_abs_error = max_abs;
        error_out->rms_error = sqrt(sse / (double)total);
        error_out->original_rms = sqrt(sso / (double)total);
        error_out->rms_relative = error_out->original_rms > 0.0 ? error_out->rms_error / error_out->original_rms : 0.0;
        error_out->clipped = clipped;
        size_t used = 0;
        for (size_t i = 0; i < levels; i++) used += seen[i] ? 1u : 0u;
        error_out->levels_used = used;
    }
    return 0;
}

int dz_quantize_dequantize(float *values, size_t rows, size_t cols, int bits, int granularity,
                           dz_quant_error_t *error_out) {
    return dz_quantize_dequantize_into(values, values, rows, cols, bits, granularity, error_out);
}

static uint32_t code_at(const uint8_t *packed, size_t idx, int bits) {
    if (bits == 8) return packed[idx];
    if (bits == 4) return (uint32_t)((packed[idx >> 1] >> ((idx & 1) * 4)) & 0xF);
    /* other widths: LSB-first bit stream */
    uint32_t v = 0;
    for (int b = 0; b < bits; b++) {
        const size_t bit = idx * (size_t)bits + (size_t)b;
        v |= (uint32_t)((packed[bit >> 3] >> (bit & 7)) & 1) << b;
    }
    return v;
}

static void code_put(uint8_t *packed, size_t idx, int bits, uint32_t v) {
    if (bits == 8) {
        packed[idx] = (uint8_t)v;
        return;
    }
    for (int b = 0; b < bits; b++) {
        const size_t bit = idx * (size_t)bits + (size_t)b;
        if ((v >> b) & 1) packed[bit >> 3] |= (uint8_t)(1u << (bit & 7));
    }
}

int dz_quantized_slice(const float *scales, size_t scales_count, const uint8_t *packed, size_t packed_size,
                       size_t rows, size_t cols, int bits, int granularity, int axis, size_t start,
                       size_t count, float *scales_out, uint8_t *packed_out) {
    size_t ns = 0, nb = 0, ns2 = 0, nb2 = 0;
    if (!scales || !packed || !scales_out || !packed_out || (axis != 0 && axis != 1) || count == 0 ||
        bits < 2 || bits > 16)
        return DZ_E_INVALID;
    const size_t lim = axis == 0 ? rows : cols;
    if (start > lim || count > lim - start) return DZ_E_INVALID;
    if (dz_quantized_scale_count(rows, cols, granularity, &ns) || dz_quantized_packed_size(rows * cols, bits, &nb) ||
        ns != scales_count || nb != packed_size)
        return DZ_E_INVALID;
    const size_t r2 = axis == 0 ? count : rows, c2 = axis == 0 ? cols : count;
    if (dz_quantized_scale_count(r2, c2, granularity, &ns2) || dz_quantized_packed_size(r2 * c2, bits, &nb2))
        return DZ_E_INVALID;
    memset(packed_out, 0, nb2);
    for (size_t r = 0; r < r2; r++)
        for (size_t c = 0; c < c2; c++) {
            const size_t sr = axis == 0 ? start + r : r, sc = axis == 0 ? c : start + c;
            code_put(packed_out, r * c2 + c, bits, code_at(packed, sr * cols + sc, bits));
        }
    if (granularity == DZ_GRAN_COLUMN) {
        for (size_t c = 0; c < c2; c++) scales_out[c] = scales[axis == 1 ? start + c : c];
    } else if (granularity == DZ_GRAN_ROW) {
        for (size_t r = 0; r < r2; r++) scales_out[r] = scales[axis == 0 ? start + r : r];
    } else {
        scales_out[0] = scales[0];
    }
    return DZ_OK;
}

int dz_quantize_unpack(const float *scales, size_t scales_count, const uint8_t *packed,
                       size_t packed_size, size_t rows, size_t cols, int bits, int granularity,
                       float *dst) {
    size_t need_scales = 0, need_bytes = 0;
    if (!scales || !packed || !dst || rows == 0 || cols == 0 || rows > SIZE_MAX / cols ||
        bits < 2 || bits > 16 ||
        dz_quantized_scale_count(rows, cols, granularity, &need_scales) != 0 ||
        dz_quantized_packed_size(rows * cols, bits, &need_bytes) != 0 ||
        scales_count != need_scales || packed_size != need_bytes) return -1;
    for (size_t g = 0; g < scales_count; g++)
        if (!finite_bits(scales[g]) || scales[g] < 0.0f) return -1;
    const size_t total = rows * cols;
    const int qmax = (1 << (bits - 1)) - 1;
    const uint32_t largest = (uint32_t)(2 * qmax);
    for (size_t i = 0; i < total; i++) {
        uint32_t code;
        if (bits == 8) {
            code = packed[i];
        } else if (bits == 4) {
            code = (packed[i >> 1] >> ((i & 1u) * 4)) & 0xFu;
        } else {
            code = 0;
            size_t bit0 = i * (size_t)bits;
            for (int b = 0; b < bits; b++)
                if (packed[(bit0 + (size_t)b) >> 3] & (1u << ((bit0 + (size_t)b) & 7u)))
                    code |= UINT32_C(1) << b;
        }
        if (code > largest) return -1;
        size_t g = granularity == DZ_GRAN_COLUMN ? i % cols : granularity == DZ_GRAN_ROW ? i / cols : 0;
        dst[i] = scales[g] * (float)((int)code - qmax);
    }
    size_t used = total * (size_t)bits;
    if (used % 8 != 0) {
        uint8_t mask = (uint8_t)(0xFFu << (used % 8));
        if (packed[packed_size - 1] & mask) return -1;
    }
    return 0;
}

/* Canonical-code check without decoding (the part of quantize_unpack the
 * loader needs): no code above 2*qmax, zero padding bits. */
static int codes_canonical(const uint8_t *packed, size_t packed_size, size_t total, int bits) {
    const int qmax = (1 << (bits - 1)) - 1;
    if (bits == 8) {
        uint8_t any255 = 0;
        for (size_t i = 0; i < total; i++) any255 |= (uint8_t)(packed[i] == 0xFF);
        return !any255;
    }
    if (bits == 4) {
        size_t full = total / 2;
        uint8_t bad = 0;
        for (size_t i = 0; i < full; i++) {
            uint8_t b = packed[i];
            bad |= (uint8_t)(((b & 0x0F) == 0x0F) | ((b >> 4) == 0x0F));
        }
        if (total & 1u) {
            uint8_t b = packed[full];
            bad |= (uint8_t)(((b & 0x0F) == 0x0F) | ((b >> 4) != 0));
        }
        return !bad;
    }
    for (size_t i = 0; i < total; i++) {
        uint32_t code = 0;
        size_t bit0 = i * (size_t)bits;
        for (int b = 0; b < bits; b++)
            if (packed[(bit0 + (size_t)b) >> 3] & (1u << ((bit0 + (size_t)b) & 7u)))
                code |= UINT32_C(1) << b;
        if (code > (uint32_t)(2 * qmax)) return 0;
    }
    size_t used = total * (size_t)bits;
    if (used % 8 != 0) {
        uint8_t mask = (uint8_t)(0xFFu << (used % 8));
        if (packed[packed_size - 1] & mask) return 0;
    }
    return 1;
}

/* ----------------------------------------------------------- positions */

int dz_positional_encoding(float *out, size_t rows, size_t dim) {
    if (!out || dim == 0) return -1;
    float *scales = malloc(dim * sizeof(float));
    if (!scales) return -1;
    /* 1 / 10000^(2i/d). The reference source writes 1.0f / powf(10000.0f, x);
     * its -ffast-math build folds that into expf(-x * ln 10000), and the
     * tables it runs with hold that result, so this computes the same form. */
    const float ln_base = logf(10000.0f);
    for (size_t i = 0; i < dim; i++)
        scales[i] = expf(-((2.0f * (float)i) / (float)dim) * ln_base);
    for (size_t pos = 0; pos < rows; pos++)
        for (size_t i = 0; i < dim; i++) {
            float angle = (float)pos * scales[i];
            out[pos * dim + i] = (i % 2 == 0) ? sinf(angle) : cosf(angle);
        }
    free(scales);
    return 0;
}

/* --------------------------------------------------------- model layout */

/* Architecture bits (src/include/core/model_types.h:26-36). */
#define ARCH_TIED 1u
#define ARCH_ROPE 2u
#define ARCH_RMSNORM 4u
#define ARCH_GELU 8u
#define ARCH_SWIGLU 16u
#define ARCH_ALL 31u

/* A supported combination: known bits, GELU and SwiGLU not both
 * (src/core/bundle.c:142-144). */
static int arch_valid(uint32_t f) { return (f & ~ARCH_ALL) == 0 && !((f & ARCH_GELU) && (f & ARCH_SWIGLU)); }

size_t dz_model_param_count(const dz_model_desc_t *d) {
    if (!d || !arch_valid(d->architecture_flags)) return 0;
    const uint32_t f = d->architecture_flags;
    size_t D = d->embedding_dim, V = d->vocab_size;
    size_t per = ((f & ARCH_SWIGLU) ? 16 : 12) * D * D + (((f & ARCH_RMSNORM) ? 7 : 9) + ((f & ARCH_SWIGLU) ? 4 : 0)) * D;
    return ((f & ARCH_TIED) ? 1 : 2) * V * D + V + d->num_layers * per;
}

static void put_layout(dz_tensor_blob_t *out, size_t cap, size_t *n, uint32_t kind, size_t r,
                       size_t c) {
    if (out && *n < cap) {
        memset(&out[*n], 0, sizeof(out[*n]));
        out[*n].kind = kind;
        out[*n].rows = r;
        out[*n].cols = c;
    }
    (*n)++;
}

/* src/core/model_params.c:39-103, default architecture (flags 0). */
size_t dz_model_tensor_layout(const dz_model_desc_t *d, dz_tensor_blob_t *out, size_t cap) {
    if (!d || !arch_valid(d->architecture_flags)) return 0;
    const uint32_t f = d->architecture_flags;
    const int tied = (f & ARCH_TIED) != 0, rms = (f & ARCH_RMSNORM) != 0, swiglu = (f & ARCH_SWIGLU) != 0;
    size_t n = 0, D = d->embedding_dim, V = d->vocab_size, F = 4 * D;
    put_layout(out, cap, &n, DZ_KIND_EMBEDDING, V, D);
    if (!tied) put_layout(out, cap, &n, DZ_KIND_PROJECTION, D, V);
    put_layout(out, cap, &n, DZ_KIND_BIAS, 1, V);
    for (size_t l = 0; l < d->num_layers; l++) {
        for (int w = 0; w < 4; w++) put_layout(out, cap, &n, DZ_KIND_PROJECTION, D, D);
        put_layout(out, cap, &n, DZ_KIND_NORM, 1, D);
        if (!rms) put_layout(out, cap, &n, DZ_KIND_NORM, 1, D);
        put_layout(out, cap, &n, DZ_KIND_PROJECTION, D, F);
        put_layout(out, cap, &n, DZ_KIND_BIAS, 1, F);
        if (swiglu) {
            put_layout(out, cap, &n, DZ_KIND_PROJECTION, D, F);
            put_layout(out, cap, &n, DZ_KIND_BIAS, 1, F);
        }
        put_layout(out, cap, &n, DZ_KIND_PROJECTION, F, D);
        put_layout(out, cap, &n, DZ_KIND_BIAS, 1, D);
        put_layout(out, cap, &n, DZ_KIND_NORM, 1, D);
        if (!rms) put_layout(out, cap, &n, DZ_KIND_NORM, 1, D);
    }
    return n;
}

/* ------------------------------------------------------------- bundles */

#define HDR_V1 152u
#define HDR_V2 184u
#define HDR_V3 192u
#define RECORD 32u

static void put_u32(uint8_t *b, uint32_t v) { for (int i = 0; i < 4; i++) b[i] = (uint8_t)(v >> (8 * i)); }
static void put_u64(uint8_t *b, uint64_t v) { for (int i = 0; i < 8; i++) b[i] = (uint8_t)(v >> (8 * i)); }
static uint32_t get_u32(const uint8_t *b) {
    uint32_t v = 0;
    for (int i = 0; i < 4; i++) v |= (uint32_t)b[i] << (8 * i);
    return v;
}
static uint64_t get_u64(const uint8_t *b) {
    uint64_t v = 0;
    for (int i = 0; i < 8; i++) v |= (uint64_t)b[i] << (8 * i);
    return v;
}

static int mul_ok(uint64_t a, uint64_t b, uint64_t *out) {
    if (a != 0 && b > UINT64_MAX / a) return 0;
    *out = a * b;
    return 1;
}
static int add_ok(uint64_t a, uint64_t b, uint64_t *out) {
    if (b > UINT64_MAX - a) return 0;
    *out = a + b;
    return 1;
}

/* bundle_shape_valid, src/core/bundle.c:136-170, default architecture. */
static int shape_valid(const uint64_t dims[6], uint32_t flags) {
    uint64_t V = dims[0], D = dims[1], H = dims[2], Lr = dims[3], T = dims[4], total = dims[5];
    uint64_t d2, ve, g, sq, lin, lp, all, comp, tt, att, lim;
    if (!arch_valid(flags) || V == 0 || D == 0 || H == 0 || Lr == 0 || T == 0 || D % H != 0) return 0;
    const uint64_t tied = (flags & ARCH_TIED) ? 1 : 2, sqm = (flags & ARCH_SWIGLU) ? 16 : 12;
    const uint64_t linm = ((flags & ARCH_RMSNORM) ? 7 : 9) + ((flags & ARCH_SWIGLU) ? 4 : 0);
    if (!mul_ok(D, D, &d2) || !mul_ok(V, D, &ve) || !mul_ok(ve, tied, &g) || !add_ok(g, V, &g) ||
        !mul_ok(d2, sqm, &sq) || !mul_ok(D, linm, &lin) || !add_ok(sq, lin, &lp) ||
        !mul_ok(Lr, lp, &all) || !add_ok(g, all, &comp) || comp != total ||
        !mul_ok(T, T, &tt) || !mul_ok(H, tt, &att) || !mul_ok(total, 64, &lim) || att > lim)
        return 0;
    return 1;
}

struct dz_bundle {
    uint8_t *map;
    size_t map_size;
    dz_model_desc_t desc;
    dz_bundle_info_t info;
    size_t n_tensors;
    dz_tensor_blob_t *tensors;
    float *scale_store; /* aligned copies of the stored scales */
    const uint8_t *tokenizer;
    size_t tokenizer_size;
};

void dz_bundle_close(dz_bundle_t *b) {
    if (!b) return;
    if (b->map) munmap(b->map, b->map_size);
    free(b->tensors);
    free(b->scale_store);
    free(b);
}

int dz_bundle_open(const char *path, dz_bundle_t **out) {
    if (!path || !out) return DZ_E_INVALID;
    *out = NULL;
    int fd = open(path, O_RDONLY);
    if (fd < 0) return DZ_E_IO;
    struct stat st;
    if (fstat(fd, &st) != 0 || st.st_size < 24) {
        close(fd);
        return st.st_size < 8 ? DZ_E_NOT_BUNDLE : DZ_E_FORMAT;
    }
    size_t size = (size_t)st.st_size;
    uint8_t *map = mmap(NULL, size, PROT_READ, MAP_PRIVATE, fd, 0);
    close(fd);
    if (map == MAP_FAILED) return DZ_E_IO;
    dz_bundle_t *b = calloc(1, sizeof(*b));
    if (!b) { munmap(map, size); return DZ_E_NOMEM; }
    b->map = map;
    b->map_size = size;
    int rc = DZ_E_FORMAT;

    if (memcmp(map, "DRNZBNDL", 8) != 0) { rc = DZ_E_NOT_BUNDLE; goto fail; }
    uint32_t version = get_u32(map + 8), numeric = get_u32(map + 16), hsize = get_u32(map + 20);
    int is_v3 = version == 3 && hsize == HDR_V3;
    int is_float = numeric == 1 && ((version == 1 && hsize == HDR_V1) || is_v3);
    int is_quant = numeric == 2 && ((version == 2 && hsize == HDR_V2) || is_v3);
    if (!is_float && !is_quant) { rc = DZ_E_UNSUPPORTED; goto fail; }
    if (size < hsize) goto fail;
    {
        uint8_t header[HDR_V3];
        memcpy(header, map, hsize);
        uint64_t stored = (uint64_t)get_u32(header + 76) | ((uint64_t)get_u32(header + 84) << 32);
        memset(header + 76, 0, 4);
        memset(header + 84, 0, 4);
        if (dz_fnv1a(DZ_FNV_OFFSET, header, hsize) != stored) { rc = DZ_E_CHECKSUM; goto fail; }
    }
    if (get_u32(map + 12) != 0x01020304u) { rc = DZ_E_UNSUPPORTED; goto fail; }

    uint64_t dims[6];
    for (int i = 0; i < 6; i++) dims[i] = get_u64(map + 24 + 8 * i);
    uint64_t train_window = get_u64(map + 88);
    uint64_t weight_bytes = get_u64(map + 120), tok_bytes = get_u64(map + 128);
    uint64_t weight_sum = get_u64(map + 136), tok_sum = get_u64(map + 144);
    uint32_t arch = is_v3 ? get_u32(map + 184) : 0;
    if (is_v3 && (arch == 0 || get_u32(map + 188) != 0)) goto fail;
    if (!arch_valid(arch)) { rc = DZ_E_UNSUPPORTED; goto fail; }
    if (!shape_valid(dims, arch) || tok_bytes < 24 || train_window == 0 ||
        train_window > dims[4] || (is_float && weight_bytes != dims[5] * 4)) goto fail;

    b->info.format_version = version;
    b->info.numeric = numeric;
    b->info.train_window = train_window;
    b->info.seed = get_u64(map + 96);
    b->info.input_fingerprint = get_u64(map + 104);
    b->info.input_bytes = get_u64(map + 112);
    b->info.training_steps = get_u32(map + 72);
    b->info.loss_bits = get_u32(map + 80);
    b->info.total_param_count = dims[5];
    int bits = 0, gran = DZ_GRAN_COLUMN;
    uint32_t policy = 0, stored_count = 0;
    if (is_quant) {
        bits = (int)get_u32(map + 152);
        gran = (int)get_u32(map + 156);
        policy = get_u32(map + 160);
        stored_count = get_u32(map + 164);
        b->info.values_quantized = get_u64(map + 168);
        b->info.scales_stored = get_u64(map + 176);
        if ((policy & ~3u) != 0 || bits < 2 || bits > 16 || !valid_granularity(gran) ||
            stored_count == 0 || b->info.values_quantized > dims[5]) goto fail;
    }
    b->info.bits = bits;
    b->info.granularity = gran;
    b->info.policy_flags = policy;

    uint64_t expect = 0;
    if (!add_ok(hsize, weight_bytes, &expect) || !add_ok(expect, tok_bytes, &expect) ||
        !add_ok(expect, 8, &expect) || expect != size) goto fail;
    if (dz_fnv1a(DZ_FNV_OFFSET, map + hsize, (size_t)weight_bytes) != weight_sum) {
        rc = DZ_E_CHECKSUM;
        goto fail;
    }

    b->desc.vocab_size = (size_t)dims[0];
    b->desc.embedding_dim = (size_t)dims[1];
    b->desc.num_heads = (size_t)dims[2];
    b->desc.num_layers = (size_t)dims[3];
    b->desc.max_seq_len = (size_t)dims[4];
    b->desc.architecture_flags = arch;
    size_t nt = dz_model_tensor_layout(&b->desc, NULL, 0);
    b->tensors = calloc(nt, sizeof(dz_tensor_blob_t));
    if (!b->tensors) { rc = DZ_E_NOMEM; goto fail; }
    dz_model_tensor_layout(&b->desc, b->tensors, nt);
    b->n_tensors = nt;

    const uint8_t *p = map + hsize;
    const uint8_t *end = p + weight_bytes;
    if (is_float) {
        /* v1 / v3 float: the flat params vector, no records */
        const uint8_t *q = p;
        for (size_t t = 0; t < nt; t++) {
            dz_tensor_blob_t *tb = &b->tensors[t];
            tb->f32 = (const float *)q;
            q += tb->rows * tb->cols * 4;
        }
    } else {
        if (stored_count != nt) goto fail;
        size_t total_scales = 0;
        for (size_t t = 0; t < nt; t++) {
            size_t ns = 0;
            dz_quantized_scale_count(b->tensors[t].rows, b->tensors[t].cols, gran, &ns);
            int included = b->tensors[t].kind == DZ_KIND_PROJECTION ||
                           (b->tensors[t].kind == DZ_KIND_EMBEDDING && (policy & 1u)) ||
                           ((b->tensors[t].kind == DZ_KIND_BIAS || b->tensors[t].kind == DZ_KIND_NORM) &&
                            (policy & 2u));
            if (included) total_scales += ns;
        }
        b->scale_store = malloc((total_scales ? total_scales : 1) * sizeof(float));
        if (!b->scale_store) { rc = DZ_E_NOMEM; goto fail; }
        float *sc = b->scale_store;
        uint64_t seen_values = 0, seen_scales = 0;
        for (size_t t = 0; t < nt; t++) {
            dz_tensor_blob_t *tb = &b->tensors[t];
            if ((size_t)(end - p) < RECORD) goto fail;
            int included = tb->kind == DZ_KIND_PROJECTION ||
                           (tb->kind == DZ_KIND_EMBEDDING && (policy & 1u)) ||
                           ((tb->kind == DZ_KIND_BIAS || tb->kind == DZ_KIND_NORM) && (policy & 2u));
            if (get_u32(p) != t || get_u32(p + 4) != tb->kind || get_u64(p + 8) != tb->rows ||
                get_u64(p + 16) != tb->cols || get_u32(p + 28) != 0 ||
                get_u32(p + 24) != (included ? 2u : 1u)) goto fail;
            p += RECORD;
            size_t count = tb->rows * tb->cols;
            if (!included) {
                if ((size_t)(end - p) < count * 4) goto fail;
                tb->f32 = (const float *)p;
                p += count * 4;
                continue;
            }
            size_t ns = 0, nb = 0;
            dz_quantized_scale_count(tb->rows, tb->cols, gran, &ns);
            dz_quantized_packed_size(count, bits, &nb);
            if ((size_t)(end - p) < ns * 4 + nb) goto fail;
            for (size_t s = 0; s < ns; s++) {
                uint32_t u = get_u32(p + 4 * s);
                memcpy(&sc[s], &u, 4);
                if (!finite_bits(sc[s]) || sc[s] < 0.0f) goto fail;
            }
            p += ns * 4;
            if (!codes_canonical(p, nb, count, bits)) goto fail;
            tb->bits = bits;
            tb->granularity = gran;
            tb->scales = sc;
            tb->scale_count = ns;
            tb->packed = p;
            tb->packed_size = nb;
            sc += ns;
            p += nb;
            seen_values += count;
            seen_scales += ns;
        }
        if (p != end || seen_values != b->info.values_quantized ||
            seen_scales != b->info.scales_stored) goto fail;
    }

    /* tokenizer payload + footer (src/core/bundle.c:777-796) */
    b->tokenizer = map + hsize + weight_bytes;
    b->tokenizer_size = (size_t)tok_bytes;
    if (memcmp(b->tokenizer + tok_bytes, "DRNZDONE", 8) != 0) goto fail;
    if (dz_fnv1a(DZ_FNV_OFFSET, b->tokenizer, b->tokenizer_size) != tok_sum) {
        rc = DZ_E_CHECKSUM;
        goto fail;
    }
    {
        /* portable header: magic "DRNZBPP2" (32 B header) or v1 (24 B);
         * max_vocab must equal the model's vocabulary */
        const uint8_t *tk = b->tokenizer;
        uint64_t max_vocab;
        if (tok_bytes >= 32 && memcmp(tk, "DRNZBPP2", 8) == 0) max_vocab = get_u64(tk + 8);
        else max_vocab = get_u64(tk);
        if (max_vocab != dims[0]) goto fail;
    }
    *out = b;
    return DZ_OK;
fail:
    dz_bundle_close(b);
    return rc;
}

int dz_bundle_desc(const dz_bundle_t *b, dz_model_desc_t *out) {
    if (!b || !out) return DZ_E_INVALID;
    *out = b->desc;
    return DZ_OK;
}

int dz_bundle_info(const dz_bundle_t *b, dz_bundle_info_t *out) {
    if (!b || !out) return DZ_E_INVALID;
    *out = b->info;
    return DZ_OK;
}

size_t dz_bundle_tensor_count(const dz_bundle_t *b) { return b ? b->n_tensors : 0; }

int dz_bundle_tensor(const dz_bundle_t *b, size_t i, dz_tensor_blob_t *out) {
    if (!b || !out || i >= b->n_tensors) return DZ_E_INVALID;
    *out = b->tensors[i];
    return DZ_OK;
}

const dz_tensor_blob_t *dz_bundle_tensors(const dz_bundle_t *b) { return b ? b->tensors : NULL; }

const uint8_t *dz_bundle_tokenizer(const dz_bundle_t *b, size_t *size) {
    if (!b) return NULL;
    if (size) *size = b->tokenizer_size;
    return b->tokenizer;
}

int dz_tokenizer_minimal(uint64_t max_vocab, uint8_t out[32]) {
    if (!out || max_vocab < 260 || max_vocab > 1048576) return DZ_E_INVALID;
    memcpy(out, "DRNZBPP2", 8);
    put_u64(out + 8, max_vocab);
    put_u64(out + 16, 260); /* byte tokens + PAD/UNK/BOS/EOS, no merges */
    put_u32(out + 24, 1);   /* frozen */
    put_u32(out + 28, 1);   /* special tokens */
    return DZ_OK;
}

typedef struct {
    FILE *f;
    uint64_t sum;
    int ok;
} sink_t;

static void sink(sink_t *s, const void *data, size_t n) {
    if (!s->ok) return;
    if (fwrite(data, 1, n, s->f) != n) s->ok = 0;
    s->sum = dz_fnv1a(s->sum, data, n);
}

int dz_bundle_save_quantized(const char *path, const dz_model_desc_t *desc, const float *params,
                             int bits, int granularity, const dz_bundle_meta_t *meta,
                             const uint8_t *tokenizer, size_t tokenizer_size) {
    if (!path || !desc || !params || !meta || !tokenizer || tokenizer_size < 24 || bits < 2 ||
        bits > 16 || !valid_granularity(granularity) || !arch_valid(desc->architecture_flags))
        return DZ_E_INVALID;
    /* v2 for the reference architecture, v3 (192-byte header, flags at 184)
     * for any other (src/core/bundle.c:357-360, 475-476) */
    const uint32_t arch = desc->architecture_flags;
    const uint32_t hdr = arch ? HDR_V3 : HDR_V2;
    uint64_t dims[6] = {desc->vocab_size, desc->embedding_dim, desc->num_heads, desc->num_layers,
                        desc->max_seq_len, dz_model_param_count(desc)};
    if (!shape_valid(dims, arch) || meta->train_window == 0 || meta->train_window > desc->max_seq_len)
        return DZ_E_INVALID;
    size_t nt = dz_model_tensor_layout(desc, NULL, 0);
    dz_tensor_blob_t *lay = calloc(nt, sizeof(*lay));
    if (!lay) return DZ_E_NOMEM;
    dz_model_tensor_layout(desc, lay, nt);

    uint64_t weight_bytes = 0, values_q = 0, scales_q = 0;
    for (size_t t = 0; t < nt; t++) {
        size_t count = lay[t].rows * lay[t].cols;
        weight_bytes += RECORD;
        if (lay[t].kind == DZ_KIND_PROJECTION) {
            size_t ns = 0, nb = 0;
            dz_quantized_scale_count(lay[t].rows, lay[t].cols, granularity, &ns);
            dz_quantized_packed_size(count, bits, &nb);
            weight_bytes += 4 * ns + nb;
            values_q += count;
            scales_q += ns;
        } else {
            weight_bytes += 4 * (uint64_t)count;
        }
    }

    size_t plen = strlen(path);
    char *tmp = malloc(plen + 32);
    if (!tmp) { free(lay); return DZ_E_NOMEM; }
    snprintf(tmp, plen + 32, "%s.tmp.%ld", path, (long)getpid());
    FILE *f = fopen(tmp, "wb");
    if (!f) { free(lay); free(tmp); return DZ_E_IO; }
    uint8_t header[HDR_V3];
    memset(header, 0, sizeof(header));
    sink_t s = {f, DZ_FNV_OFFSET, 1};
    if (fwrite(header, 1, hdr, f) != hdr) s.ok = 0;
    int rc = DZ_OK;
    const float *cursor = params;
    for (size_t t = 0; t < nt && s.ok; t++) {
        size_t count = lay[t].rows * lay[t].cols;
        int included = lay[t].kind == DZ_KIND_PROJECTION;
        uint8_t rec[RECORD];
        memset(rec, 0, sizeof(rec));
        put_u32(rec, (uint32_t)t);
        put_u32(rec + 4, lay[t].kind);
        put_u64(rec + 8, lay[t].rows);
        put_u64(rec + 16, lay[t].cols);
        put_u32(rec + 24, included ? 2u : 1u);
        sink(&s, rec, RECORD);
        if (included) {
            size_t ns = 0, nb = 0;
            dz_quantized_scale_count(lay[t].rows, lay[t].cols, granularity, &ns);
            dz_quantized_packed_size(count, bits, &nb);
            float *sc = malloc(ns * sizeof(float));
            uint8_t *pk = malloc(nb);
            if (!sc || !pk) {
                rc = DZ_E_NOMEM;
                s.ok = 0;
            } else if (dz_quantize_pack(cursor, lay[t].rows, lay[t].cols, bits, granularity, sc, ns,
                                        pk, nb) != 0) {
                rc = DZ_E_INVALID;
                s.ok = 0;
            } else {
                uint8_t *le = malloc(ns * 4);
                if (!le) { rc = DZ_E_NOMEM; s.ok = 0; }
                else {
                    for (size_t i = 0; i < ns; i++) {
                        uint32_t u;
                        memcpy(&u, &sc[i], 4);
                        put_u32(le + 4 * i, u);
                    }
                    sink(&s, le, ns * 4);
                    free(le);
                }
                sink(&s, pk, nb);
            }
            free(sc);
            free(pk);
        } else {
            uint8_t *le = malloc(count * 4);
            if (!le) { rc = DZ_E_NOMEM; s.ok = 0; }
            else {
                for (size_t i = 0; i < count; i++) {
                    uint32_t u;
                    memcpy(&u, &cursor[i], 4);
                    put_u32(le + 4 * i, u);
                }
                sink(&s, le, count * 4);
                free(le);
            }
        }
        cursor += count;
    }
    uint64_t weight_sum = s.sum;
    if (s.ok && (fwrite(tokenizer, 1, tokenizer_size, f) != tokenizer_size ||
                 fwrite("DRNZDONE", 1, 8, f) != 8)) s.ok = 0;

    memcpy(header, "DRNZBNDL", 8);
    put_u32(header + 8, arch ? 3 : 2);
    put_u32(header + 12, 0x01020304u);
    put_u32(header + 16, 2);
    put_u32(header + 20, hdr);
    for (int i = 0; i < 6; i++) put_u64(header + 24 + 8 * i, dims[i]);
    put_u32(header + 72, meta->training_steps);
    put_u32(header + 80, meta->loss_bits);
    put_u64(header + 88, meta->train_window);
    put_u64(header + 96, meta->seed);
    put_u64(header + 104, meta->input_fingerprint);
    put_u64(header + 112, meta->input_bytes);
    put_u64(header + 120, weight_bytes);
    put_u64(header + 128, tokenizer_size);
    put_u64(header + 136, weight_sum);
    put_u64(header + 144, dz_fnv1a(DZ_FNV_OFFSET, tokenizer, tokenizer_size));
    put_u32(header + 152, (uint32_t)bits);
    put_u32(header + 156, (uint32_t)granularity);
    put_u32(header + 160, 0);
    put_u32(header + 164, (uint32_t)nt);
    put_u64(header + 168, values_q);
    put_u64(header + 176, scales_q);
    if (arch) put_u32(header + 184, arch);
    uint64_t hs = dz_fnv1a(DZ_FNV_OFFSET, header, hdr);
    put_u32(header + 76, (uint32_t)hs);
    put_u32(header + 84, (uint32_t)(hs >> 32));
    if (s.ok && (fseek(f, 0, SEEK_SET) != 0 || fwrite(header, 1, hdr, f) != hdr)) s.ok = 0;
    if (fclose(f) != 0) s.ok = 0;
    if (!s.ok || rename(tmp, path) != 0) {
        remove(tmp);
        if (rc == DZ_OK) rc = DZ_E_IO;
    }
    free(tmp);
    free(lay);
    return rc;
}
