/*
 * The reference-side binding of the device path, as a maintainer would add
 * it, built around the reference's UNCHANGED objects (test infrastructure).
 *
 * `make -C oracle bridge` links the reference's core objects, ref_harness.o
 * and this file into oracle/_ref/libdzref_bridge.so with
 *   -Wl,--wrap=model_forward_token,--wrap=model_kv_cache_init,
 *   --wrap=model_kv_cache_reset,--wrap=model_kv_cache_free
 * so that every call the reference's generation loop makes from another
 * object (src/cli/generation.c:222-306) reaches the __wrap_ functions below.
 * They are the early branch of the integration guide: a model attached to a
 * dz_cuda_model_t runs its decode step on the GPU through
 * dz_cuda_forward_tokens (batch 1), keeping the reference's ring bookkeeping
 * (src/core/transformer.c:765-775) in the host cache; a model without one
 * runs the reference's own code. Nothing of the reference is re-implemented.
 */
#include "core/transformer.h"
#include "dz_cuda.h"
#include "dz_host.h"

#include <stdlib.h>
#include <string.h>

model_errors_t __real_model_forward_token(neural_model_t *model, model_kv_cache_t *cache, uint32_t token_id,
                                          float *output_logits);
model_errors_t __real_model_kv_cache_init(model_kv_cache_t *cache, const neural_model_t *model);
void __real_model_kv_cache_reset(model_kv_cache_t *cache);
void __real_model_kv_cache_free(model_kv_cache_t *cache);

/* attached models and the device caches of live host caches (a handful at
 * most: linear tables) */
#define BR_MAX 64
static struct { const neural_model_t *model; dz_cuda_model_t *dz; } br_models[BR_MAX];
static struct { const model_kv_cache_t *cache; dz_cuda_cache_t *dz; } br_caches[BR_MAX];
static size_t br_forwards;   /* decode steps served by the device */

/* a device model waiting for the next model that starts a sequence
 * (br_attach_next: for handles whose neural_model_t the caller cannot name,
 * such as the public API's opaque dranzer_model_t) */
static dz_cuda_model_t *br_pending;

static int br_bind(const neural_model_t *model, dz_cuda_model_t *dz) {
    for (int i = 0; i < BR_MAX; i++)
        if (!br_models[i].model) {
            br_models[i].model = model;
            br_models[i].dz = dz;
            return 0;
        }
    return DZ_E_NOMEM;
}

static dz_cuda_model_t *br_model_of(const neural_model_t *model) {
    for (int i = 0; i < BR_MAX; i++)
        if (br_models[i].model == model) return br_models[i].dz;
    if (br_pending && br_bind(model, br_pending) == 0) {
        dz_cuda_model_t *dz = br_pending;
        br_pending = NULL;
        return dz;
    }
    return NULL;
}

static dz_cuda_cache_t **br_cache_slot(const model_kv_cache_t *cache) {
    for (int i = 0; i < BR_MAX; i++)
        if (br_caches[i].cache == cache && br_caches[i].dz) return &br_caches[i].dz;
    return NULL;
}

/* The model's bundle reopened with its codes kept (dz_bundle_open) and
 * uploaded to `device`. */
static int br_upload(const char *bundle_path, int device, dz_cuda_model_t **out) {
    dz_bundle_t *b = NULL;
    dz_model_desc_t desc;
    int rc = dz_bundle_open(bundle_path, &b);
    if (rc) return rc;
    rc = dz_bundle_desc(b, &desc);
    if (!rc) rc = dz_cuda_model_create(&desc, dz_bundle_tensors(b), dz_bundle_tensor_count(b), device, out);
    dz_bundle_close(b);
    return rc;
}

/* Attach the device copy of `bundle_path` to `model`. Returns 0 or a DZ_E_*
 * code. */
int br_attach(const neural_model_t *model, const char *bundle_path, int device) {
    dz_cuda_model_t *dz = NULL;
    int rc = br_upload(bundle_path, device, &dz);
    if (rc) return rc;
    if ((rc = br_bind(model, dz))) dz_cuda_model_free(dz);
    return rc;
}

/* Attach it to the next model that starts a sequence on an empty cache. */
int br_attach_next(const char *bundle_path, int device) {
    if (br_pending) return DZ_E_INVALID;
    return br_upload(bundle_path, device, &br_pending);
}

void br_detach(const neural_model_t *model) {
    for (int i = 0; i < BR_MAX; i++)
        if (br_models[i].model == model) {
            dz_cuda_model_free(br_models[i].dz);
            br_models[i].model = NULL;
            br_models[i].dz = NULL;
        }
}

size_t br_device_forwards(void) { return br_forwards; }

/* The device cache of a host cache of an attached model, made on first use
 * while the host cache is empty (a cache initialised before the model was
 * attached gets one at its next sequence); NULL: the CPU path. */
static dz_cuda_cache_t **br_cache_for(const neural_model_t *model, model_kv_cache_t *cache) {
    dz_cuda_cache_t **slot = br_cache_slot(cache);
    if (slot) return slot;
    dz_cuda_model_t *dz = br_model_of(model);
    if (!dz || cache->total_tokens != 0) return NULL;
    for (int i = 0; i < BR_MAX; i++)
        if (!br_caches[i].dz) {
            if (dz_cuda_cache_create(dz, 1, cache->capacity, &br_caches[i].dz) != DZ_OK) {
                br_caches[i].dz = NULL;   /* never fatal: this cache stays on the CPU */
                return NULL;
            }
            br_caches[i].cache = cache;
            return &br_caches[i].dz;
        }
    return NULL;
}

model_errors_t __wrap_model_kv_cache_init(model_kv_cache_t *cache, const neural_model_t *model) {
    model_errors_t rc = __real_model_kv_cache_init(cache, model);
    if (rc == MODEL_SUCCESS) (void)br_cache_for(model, cache);
    return rc;
}

void __wrap_model_kv_cache_reset(model_kv_cache_t *cache) {
    dz_cuda_cache_t **slot = cache ? br_cache_slot(cache) : NULL;
    if (slot) dz_cuda_cache_reset(*slot, NULL);
    __real_model_kv_cache_reset(cache);
}

void __wrap_model_kv_cache_free(model_kv_cache_t *cache) {
    dz_cuda_cache_t **slot = br_cache_slot(cache);
    if (slot) {
        dz_cuda_cache_free(*slot);
        *slot = NULL;
        for (int i = 0; i < BR_MAX; i++)
            if (br_caches[i].cache == cache) br_caches[i].cache = NULL;
    }
    __real_model_kv_cache_free(cache);
}

model_errors_t __wrap_model_forward_token(neural_model_t *model, model_kv_cache_t *cache, uint32_t token_id,
                                          float *output_logits) {
    dz_cuda_cache_t **slot = cache ? br_cache_for(model, cache) : NULL;
    if (slot && output_logits) {
        if (dz_cuda_forward_tokens(*slot, &token_id, output_logits) != DZ_OK) {
            /* before the first token the CPU path takes over (never fatal);
             * later the host cache holds no keys to continue from */
            if (cache->total_tokens != 0) return MODEL_INVALID_INPUT;
            dz_cuda_cache_free(*slot);
            *slot = NULL;
            return __real_model_forward_token(model, cache, token_id, output_logits);
        }
        /* the ring bookkeeping of model_forward_token (transformer.c:765-775) */
        if (cache->length < cache->capacity) {
            cache->length++;
        } else {
            cache->start = (cache->start + 1) % cache->capacity;
        }
        cache->total_tokens++;
        br_forwards++;
        return MODEL_SUCCESS;
    }
    return __real_model_forward_token(model, cache, token_id, output_logits);
}
