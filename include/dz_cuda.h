/*
 * dranzer-b200 CUDA shim: the C ABI the reference's host code binds to run its
 * quantized-weight inference path on a B200. Plain C types only; every
 * function returns DZ_OK (0) or a negative DZ_E_* (dz_types.h), never throws
 * and never prints. dz_cuda_last_error() holds the message of the calling
 * thread's last failure. Handles are not safe for concurrent calls (the
 * reference's rule for its own handles, docs/public-api.md:13-15).
 *
 * Reference interfaces each entry point replaces are cited beside it
 * (paths relative to the DRANZER source tree).
 */
#ifndef DZ_CUDA_H
#define DZ_CUDA_H

#include "dz_types.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct dz_cuda_qmatrix dz_cuda_qmatrix_t;
typedef struct dz_cuda_model dz_cuda_model_t;
typedef struct dz_cuda_cache dz_cuda_cache_t;

/* Token selection, the arguments of sample_next_token
 * (src/include/cli/sampling.h: sample_next_token) plus the ids the generation
 * loop masks to -FLT_MAX before each draw (src/cli/generation.c:31-46 control
 * tokens, :250-254 EOS under a minimum length). */
typedef struct {
    int strategy;            /* 0 greedy, 1 top-k, 2 top-p (sampling_strategy_t) */
    float temperature;
    uint32_t top_k;
    float top_p;
    const uint32_t *masked_ids;
    size_t n_masked;
} dz_sampling_t;

/* 1 when a CUDA device of compute capability 10.x is usable, else 0.
 * Replaces gpu_matmul_available (src/include/backends/gpu/gpu_matmul.h:36). */
int dz_cuda_available(void);

/* Copies the calling thread's last error message (NUL-terminated, truncated to
 * n) and returns its status. Replaces the structured error of gpu_cuda.h
 * (src/include/backends/gpu/gpu_cuda.h:25-36). */
int dz_cuda_last_error(char *buf, size_t n);

/* ---- Standalone quantized weight matrix: quantized_weight_matrix_t
 * (src/include/core/quantized_matmul.h:13-22) resident on a device. The blob is
 * the reference storage form (codes + scales); bits 4 or 8, any granularity. */
int dz_cuda_qmatrix_create(int device, const dz_tensor_blob_t *weights, dz_cuda_qmatrix_t **out);
void dz_cuda_qmatrix_free(dz_cuda_qmatrix_t *matrix);
/* Device bytes of codes + scales the matmul streams per call. */
size_t dz_cuda_qmatrix_bytes(const dz_cuda_qmatrix_t *matrix);
/* quantize_unpack (src/core/quantize.c:272-303) computed on the device:
 * dst[k*n] = scale * (code - qmax). Host destination. */
int dz_cuda_qmatrix_unpack(const dz_cuda_qmatrix_t *matrix, float *dst);
/* The device-resident codes converted back to the reference's packed bytes
 * (host destination of quantized_packed_size bytes) - the layout round trip. */
int dz_cuda_qmatrix_codes(const dz_cuda_qmatrix_t *matrix, uint8_t *packed);

/* C (m x n) = A (m x k) . deq(W), host buffers, synchronous: the contract of
 * matmul_quantized_weight (src/include/core/quantized_matmul.h:36-42,
 * src/core/quantized_matmul.c:253-295); fp32 products and accumulation. */
int dz_cuda_matmul_quantized(const float *A, const dz_cuda_qmatrix_t *weights, float *C,
                             size_t m, size_t k);
/* Same on device buffers, enqueued on `stream` (a cudaStream_t, NULL = legacy
 * default stream), no synchronisation. */
int dz_cuda_matmul_quantized_async(const float *A_dev, const dz_cuda_qmatrix_t *weights,
                                   float *C_dev, size_t m, size_t k, void *stream);

/* Same product as dz_cuda_matmul_quantized_async, for callers that cannot call
 * cudaMalloc when they multiply: hosts that budget all device memory at
 * start-up and hand the library no allocation rights afterwards, or that run
 * it where an allocation could stall or fail mid-step. The async entry point
 * grows a per-matrix scratch
 * buffer with cudaMalloc the first time it sees a larger m; this one allocates
 * nothing and uses a fixed DZ_NOALLOC_SCRATCH_BYTES (8 MiB) array that every
 * GPU which loads the library holds until exit. The call's scratch must fit in
 * it: 16 KB of tensor-core GEMV tile counters plus the largest of the split
 * activations (ceil(m / 2) * 16 * kp bytes, kp = k rounded up to 32 for INT8,
 * 64 for INT4, + 4 * m), the tensor-core limbs (3 * m * k rounded up to 128,
 * + 4 * m) and, for m <= 16, the GEMV's partial sums (up to 148 x 32 KB).
 * That allows m <= 254 at k = 4096; larger calls return DZ_E_INVALID.
 * The first call on a device looks up the array's device address (make that
 * call before any stream capture). All calls on a device share the array, so
 * calls whose work overlaps on the GPU (different streams, no ordering) race;
 * each call zeroes the counters it relies on before its kernels run.
 * The address is kept per device ordinal for the life of the process: after
 * cudaDeviceReset (or any other teardown of the device's primary context) the
 * array can load at another address, so this entry point must not be called
 * on that device again.
 * No counterpart in the reference. */
#define DZ_NOALLOC_SCRATCH_BYTES (8u << 20)
int dz_cuda_matmul_quantized_noalloc(const float *A_dev, const dz_cuda_qmatrix_t *weights, float *C_dev,
                                     size_t m, size_t k, void *stream);

/* ---- Model: the parameters of a v2/v3 bundle kept as codes on the device.
 * `tensors` are the n blobs of model_param_tensors() order
 * (src/core/model_params.c:39-103), as dz_bundle_tensors() returns them; they are
 * copied, the caller keeps ownership. Replaces the fp32 unpack at load
 * (src/core/bundle.c:748) and the per-call weight cache of gpu_matmul
 * (src/backends/gpu/gpu_matmul.c:419-519). Projections must be 4- or 8-bit;
 * other tensors float32 (the default policy). */
int dz_cuda_model_create(const dz_model_desc_t *desc, const dz_tensor_blob_t *tensors, size_t n,
                         int device, dz_cuda_model_t **out);
void dz_cuda_model_free(dz_cuda_model_t *model);
/* Bytes of weights (codes, scales, fp32 tensors) one decode step reads. */
size_t dz_cuda_model_step_bytes(const dz_cuda_model_t *model);

/* ---- KV cache for `batch` independent sequences with ring capacity
 * `capacity` (<= max_seq_len): model_kv_cache_init_with_capacity
 * (src/core/transformer.c:586-645) per sequence. The cache retains its model
 * (dranzer_cache_create semantics, src/include/dranzer.h:103-119). */
int dz_cuda_cache_create(dz_cuda_model_t *model, size_t batch, size_t capacity,
                         dz_cuda_cache_t **out);
void dz_cuda_cache_free(dz_cuda_cache_t *cache);
/* Use `stream` (a cudaStream_t) for all later work on this cache. */
int dz_cuda_cache_set_stream(dz_cuda_cache_t *cache, void *stream);
void *dz_cuda_cache_stream(const dz_cuda_cache_t *cache);
/* model_kv_cache_reset (src/core/transformer.c:651-657) for the sequences
 * whose seq_mask byte is non-zero (NULL: all). */
int dz_cuda_cache_reset(dz_cuda_cache_t *cache, const uint8_t *seq_mask);

/* One model_forward_token (src/core/transformer.c:755-858) for every sequence:
 * token_ids[batch] (host) in, logits_out[batch][vocab] (host) out when not
 * NULL. Synchronous. The early branch a GPU-backed model_forward_token /
 * dranzer_cache_forward (src/api/dranzer.c:260-270) forwards to. */
int dz_cuda_forward_tokens(dz_cuda_cache_t *cache, const uint32_t *token_ids, float *logits_out);

/* sample_next_token on the logits of the last forward (src/cli/sampling.c:179-207)
 * for every sequence, after masking sampling->masked_ids. rng_states[batch]
 * (host, in/out) are dranzer_rng streams; NULL selects greedily as the
 * reference does for a NULL stream. out_ids[batch] host. Synchronous. */
int dz_cuda_select(dz_cuda_cache_t *cache, const dz_sampling_t *sampling, uint64_t *rng_states,
                   uint32_t *out_ids);

/* The generation loop of generation_decode_with_options
 * (src/cli/generation.c:231-295) for every sequence at once, on the device:
 * reset, prefill prompts[batch][prompt_len] token by token, then n_new draws,
 * each followed by a forward of the drawn token except the last. seeds[batch]
 * give the per-sequence streams dranzer_rng_stream(seed, SAMPLING) (NULL:
 * greedy). out_tokens[batch][n_new]. Host buffers, synchronous; the whole loop
 * runs as one CUDA graph. */
int dz_cuda_generate(dz_cuda_cache_t *cache, const uint32_t *prompts, size_t prompt_len,
                     size_t n_new, const dz_sampling_t *sampling, const uint64_t *seeds,
                     uint32_t *out_tokens);
/* Same with device-resident prompts/seeds/out_tokens, enqueued on the cache's
 * stream without synchronisation. */
int dz_cuda_generate_async(dz_cuda_cache_t *cache, const uint32_t *prompts_dev, size_t prompt_len,
                           size_t n_new, const dz_sampling_t *sampling, const uint64_t *seeds_dev,
                           uint32_t *out_tokens_dev);
/* The generation loop's controls beyond token selection, the fields of
 * generation_options_t (src/include/cli/generation.h) that
 * generation_decode_with_options (src/cli/generation.c:198-308) applies per
 * draw: the sign-aware repetition penalty over every id the sequence holds
 * (prompt and generated, :52-72), the tokenizer's unassigned ids masked
 * (ids >= mask_from, :43-45), EOS masked until minimum_new_tokens tokens are
 * drawn (:250-254), and the end of a sequence at a draw of EOS (:262-269)
 * or when its generated tail equals a stop sequence starting at or after
 * minimum_new_tokens (:120-138, :271-280). The control ids PAD/UNK/BOS go in
 * dz_sampling_t.masked_ids as before. */
typedef struct {
    float repetition_penalty;     /* >= 1; 1 leaves the logits as they are */
    uint32_t eos_id;              /* >= vocab: no EOS */
    size_t minimum_new_tokens;
    uint32_t mask_from;           /* >= vocab: nothing masked */
    const uint32_t *stop_tokens;  /* the stop sequences' ids, concatenated */
    const size_t *stop_lengths;   /* [n_stops], each 1..256 */
    size_t n_stops;               /* <= 64 */
} dz_generation_controls_t;

/* generation_result_t (src/include/cli/generation.h) per sequence. */
typedef struct {
    uint32_t new_count;                /* tokens drawn, the ending one included */
    uint32_t emitted_count;            /* tokens delivered: before EOS or the matched stop sequence */
    uint32_t stopped_on_eos;
    uint32_t stopped_on_stop_sequence;
    uint32_t stop_sequence_index;      /* 0xffffffff: none */
} dz_generation_result_t;

/* dz_cuda_generate with the loop's controls (NULL: none): the loop of
 * generation_decode_with_options for every sequence at once. A sequence that
 * ends draws no more tokens; out_tokens after its end hold 0xffffffff.
 * results[batch] (host, or NULL) as generation_result_t. Runs on the layered
 * path (the fused kernel has no controls). Host buffers, synchronous. */
int dz_cuda_generate_ex(dz_cuda_cache_t *cache, const uint32_t *prompts, size_t prompt_len, size_t n_new,
                        const dz_sampling_t *sampling, const dz_generation_controls_t *controls,
                        const uint64_t *seeds, uint32_t *out_tokens, dz_generation_result_t *results);

/* dz_cuda_select with the repetition penalty (over the tokens each sequence
 * was fed since its reset) and the unassigned-id mask of `controls`; EOS,
 * the minimum length and stop sequences stay with the caller's loop, as in
 * the reference (src/cli/generation.c:246-280). DZ_E_UNSUPPORTED for a
 * penalty after a generation on the fused path (it keeps no token history)
 * until the cache is reset. */
int dz_cuda_select_ex(dz_cuda_cache_t *cache, const dz_sampling_t *sampling, const dz_generation_controls_t *controls,
                      uint64_t *rng_states, uint32_t *out_ids);

/* Execution path of dz_cuda_generate(_async). AUTO runs the fused kernel (one
 * thread block per sequence runs the whole generation, weights streamed into
 * shared memory by TMA bulk copies) whenever the model fits it (every
 * projection <= 96 KB in the device layout, column or tensor scales), else the
 * layered path (one kernel per projection / attention / norm per step, one
 * CUDA graph per job). No counterpart in the reference. */
enum { DZ_PATH_AUTO = 0, DZ_PATH_LAYERED = 1, DZ_PATH_FUSED = 2 };
int dz_cuda_cache_set_path(dz_cuda_cache_t *cache, int path);
/* 1 when dz_cuda_generate with this sampling would take the fused path. */
int dz_cuda_cache_uses_fused(const dz_cuda_cache_t *cache, const dz_sampling_t *sampling);

/* Number of kernel launches one dz_cuda_generate(_async) call issues. */
size_t dz_cuda_generate_launches(const dz_cuda_cache_t *cache, size_t prompt_len, size_t n_new,
                                 const dz_sampling_t *sampling);

/* ---- Measurement. Kernel classes of the decode path. */
enum {
    DZ_KERNEL_STEP_BEGIN = 0, /* ring bookkeeping + embedding + position */
    DZ_KERNEL_QMV = 1,        /* quantized matvec / skinny GEMM with fused epilogue */
    DZ_KERNEL_ATTENTION = 2,  /* ring-KV decode attention */
    DZ_KERNEL_LAYERNORM = 3,
    DZ_KERNEL_SELECT = 4,     /* greedy / top-k / top-p selection */
    DZ_KERNEL_SEQGEN = 5,     /* fused whole-generation kernel */
    DZ_KERNEL_SPLIT = 6,      /* activation rows -> integer limbs / fp16 parts, the MMA operands */
    DZ_KERNEL_ALLREDUCE = 7,  /* tensor parallelism: NCCL sum of the ranks' partial products */
    DZ_KERNEL_CLASSES = 8,
    /* Phases inside the fused kernel, timed on its first thread block with the
     * device's global timer (launches = 0, total_ms = time in the phase). */
    DZ_PHASE_EMBED = 8, DZ_PHASE_WAIT = 9, DZ_PHASE_QMV = 10, DZ_PHASE_ATTENTION = 11,
    DZ_PHASE_NORM = 12, DZ_PHASE_SELECT = 13, DZ_PROFILE_SLOTS = 14
};

typedef struct {
    uint32_t kind;
    uint32_t launches;
    double total_ms;   /* sum of per-launch CUDA-event durations */
    double bytes;      /* algorithmic bytes of those launches */
    double flops;
} dz_kernel_stat_t;

/* Tensor parallelism across GPUs (one process or thread per rank), the
 * layout of the large configuration: each rank holds the Q/K/V columns and
 * the W_o rows of num_heads/world heads, and the W1 columns (with their b1)
 * and W2 rows of 4*d_model/world FFN columns; embeddings, LayerNorms, the
 * head and its bias are replicated. Per layer and step, the attention-out and
 * FFN-down partial products [rows x d_model] are summed over the ranks with
 * an fp32 NCCL all-reduce (b2 and the residual are added once, before it),
 * so every rank ends each layer with the full hidden state and computes the
 * same logits and tokens. Shards are exact: a column (row) slice of a
 * per-column quantized matrix keeps its codes and scales
 * (dz_quantized_slice). Rank 0 makes the NCCL unique id with
 * dz_cuda_tp_unique_id and the host hands it to every rank; every rank
 * calls dz_cuda_model_create_tp (collective) and then makes the same calls
 * with the same arguments (generate, forward, select). With world = 1 this is
 * dz_cuda_model_create. The fused one-CTA-per-sequence path is not used.
 * No counterpart in the reference (its backend runs on one device). */
#define DZ_TP_ID_BYTES 128
int dz_cuda_tp_unique_id(uint8_t *id);
int dz_cuda_model_create_tp(const dz_model_desc_t *desc, const dz_tensor_blob_t *tensors, size_t n_tensors,
                            int device, int tp_rank, int tp_world, const uint8_t *id, dz_cuda_model_t **out);

/* Prefill policy of the layered path (dz_cuda_generate and
 * dz_cuda_prefill). TOKENS feeds the prompt one position per step through
 * dz_cuda_forward_tokens' step, as the reference's generation loop does
 * (src/cli/generation.c:231-238). BATCHED runs every prompt position of a
 * group of sequences in one pass per layer: one GEMM over all rows per
 * projection and a causal attention over each prompt, the arithmetic of
 * model_forward_hidden_masked (src/core/transformer.c:392-519). AUTO picks
 * BATCHED for models with d_model >= 512 and a head dimension of 32, 64 or
 * 128. */
#define DZ_PREFILL_AUTO 0
#define DZ_PREFILL_TOKENS 1
#define DZ_PREFILL_BATCHED 2
int dz_cuda_cache_set_prefill(dz_cuda_cache_t *cache, int mode);

/* Batched prefill of every sequence from an empty ring: ids [batch x
 * prompt_len] (host), lens [batch] positions per sequence (1..prompt_len) or
 * NULL for all, logits_out [batch x V] (host) of each sequence's last
 * position or NULL. Leaves each ring holding its prompt, ready for
 * dz_cuda_forward_tokens / dz_cuda_select. Replaces the per-token prefill
 * loop of generation_decode_with_options (src/cli/generation.c:231-238) and
 * model_forward_hidden_masked's full-prefix pass (src/core/transformer.c:
 * 392-519). Synchronous. */
int dz_cuda_prefill(dz_cuda_cache_t *cache, const uint32_t *ids, const uint32_t *lens, size_t prompt_len,
                    float *logits_out);

/* The masked full-prefix forward of model_forward_masked
 * (src/core/transformer.c:527-576, mask semantics of model_attention_mask_t,
 * src/include/core/transformer.h:43-58) for every sequence of the cache:
 * ids [batch x seq_len] (host); padding_mask [batch x seq_len] (0 = padding)
 * or NULL; attention_mask [batch x seq_len x seq_len] (row = query, 0 removes
 * the edge; causality always holds) or NULL; logits_out [batch x V] (host) of
 * each sequence's last real position. Padded rows are zeroed after the
 * embedding and after each norm, a query with no allowed key attends to
 * nothing, as in the reference. The reference's call is one sequence with
 * its own activation buffers; this one runs `batch` sequences through the
 * batched-prefill kernels and uses the cache's rings as working storage,
 * leaving every sequence empty (as after dz_cuda_cache_reset). DZ_E_INVALID
 * for seq_len 0, seq_len above max_seq_len or the cache capacity, or a
 * padding mask without a real position (MODEL_INVALID_INPUT in the
 * reference); DZ_E_UNSUPPORTED for a head dimension other than 32, 64 or
 * 128. Synchronous. */
int dz_cuda_forward_masked(dz_cuda_cache_t *cache, const uint32_t *ids, size_t seq_len,
                           const uint8_t *padding_mask, const uint8_t *attention_mask, float *logits_out);

/* Runs one dz_cuda_generate_async loop eagerly (no graph) with CUDA events
 * around every launch on the cache's stream, synchronises, and fills
 * stats[kind] for kind < n_stats. No counterpart in the reference (its
 * profiling is tools/gpu_latency.c wall-clock attribution). */
int dz_cuda_profile_generate(dz_cuda_cache_t *cache, const uint32_t *prompts_dev, size_t prompt_len,
                             size_t n_new, const dz_sampling_t *sampling, const uint64_t *seeds_dev,
                             uint32_t *out_tokens_dev, dz_kernel_stat_t *stats, size_t n_stats);

#ifdef __cplusplus
}
#endif

#endif
