// Token selection on the device: sample_next_token (src/cli/sampling.c:179-207)
// with greedy (:38-53), top-k (:56-102) and top-p (:105-177), after the
// generation loop's control-logit masking (src/cli/generation.c:31-46,250-254).
//
// Ordering: the reference sorts (logit, index) pairs with qsort and a
// descending comparator; glibc's qsort is a stable merge sort, so equal logits
// keep ascending index order. Here the pairs sort on the 64-bit key
// (descending-orderable float bits << 32 | index) - the same total order, with
// -0.0 folded onto +0.0 as the comparator treats them equal.
//
// Arithmetic that decides the draw (the exp values, their fp32 running sums,
// the threshold r = (float)unit * sum and the cumulative scan) is done in the
// reference's sequential order by one thread, so the chosen token matches the
// CPU path except where logits themselves differ in the last bits.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

#ifndef DZ_KERNEL_LINKAGE
#define DZ_KERNEL_LINKAGE
#endif

namespace dz {

constexpr int SEL_THREADS = 512;
constexpr int SEL_SORT_CAP = 8192;   // vocabularies sorted whole in shared memory
constexpr int SEL_TOPK_CAP = 1024;   // top-k bound for larger vocabularies

// Per-sequence state of the generation loop's controls (dz_cuda_generate_ex):
// words of one sequence's row of DZ_GEN_WORDS.
enum { GEN_NEW = 0, GEN_EMITTED = 1, GEN_EOS = 2, GEN_STOP = 3, GEN_STOP_INDEX = 4, GEN_DONE = 5, DZ_GEN_WORDS = 8 };

// The generation loop's controls beyond sample_next_token
// (src/cli/generation.c:52-72, 31-46, 250-280), all optional.
struct SelectControls {
    const uint32_t* seen;     // [B][seen_words] bit per id fed through the model since reset, or null
    int seen_words;
    float penalty;            // > 1: the sign-aware repetition penalty on the seen ids
    uint32_t mask_from;       // ids >= mask_from masked (the tokenizer's unassigned ids)
    uint32_t* state;          // [B][DZ_GEN_WORDS] loop state, or null: no EOS, stops or end
    uint32_t eos_id;          // a draw of it ends the sequence (>= V: none)
    int min_new;              // EOS masked and stops unmatched before this many new tokens
    const uint32_t* stop_tok; // the stop sequences' ids, concatenated
    const int* stop_off;      // [n_stops + 1] offsets into stop_tok
    int n_stops;
};

struct SelectArgs {
    const float* logits;   // [B][ld]
    long long ld;
    int V;
    int strategy;          // 0 greedy, 1 top-k, 2 top-p
    float temperature;
    int top_k;
    float top_p;
    const uint32_t* masked;  // ids set to -FLT_MAX before the draw
    int n_masked;
    uint64_t* rng;         // [B] xorshift64* states, or nullptr (greedy)
    uint32_t* out;         // out[b * out_stride]
    long long out_stride;
    uint32_t* out2;        // optional second copy, [B]
    SelectControls ctl;    // zero: plain selection
};

__device__ __forceinline__ uint64_t dz_rng_next(uint64_t* s) {
    uint64_t x = *s ? *s : 0x9e3779b97f4a7c15ull;
    x ^= x >> 12;
    x ^= x << 25;
    x ^= x >> 27;
    *s = x;
    return x * 2685821657736338717ull;
}

__device__ __forceinline__ double dz_rng_unit(uint64_t* s) {
    return (double)(dz_rng_next(s) >> 11) * (1.0 / 9007199254740992.0);
}

// exp rounded once to fp32 from the double-precision exponential.
__device__ __forceinline__ float dz_expf(float x) { return (float)exp((double)x); }

__device__ __forceinline__ uint64_t dz_desc_key(float v, uint32_t idx) {
    uint32_t u = __float_as_uint(v == 0.0f ? 0.0f : v);
    u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);   // ascending-orderable
    return ((uint64_t)(~u) << 32) | idx;               // descending value, ascending index
}

__device__ __forceinline__ float dz_key_value(uint64_t key) {
    uint32_t u = ~(uint32_t)(key >> 32);
    u = (u & 0x80000000u) ? (u & 0x7fffffffu) : ~u;
    return __uint_as_float(u);
}

static __device__ void dz_bitonic_sort(uint64_t* a, int n) {  // n power of two, ascending
    for (int size = 2; size <= n; size <<= 1) {
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            for (int i = threadIdx.x; i < n / 2; i += blockDim.x) {
                const int lo = 2 * i - (i & (stride - 1));
                const int hi = lo + stride;
                const bool up = (lo & size) == 0;
                const uint64_t x = a[lo], y = a[hi];
                if ((x > y) == up) { a[lo] = y; a[hi] = x; }
            }
            __syncthreads();
        }
    }
}

// Logit i as the draw sees it: repetition penalty on an id the sequence
// holds (generation_apply_repetition_penalty: multiplied when negative,
// divided otherwise), then the masked ids, the unassigned range and EOS
// under the minimum length set to -FLT_MAX.
struct SelRow {
    const uint32_t* seen;   // this sequence's bits, or null
    bool eos_masked;
};
__device__ __forceinline__ float dz_masked_logit(const SelectArgs& a, const SelRow& row, const float* lg, int i) {
    float v = lg[i];
    if (row.seen && ((row.seen[i >> 5] >> (i & 31)) & 1u))
        v = v < 0.0f ? v * a.ctl.penalty : __fdiv_rn(v, a.ctl.penalty);
    for (int m = 0; m < a.n_masked; m++)
        if (a.masked[m] == (uint32_t)i) v = -3.402823466e38f;
    if ((uint32_t)i >= a.ctl.mask_from) v = -3.402823466e38f;
    if (row.eos_masked && (uint32_t)i == a.ctl.eos_id) v = -3.402823466e38f;
    return v;
}

// One block per sequence. Dynamic shared memory: 8 * max(pow2(V), 2*TOPK) + 4*V bytes
// (sort path) - see dz_select_smem_bytes.
DZ_KERNEL_LINKAGE __global__ void __launch_bounds__(SEL_THREADS) dz_select_kernel(SelectArgs a) {
    extern __shared__ unsigned char sel_smem[];
    __shared__ uint64_t best_key[SEL_THREADS / 32];
    __shared__ uint32_t sel_result;
    const int b = blockIdx.x;
    const float* lg = a.logits + (long long)b * a.ld;
    const int V = a.V;
    uint32_t* gst = a.ctl.state ? a.ctl.state + (long long)b * DZ_GEN_WORDS : nullptr;
    if (gst && gst[GEN_DONE]) {   // the sequence has ended: no draw (uniform over the block)
        if (threadIdx.x == 0) {
            a.out[(long long)b * a.out_stride] = 0xffffffffu;
            if (a.out2) a.out2[b] = 0u;
        }
        return;
    }
    SelRow row;
    row.seen = a.ctl.seen && a.ctl.penalty > 1.0f ? a.ctl.seen + (long long)b * a.ctl.seen_words : nullptr;
    row.eos_masked = gst && (int)gst[GEN_NEW] < a.ctl.min_new && a.ctl.eos_id < (uint32_t)V;
    const bool greedy = a.strategy == 0 || !(a.temperature > 0.0f) || a.rng == nullptr ||
                        (a.strategy == 1 && a.top_k == 0) ||
                        (a.strategy == 2 && (a.top_p <= 0.0f || a.top_p > 1.0f)) ||
                        (a.strategy != 1 && a.strategy != 2);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (greedy) {
        // first index of the strict maximum: smallest descending key
        uint64_t best = ~0ull;
        for (int i = threadIdx.x; i < V; i += SEL_THREADS) {
            const uint64_t k = dz_desc_key(dz_masked_logit(a, row, lg, i), (uint32_t)i);
            best = k < best ? k : best;
        }
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) {
            const uint64_t o = __shfl_xor_sync(0xffffffffu, best, off);
            best = o < best ? o : best;
        }
        if (lane == 0) best_key[warp] = best;
        __syncthreads();
        if (threadIdx.x == 0) {
            uint64_t m = best_key[0];
            for (int w = 1; w < SEL_THREADS / 32; w++) m = best_key[w] < m ? best_key[w] : m;
            sel_result = (uint32_t)(m & 0xffffffffu);
        }
        __syncthreads();
    } else {
        const float inv_t = 1.0f / a.temperature;
        uint64_t* keys = reinterpret_cast<uint64_t*>(sel_smem);
        int n_sorted;       // sorted prefix available in keys[]
        if (V <= SEL_SORT_CAP) {
            int P = 1;
            while (P < V) P <<= 1;
            for (int i = threadIdx.x; i < P; i += SEL_THREADS)
                keys[i] = i < V ? dz_desc_key(dz_masked_logit(a, row, lg, i) * inv_t, (uint32_t)i) : ~0ull;
            __syncthreads();
            dz_bitonic_sort(keys, P);
            n_sorted = V;
        } else {
            // top-k over a large vocabulary: radix-select the k-th smallest
            // composite key (all keys distinct), gather the k smallest, sort them.
            __shared__ unsigned int hist[256];
            __shared__ unsigned long long prefix_s;
            __shared__ unsigned int remaining_s, count_s;
            const int k = a.top_k < V ? a.top_k : V;
            if (threadIdx.x == 0) { prefix_s = 0; remaining_s = (unsigned)k; count_s = 0; }
            __syncthreads();
            for (int pass = 7; pass >= 0; pass--) {
                for (int i = threadIdx.x; i < 256; i += SEL_THREADS) hist[i] = 0;
                __syncthreads();
                const unsigned long long prefix = prefix_s;
                const int shift = pass * 8;
                const unsigned long long hi_mask = pass == 7 ? 0ull : (~0ull << (shift + 8));
                for (int i = threadIdx.x; i < V; i += SEL_THREADS) {
                    const uint64_t key = dz_desc_key(dz_masked_logit(a, row, lg, i) * inv_t, (uint32_t)i);
                    if ((key & hi_mask) == prefix) atomicAdd(&hist[(key >> shift) & 0xff], 1u);
                }
                __syncthreads();
                if (threadIdx.x == 0) {
                    unsigned int rem = remaining_s, acc = 0;
                    int d = 0;
                    for (; d < 256; d++) {
                        if (acc + hist[d] >= rem) break;
                        acc += hist[d];
                    }
                    remaining_s = rem - acc;
                    prefix_s = prefix | ((unsigned long long)d << shift);
                }
                __syncthreads();
            }
            const unsigned long long kth = prefix_s;
            for (int i = threadIdx.x; i < V; i += SEL_THREADS) {
                const uint64_t key = dz_desc_key(dz_masked_logit(a, row, lg, i) * inv_t, (uint32_t)i);
                if (key <= kth) {
                    const unsigned int slot = atomicAdd(&count_s, 1u);
                    if (slot < (unsigned)SEL_TOPK_CAP) keys[slot] = key;
                }
            }
            __syncthreads();
            int P = 1;
            while (P < k) P <<= 1;
            for (int i = k + threadIdx.x; i < P; i += SEL_THREADS) keys[i] = ~0ull;
            __syncthreads();
            dz_bitonic_sort(keys, P);
            n_sorted = k;
        }
        float* e = reinterpret_cast<float*>(keys + (n_sorted > 1 ? n_sorted : 1) + 1);
        const float top = dz_key_value(keys[0]);
        const int nexp = a.strategy == 1 ? (a.top_k < n_sorted ? a.top_k : n_sorted) : n_sorted;
        for (int i = threadIdx.x; i < nexp; i += SEL_THREADS) e[i] = dz_expf(dz_key_value(keys[i]) - top);
        __syncthreads();
        if (threadIdx.x == 0) {
            uint64_t* st = a.rng + b;
            uint32_t selected = (uint32_t)(keys[0] & 0xffffffffu);
            if (a.strategy == 1) {
                float sum = 0.0f;
                for (int i = 0; i < nexp; i++) sum += e[i];
                const float r = (float)dz_rng_unit(st) * sum;
                float acc = 0.0f;
                for (int i = 0; i < nexp; i++) {
                    acc += e[i];
                    if (acc >= r) { selected = (uint32_t)(keys[i] & 0xffffffffu); break; }
                }
            } else {
                float sum_all = 0.0f;
                for (int i = 0; i < nexp; i++) sum_all += e[i];
                const float inv = 1.0f / sum_all;
                float cum = 0.0f;
                int cand = nexp;
                for (int i = 0; i < nexp; i++) {
                    cum += e[i] * inv;
                    if (cum >= a.top_p) { cand = i + 1; break; }
                }
                float nsum = 0.0f;
                for (int i = 0; i < cand; i++) nsum += e[i];
                const float r = (float)dz_rng_unit(st) * nsum;
                float acc = 0.0f;
                for (int i = 0; i < cand; i++) {
                    acc += e[i];
                    if (acc >= r) { selected = (uint32_t)(keys[i] & 0xffffffffu); break; }
                }
            }
            sel_result = selected;
        }
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        const uint32_t tok = sel_result;
        uint32_t* o = a.out + (long long)b * a.out_stride;
        *o = tok;
        if (a.out2) a.out2[b] = tok;
        if (gst) {
            // the end of a sequence (src/cli/generation.c:262-280): EOS, or the
            // generated tail equal to a stop sequence that starts at or after
            // the minimum length; `o` is column new_count - 1 of the row
            const uint32_t nc = gst[GEN_NEW] + 1;
            gst[GEN_NEW] = nc;
            uint32_t done = 0;
            if (tok == a.ctl.eos_id) {
                gst[GEN_EMITTED] = nc - 1;
                gst[GEN_EOS] = 1;
                done = 1;
            } else {
                for (int q = 0; q < a.ctl.n_stops && !done; q++) {
                    const int len = a.ctl.stop_off[q + 1] - a.ctl.stop_off[q];
                    if ((uint32_t)len > nc || (int)(nc - (uint32_t)len) < a.ctl.min_new) continue;
                    bool eq = true;
                    for (int j = 0; j < len && eq; j++)
                        eq = o[-(long long)(len - 1 - j)] == a.ctl.stop_tok[a.ctl.stop_off[q] + j];
                    if (eq) {
                        gst[GEN_EMITTED] = nc - (uint32_t)len;
                        gst[GEN_STOP] = 1;
                        gst[GEN_STOP_INDEX] = (uint32_t)q;
                        done = 1;
                    }
                }
                if (!done) gst[GEN_EMITTED] = nc;
            }
            gst[GEN_DONE] = done;
        }
    }
}

// Fresh loop state for every sequence of a generation.
DZ_KERNEL_LINKAGE __global__ void dz_gen_init_kernel(uint32_t* __restrict__ state, int B) {
    const int b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= B) return;
    uint32_t* s = state + (long long)b * DZ_GEN_WORDS;
    for (int w = 0; w < DZ_GEN_WORDS; w++) s[w] = 0u;
    s[GEN_STOP_INDEX] = 0xffffffffu;
}

// Clears the token history of the sequences whose mask byte is set (all
// when mask is null): grid (ceil(words / 256), B).
DZ_KERNEL_LINKAGE __global__ void dz_seen_clear_kernel(uint32_t* __restrict__ seen, int words, const uint8_t* __restrict__ mask) {
    const int b = blockIdx.y;
    const int w = blockIdx.x * blockDim.x + threadIdx.x;
    if (w < words && (!mask || mask[b])) seen[(long long)b * words + w] = 0u;
}

inline size_t dz_select_smem_bytes(int V, int strategy, int top_k) {
    if (strategy == 0) return 0;
    size_t n;
    if (V <= SEL_SORT_CAP) {
        size_t P = 1;
        while (P < (size_t)V) P <<= 1;
        n = P;
    } else {
        size_t P = 1;
        while (P < (size_t)(top_k < SEL_TOPK_CAP ? top_k : SEL_TOPK_CAP)) P <<= 1;
        n = P > (size_t)SEL_TOPK_CAP ? P : (size_t)SEL_TOPK_CAP;
    }
    return n * 8 + 8 + (size_t)(V <= SEL_SORT_CAP ? V : SEL_TOPK_CAP) * 4 + 16;
}

// rng state per sequence from its seed: dranzer_rng_stream(seed, SAMPLING)
// (src/core/rng.c:25-33).
__device__ __forceinline__ uint64_t dz_splitmix64(uint64_t x) {
    x += 0x9e3779b97f4a7c15ull;
    x = (x ^ (x >> 30)) * 0xbf58476d1ce4e5b9ull;
    x = (x ^ (x >> 27)) * 0x94d049bb133111ebull;
    return x ^ (x >> 31);
}

DZ_KERNEL_LINKAGE __global__ void dz_seed_kernel(const uint64_t* __restrict__ seeds, uint64_t* __restrict__ states, int B,
                               uint64_t stream) {
    const int b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= B) return;
    uint64_t s = dz_splitmix64(seeds[b] ^ dz_splitmix64(stream));
    states[b] = s ? s : 0x9e3779b97f4a7c15ull;
}

}  // namespace dz
