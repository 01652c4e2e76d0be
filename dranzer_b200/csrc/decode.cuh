// Decode-step kernels: ring-slot bookkeeping + embedding, ring-KV causal
// attention for one new token per sequence, LayerNorm. fp32 throughout, the
// arithmetic of src/core/transformer.c:686-858 and src/core/tensor_ops.c.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace dz {

// Per-sequence ring state, the fields of model_kv_cache_t
// (src/include/core/transformer.h:10-31) one entry per sequence.
struct RingState {
    int* start;       // physical slot of the oldest token
    int* length;      // retained tokens (<= capacity)
    long long* total; // absolute tokens consumed since reset
    int* slot;        // this step: slot the new K/V row is written to
    int* ctx;         // this step: context length attended over
    int* row_off;     // this step: slot * dim (epilogue scatter offset)
    uint32_t* seen;   // [B][seen_words]: a bit per token id fed since reset (the
    int seen_words;   // sequence the repetition penalty looks at)
};

// One block per sequence: the ring bookkeeping of model_forward_token
// (src/core/transformer.c:765-775), then hidden = emb[token] + PE[position]
// (:780-799, out-of-vocabulary ids map to 0). Positions past the host table
// are computed as compute_positional_encoding_at (src/core/tensor_ops.c:250-260)
// in the exp(-x ln 10000) form the host table uses.
__global__ void dz_step_begin_kernel(RingState rs, const uint32_t* __restrict__ tokens, long long tok_stride,
                                     const float* __restrict__ emb, const float* __restrict__ pe,
                                     long long pe_rows, float* __restrict__ hidden, int dim, int kv_dim, int vocab,
                                     int capacity) {
    const int b = blockIdx.x;
    const int len = rs.length[b], start = rs.start[b];
    const long long pos = rs.total[b];
    int slot, ctx, new_start = start;
    if (len < capacity) {
        slot = (start + len) % capacity;
        ctx = len + 1;
    } else {
        slot = start;
        new_start = (start + 1) % capacity;
        ctx = capacity;
    }
    uint32_t tok = tokens[(long long)b * tok_stride];
    if (tok >= (uint32_t)vocab) tok = 0;
    else if (rs.seen && threadIdx.x == 0)
        rs.seen[(long long)b * rs.seen_words + (tok >> 5)] |= 1u << (tok & 31);
    const float* e = emb + (long long)tok * dim;
    float* h = hidden + (long long)b * dim;
    if (!pe) {   // rotary positions: no additive encoding (src/core/transformer.c:780-799)
        for (int i = threadIdx.x; i < dim; i += blockDim.x) h[i] = __fadd_rn(e[i], 0.0f);
    } else if (pos < pe_rows) {
        const float* p = pe + pos * dim;
        for (int i = threadIdx.x; i < dim; i += blockDim.x) h[i] = e[i] + p[i];
    } else {
        const float ln_base = logf(10000.0f);
        for (int i = threadIdx.x; i < dim; i += blockDim.x) {
            const float scale = expf(-((2.0f * (float)i) / (float)dim) * ln_base);
            const float angle = (float)pos * scale;
            h[i] = e[i] + ((i % 2 == 0) ? sinf(angle) : cosf(angle));
        }
    }
    __syncthreads();  // every thread has read the old ring state
    if (threadIdx.x == 0) {
        rs.slot[b] = slot;
        rs.ctx[b] = ctx;
        rs.row_off[b] = slot * kv_dim;   // this rank's K / V row width
        rs.start[b] = new_start;
        rs.length[b] = len < capacity ? len + 1 : len;
        rs.total[b] = pos + 1;
    }
}

constexpr int ATT_THREADS = 128;

// attention_head_forward_token (src/core/transformer.c:686-713) for one
// (head, sequence): score_j = (q . k_j) / sqrtf(hd) over the logical context
// j = 0..ctx-1 at physical row (start + j) % capacity, softmax, then
// o = sum_j p_j v_j. Scores live in shared memory (capacity floats).
__global__ void __launch_bounds__(ATT_THREADS) dz_attention_decode_kernel(
    const float* __restrict__ q, const float* __restrict__ keys, const float* __restrict__ values,
    const int* __restrict__ start_arr, const int* __restrict__ ctx_arr, float* __restrict__ out,
    int dim, int head_dim, int capacity) {
    extern __shared__ float smem[];
    float* scores = smem;                 // [capacity]
    float* qs = smem + capacity;          // [head_dim]
    float* part = qs + head_dim;          // [ATT_THREADS]
    __shared__ float red[ATT_THREADS / 32];

    const int h = blockIdx.x, b = blockIdx.y;
    const int ctx = ctx_arr[b], start = start_arr[b];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const float* K = keys + (long long)b * capacity * dim + h * head_dim;
    const float* V = values + (long long)b * capacity * dim + h * head_dim;
    for (int e = threadIdx.x; e < head_dim; e += ATT_THREADS) qs[e] = q[(long long)b * dim + h * head_dim + e];
    __syncthreads();

    const float denom = sqrtf((float)head_dim);
    for (int j = warp; j < ctx; j += ATT_THREADS / 32) {
        const int phys = (start + j) % capacity;
        const float* kr = K + (long long)phys * dim;
        float s = 0.0f;
        for (int e = lane; e < head_dim; e += 32) s = fmaf(qs[e], kr[e], s);
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
        if (lane == 0) scores[j] = s / denom;
    }
    __syncthreads();

    // softmax (src/core/tensor_ops.c:55-76): max, exp(x - max), sum, * 1/sum
    float mx = -3.402823466e38f;
    for (int j = threadIdx.x; j < ctx; j += ATT_THREADS) mx = fmaxf(mx, scores[j]);
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
    if (lane == 0) red[warp] = mx;
    __syncthreads();
    mx = red[0];
    for (int w = 1; w < ATT_THREADS / 32; w++) mx = fmaxf(mx, red[w]);
    __syncthreads();
    float sum = 0.0f;
    for (int j = threadIdx.x; j < ctx; j += ATT_THREADS) {
        const float ev = expf(scores[j] - mx);
        scores[j] = ev;
        sum += ev;
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
    if (lane == 0) red[warp] = sum;
    __syncthreads();
    sum = 0.0f;
    for (int w = 0; w < ATT_THREADS / 32; w++) sum += red[w];
    const float inv = 1.0f / sum;

    // o[e] = sum_j p_j v_j[e], p_j = e_j * (1/sum) as the reference's softmax
    // stores it. Thread (g, e) sums rows j = g, g + G, ...; groups combine in smem.
    if (head_dim <= ATT_THREADS) {
        const int groups = ATT_THREADS / head_dim;
        const int e = threadIdx.x % head_dim, g = threadIdx.x / head_dim;
        float acc = 0.0f;
        if (g < groups) {
            for (int j = g; j < ctx; j += groups) {
                const int phys = (start + j) % capacity;
                acc = fmaf(scores[j] * inv, V[(long long)phys * dim + e], acc);
            }
        }
        part[threadIdx.x] = acc;
        __syncthreads();
        if (threadIdx.x < head_dim) {
            float o = 0.0f;
            for (int gg = 0; gg < groups; gg++) o += part[gg * head_dim + threadIdx.x];
            out[(long long)b * dim + h * head_dim + threadIdx.x] = o;
        }
    } else {
        for (int e = threadIdx.x; e < head_dim; e += ATT_THREADS) {
            float acc = 0.0f;
            for (int j = 0; j < ctx; j++) {
                const int phys = (start + j) % capacity;
                acc = fmaf(scores[j] * inv, V[(long long)phys * dim + e], acc);
            }
            out[(long long)b * dim + h * head_dim + e] = acc;
        }
    }
}

// attention_head_forward_token for head dimensions of 64 / 128 at long
// contexts, streaming the K / V rows at bandwidth: one block per (head,
// sequence), four warps; warp w takes keys w*8 .. w*8+7, then +32, ...; lanes
// hold HDW consecutive elements of the head dimension, so every K or V row is
// one coalesced 256- or 512-byte read, and eight keys are in flight per warp.
// The softmax runs online per warp (running max and sum, rescaled) and the
// four warps combine in shared memory, so rounding differs from the
// reference's two-pass softmax within fp32 noise.
constexpr int ATT2_THREADS = 128;
constexpr int ATT2_KEYS = 8;

template <int HDW>   // head_dim / 32: 2 or 4
__global__ void __launch_bounds__(ATT2_THREADS) dz_attention_decode2_kernel(
    const float* __restrict__ q, const float* __restrict__ keys, const float* __restrict__ values,
    const int* __restrict__ start_arr, const int* __restrict__ ctx_arr, float* __restrict__ out, int dim,
    int capacity) {
    constexpr int HD = HDW * 32;
    constexpr int NW = ATT2_THREADS / 32;
    __shared__ float sm_m[NW], sm_l[NW];
    __shared__ float sm_o[NW][HD];
    const int h = blockIdx.x, b = blockIdx.y;
    const int ctx = ctx_arr[b], start = start_arr[b];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const float* K = keys + (long long)b * capacity * dim + h * HD + lane * HDW;
    const float* V = values + (long long)b * capacity * dim + h * HD + lane * HDW;
    // a lane's HDW elements of a row are one 16-byte (hd 128) or 8-byte
    // (hd 64) load: rows start on 16-byte boundaries (dim and hd are
    // multiples of 64)
    auto load_row = [&](const float* p, float* v) {
        if (HDW == 4) {
            const float4 x = *reinterpret_cast<const float4*>(p);
            v[0] = x.x; v[1] = x.y; v[2] = x.z; v[3] = x.w;
        } else {
            const float2 x = *reinterpret_cast<const float2*>(p);
            v[0] = x.x; v[1] = x.y;
        }
    };
    float qv[HDW];
    load_row(q + (long long)b * dim + h * HD + lane * HDW, qv);
    const float denom = sqrtf((float)HD);
    float m = -3.402823466e38f, l = 0.0f, o[HDW];
#pragma unroll
    for (int c = 0; c < HDW; c++) o[c] = 0.0f;
    for (int j0 = warp * ATT2_KEYS; j0 < ctx; j0 += NW * ATT2_KEYS) {
        float kv[ATT2_KEYS][HDW], sc[ATT2_KEYS];
#pragma unroll
        for (int u = 0; u < ATT2_KEYS; u++) {
            const int j = j0 + u;
            int phys = start + j;
            if (phys >= capacity) phys -= capacity;
            if (j < ctx) {
                load_row(K + (long long)phys * dim, kv[u]);
            } else {
#pragma unroll
                for (int c = 0; c < HDW; c++) kv[u][c] = 0.0f;
            }
        }
#pragma unroll
        for (int u = 0; u < ATT2_KEYS; u++) {
            float d = 0.0f;
#pragma unroll
            for (int c = 0; c < HDW; c++) d = fmaf(qv[c], kv[u][c], d);
            sc[u] = d;
        }
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1)
#pragma unroll
            for (int u = 0; u < ATT2_KEYS; u++) sc[u] += __shfl_xor_sync(0xffffffffu, sc[u], off);
        float tmax = m;
#pragma unroll
        for (int u = 0; u < ATT2_KEYS; u++) {
            sc[u] = sc[u] / denom;
            if (j0 + u < ctx) tmax = fmaxf(tmax, sc[u]);
        }
        const float corr = expf(m - tmax);
        l *= corr;
#pragma unroll
        for (int c = 0; c < HDW; c++) o[c] *= corr;
        m = tmax;
#pragma unroll
        for (int u = 0; u < ATT2_KEYS; u++) {
            const int j = j0 + u;
            if (j >= ctx) break;
            const float p = expf(sc[u] - m);
            l += p;
            int phys = start + j;
            if (phys >= capacity) phys -= capacity;
            float vv[HDW];
            load_row(V + (long long)phys * dim, vv);
#pragma unroll
            for (int c = 0; c < HDW; c++) o[c] = fmaf(p, vv[c], o[c]);
        }
    }
    if (lane == 0) {
        sm_m[warp] = m;
        sm_l[warp] = l;
    }
#pragma unroll
    for (int c = 0; c < HDW; c++) sm_o[warp][lane * HDW + c] = o[c];
    __syncthreads();
    if (warp == 0) {
        float M = sm_m[0];
        for (int w = 1; w < NW; w++) M = fmaxf(M, sm_m[w]);
        float L = 0.0f, acc[HDW];
#pragma unroll
        for (int c = 0; c < HDW; c++) acc[c] = 0.0f;
        for (int w = 0; w < NW; w++) {
            const float f = sm_l[w] > 0.0f ? expf(sm_m[w] - M) : 0.0f;
            L += sm_l[w] * f;
#pragma unroll
            for (int c = 0; c < HDW; c++) acc[c] = fmaf(sm_o[w][lane * HDW + c], f, acc[c]);
        }
        const float inv = 1.0f / L;
#pragma unroll
        for (int c = 0; c < HDW; c++) out[(long long)b * dim + h * HD + lane * HDW + c] = acc[c] * inv;
    }
}

constexpr int LN_THREADS = 256;

// layer_normalize (src/core/tensor_ops.c:88-111), eps 1e-6: mean, biased
// variance of (x - mean), sigma = sqrtf(var + eps), y = gamma*((x-mean)/sigma)+beta.
// One block per row. `residual`, when given, is added to x first (the
// attention sub-block's attn_raw += hidden, src/core/transformer.c:804-806).
//
// The row statistics and the element formula are shared with the norm that
// also writes the next product's limbs (umma.cuh), so both give the same y
// bit for bit.
__device__ __forceinline__ void dz_ln_stats(const float* __restrict__ xr, const float* __restrict__ rr, int dim,
                                            float eps, float* red, float* stat, float& mean, float& sd) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float s = 0.0f;
    for (int i = threadIdx.x; i < dim; i += LN_THREADS) s += rr ? xr[i] + rr[i] : xr[i];
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
    if (lane == 0) red[warp] = s;
    __syncthreads();
    if (threadIdx.x == 0) {
        float t = 0.0f;
        for (int w = 0; w < LN_THREADS / 32; w++) t += red[w];
        *stat = t / (float)dim;
    }
    __syncthreads();
    mean = *stat;
    float v = 0.0f;
    for (int i = threadIdx.x; i < dim; i += LN_THREADS) {
        const float d = (rr ? xr[i] + rr[i] : xr[i]) - mean;
        v = fmaf(d, d, v);
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    if (threadIdx.x == 0) {
        float t = 0.0f;
        for (int w = 0; w < LN_THREADS / 32; w++) t += red[w];
        *stat = sqrtf(t / (float)dim + eps);
    }
    __syncthreads();
    sd = *stat;
}
__device__ __forceinline__ float dz_ln_value(float xv, float mean, float sd, float g, float b) {
    return g * ((xv - mean) / sd) + b;
}

__global__ void __launch_bounds__(LN_THREADS) dz_layernorm_kernel(
    const float* __restrict__ x, const float* __restrict__ residual, const float* __restrict__ gamma,
    const float* __restrict__ beta, float* __restrict__ y, int dim, float eps) {
    __shared__ float red[LN_THREADS / 32];
    __shared__ float stat;
    const int r = blockIdx.x;
    const float* xr = x + (long long)r * dim;
    const float* rr = residual ? residual + (long long)r * dim : nullptr;
    float* yr = y + (long long)r * dim;
    float mean, sd;
    dz_ln_stats(xr, rr, dim, eps, red, &stat, mean, sd);
    for (int i = threadIdx.x; i < dim; i += LN_THREADS) {
        const float xv = rr ? xr[i] + rr[i] : xr[i];
        yr[i] = dz_ln_value(xv, mean, sd, gamma[i], beta[i]);
    }
}

}  // namespace dz
