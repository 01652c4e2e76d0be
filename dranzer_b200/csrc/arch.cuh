// Kernels of the architecture bits (src/include/core/model_types.h:26-36)
// beyond the default post-LN / ReLU / learned-head block: rotary position
// embedding of Q and K, RMSNorm, the SwiGLU gate, and the output head tied to
// the token embeddings. fp32, the reference's operation order, no contraction
// where the reference has none.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace dz {

// rope_rotate (src/core/transformer.c:24-54): pair (2p, 2p + 1) of every head
// rotated by position * 10000^(-2p / head_dim); cosine and sine are those of
// the double-precision angle, rounded to float. Positions below tab_rows come
// from the host table (cos, sin interleaved per pair), the rest are computed
// here in double.
__device__ __forceinline__ void dz_rope_pair(float* x, long long pos, int p, int hd, const float* __restrict__ tab,
                                             long long tab_rows) {
    float c, s;
    if (pos < tab_rows) {
        c = tab[(pos * (hd / 2) + p) * 2];
        s = tab[(pos * (hd / 2) + p) * 2 + 1];
    } else {
        const double angle = (double)pos * pow(10000.0, -(double)(2 * p) / (double)hd);
        c = (float)cos(angle);
        s = (float)sin(angle);
    }
    const float a = x[2 * p], b = x[2 * p + 1];
    x[2 * p] = __fsub_rn(__fmul_rn(a, c), __fmul_rn(b, s));
    x[2 * p + 1] = __fadd_rn(__fmul_rn(a, s), __fmul_rn(b, c));
}

// Decode step: sequence b's query row and its new key row (ring slot
// row_off[b]) at position total[b] - 1 (the step's position; the step-begin
// kernel has advanced total). One block per sequence.
__global__ void dz_rope_decode_kernel(float* __restrict__ q, float* __restrict__ keys, long long seq_stride,
                                      const int* __restrict__ row_off, const long long* __restrict__ total,
                                      int width, int hd, const float* __restrict__ tab, long long tab_rows) {
    const int b = blockIdx.x;
    const long long pos = total[b] - 1;
    float* qr = q + (long long)b * width;
    float* kr = keys + (long long)b * seq_stride + row_off[b];
    const int pairs = width / 2;
    for (int i = threadIdx.x; i < pairs; i += blockDim.x) {
        const int h = (2 * i) / hd, p = i - h * (hd / 2);
        dz_rope_pair(qr + h * hd, pos, p, hd, tab, tab_rows);
        dz_rope_pair(kr + h * hd, pos, p, hd, tab, tab_rows);
    }
}

// Batched prefill: row r = s * T + t of the query rows and sequence s's key
// row in slot t, at position t. One block per row.
__global__ void dz_rope_prefill_kernel(float* __restrict__ q, float* __restrict__ keys, long long seq_stride, int T,
                                       int width, int hd, const float* __restrict__ tab, long long tab_rows) {
    const long long r = blockIdx.x;
    const int s = (int)(r / T), t = (int)(r % T);
    float* qr = q + r * width;
    float* kr = keys + (long long)s * seq_stride + (long long)t * width;
    const int pairs = width / 2;
    for (int i = threadIdx.x; i < pairs; i += blockDim.x) {
        const int h = (2 * i) / hd, p = i - h * (hd / 2);
        dz_rope_pair(qr + h * hd, t, p, hd, tab, tab_rows);
        dz_rope_pair(kr + h * hd, t, p, hd, tab, tab_rows);
    }
}

// rms_normalize (src/core/tensor_ops.c:173-179), eps 1e-6: rms =
// sqrtf(sum(x^2) / dim + eps), y = gamma * x / rms. One block per row;
// `residual`, when given, is added to x first.
constexpr int RMS_THREADS = 256;
__global__ void __launch_bounds__(RMS_THREADS) dz_rmsnorm_kernel(const float* __restrict__ x,
                                                                 const float* __restrict__ residual,
                                                                 const float* __restrict__ gamma,
                                                                 float* __restrict__ y, int dim, float eps) {
    __shared__ float red[RMS_THREADS / 32];
    __shared__ float stat;
    const int r = blockIdx.x;
    const float* xr = x + (long long)r * dim;
    const float* rr = residual ? residual + (long long)r * dim : nullptr;
    float* yr = y + (long long)r * dim;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float s = 0.0f;
    for (int i = threadIdx.x; i < dim; i += RMS_THREADS) {
        const float v = rr ? xr[i] + rr[i] : xr[i];
        s = fmaf(v, v, s);
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
    if (lane == 0) red[warp] = s;
    __syncthreads();
    if (threadIdx.x == 0) {
        float t = 0.0f;
        for (int w = 0; w < RMS_THREADS / 32; w++) t += red[w];
        stat = sqrtf(t / (float)dim + eps);
    }
    __syncthreads();
    const float rms = stat;
    for (int i = threadIdx.x; i < dim; i += RMS_THREADS) {
        const float v = rr ? xr[i] + rr[i] : xr[i];
        yr[i] = __fdiv_rn(__fmul_rn(gamma[i], v), rms);
    }
}

// silu (src/core/tensor_ops.c:29-40): x * sigmoid(x), the sigmoid formed
// from exp(-|x|) on the side that cannot overflow.
__device__ __forceinline__ float dz_silu(float x) {
    float sg;
    if (x >= 0.0f) {
        const float z = expf(-x);
        sg = __fdiv_rn(1.0f, __fadd_rn(1.0f, z));
    } else {
        const float z = expf(x);
        sg = __fdiv_rn(z, __fadd_rn(1.0f, z));
    }
    return __fmul_rn(x, sg);
}

// The SwiGLU hidden (src/core/transformer.c:819-828): per row, the first F
// columns hold x W1 + b1 and the next F hold x W_gate + b_gate; column j
// becomes silu(pre_j) * gate_j, in place. Grid (ceil(F / 256), <= 65535),
// rows strided over grid y.
__global__ void dz_swiglu_kernel(float* __restrict__ buf, int rows, int F, long long ld) {
    const int j = blockIdx.x * blockDim.x + threadIdx.x;
    if (j >= F) return;
    for (int r = blockIdx.y; r < rows; r += gridDim.y) {
        float* row = buf + (long long)r * ld;
        row[j] = __fmul_rn(dz_silu(row[j]), row[F + j]);
    }
}

// The tied output head (src/core/lm_head.c:21-46): logits[b][v] =
// hidden[b] . token_embeddings[v] + bias[v]. One warp per vocabulary row
// (eight per block), each lane a strided share of the dimension, rows of
// hidden read through L1.
constexpr int TIED_ROWS = 8;
__global__ void __launch_bounds__(256) dz_tied_head_kernel(const float* __restrict__ hidden, int B,
                                                           const float* __restrict__ emb,
                                                           const float* __restrict__ bias, float* __restrict__ logits,
                                                           int V, int dim) {
    const int v = blockIdx.x * TIED_ROWS + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (v >= V) return;
    const float* e = emb + (long long)v * dim;
    for (int b = 0; b < B; b++) {
        const float* h = hidden + (long long)b * dim;
        float s = 0.0f;
        for (int i = lane; i < dim; i += 32) s = fmaf(h[i], e[i], s);
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
        if (lane == 0) logits[(long long)b * V + v] = s + bias[v];
    }
}

}  // namespace dz
