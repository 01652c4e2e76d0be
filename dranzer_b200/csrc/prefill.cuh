// Batched prefill: every prompt position of a group of sequences in one pass
// per layer, the arithmetic of model_forward_hidden_masked
// (src/core/transformer.c:392-519) with the causal prefix softmax of
// attention_head_forward (:161-188), for caches whose sequences start empty.
// The projections run as one GEMM over all rows (launch_qmv); these kernels
// cover the embedding, the causal attention over each prompt (reading the
// K/V rows the QKV product wrote into the ring), the last-position gather
// and the ring bookkeeping.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace dz {

// Row r = s * T + t of the group: hidden = emb[token] + PE[t] (the prompt
// starts at position 0; out-of-vocabulary ids map to 0, PE past the host
// table as compute_positional_encoding_at, src/core/tensor_ops.c:250-260).
__global__ void dz_prefill_embed_kernel(const uint32_t* __restrict__ tokens, long long ld_tok, int T,
                                        const float* __restrict__ emb, const float* __restrict__ pe,
                                        long long pe_rows, float* __restrict__ hidden, int dim, int vocab) {
    const long long r = blockIdx.x;
    const int s = (int)(r / T), t = (int)(r % T);
    uint32_t tok = tokens[(long long)s * ld_tok + t];
    if (tok >= (uint32_t)vocab) tok = 0;
    const float* e = emb + (long long)tok * dim;
    float* h = hidden + r * dim;
    if (t < pe_rows) {
        const float* p = pe + (long long)t * dim;
        for (int i = threadIdx.x; i < dim; i += blockDim.x) h[i] = e[i] + p[i];
    } else {
        const float ln_base = logf(10000.0f);
        for (int i = threadIdx.x; i < dim; i += blockDim.x) {
            const float scale = expf(-((2.0f * (float)i) / (float)dim) * ln_base);
            const float angle = (float)t * scale;
            h[i] = e[i] + ((i % 2 == 0) ? sinf(angle) : cosf(angle));
        }
    }
}

// Epilogue row offsets of the K / V ring rows the QKV product writes: row
// r = s * T + t -> sequence s, slot t (offset s * capacity * dim + t * dim
// from the group's first sequence).
__global__ void dz_prefill_rowoff_kernel(int* __restrict__ row_off, int rows, int T, int capacity, int dim) {
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= rows) return;
    row_off[r] = (r / T) * capacity * dim + (r % T) * dim;
}

constexpr int PF_QT = 64;        // queries per block
constexpr int PF_KT = 32;        // keys per tile
constexpr int PF_THREADS = 256;  // 8 warps x 8 queries
constexpr int PF_QW = PF_QT / (PF_THREADS / 32);

// Shared memory of dz_attention_prefill_kernel for head dimension hd.
__host__ __device__ constexpr size_t dz_prefill_att_smem(int hd) {
    return ((size_t)PF_QT * hd + 2 * (size_t)PF_KT * (hd + 1)) * sizeof(float);
}

// Causal attention over one prompt, for queries [q0, q0 + PF_QT) of one
// (head, sequence): score_j = (q . k_j) / sqrtf(hd) for j <= t, softmax, o =
// sum_j p_j v_j, with the keys and values read from ring slots 0..T-1. The
// softmax runs online over key tiles (running max and sum, rescaled), so its
// rounding differs from the reference's two-pass form within fp32 noise.
// Warp w owns queries q0 + w*PF_QW .. +PF_QW; lane = key within a tile for the
// scores, lane = head-dimension element (hd/32 each) for the output.
template <int HDW>   // head_dim / 32
__global__ void __launch_bounds__(PF_THREADS) dz_attention_prefill_kernel(
    const float* __restrict__ q, const float* __restrict__ keys, const float* __restrict__ values,
    const int* __restrict__ lens, float* __restrict__ out, int T, int dim, int capacity) {
    constexpr int HD = HDW * 32;
    extern __shared__ float pf_smem[];
    float* qs = pf_smem;                         // [PF_QT][HD]
    float* ks = qs + PF_QT * HD;                 // [PF_KT][HD + 1]
    float* vs = ks + PF_KT * (HD + 1);           // [PF_KT][HD + 1]
    const int q0 = blockIdx.x * PF_QT, h = blockIdx.y, s = blockIdx.z;
    const int len = lens ? lens[s] : T;
    if (q0 >= len) return;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const float* K = keys + (long long)s * capacity * dim + h * HD;
    const float* Vv = values + (long long)s * capacity * dim + h * HD;
    const long long row0 = (long long)s * T;
    for (int i = threadIdx.x; i < PF_QT * HD; i += PF_THREADS) {
        const int qi = i / HD, e = i - qi * HD;
        const int t = q0 + qi;
        qs[i] = t < len ? q[(row0 + t) * dim + h * HD + e] : 0.0f;
    }
    const float denom = sqrtf((float)HD);
    float m[PF_QW], l[PF_QW], o[PF_QW][HDW];
#pragma unroll
    for (int i = 0; i < PF_QW; i++) {
        m[i] = -3.402823466e38f;
        l[i] = 0.0f;
#pragma unroll
        for (int c = 0; c < HDW; c++) o[i][c] = 0.0f;
    }
    const int tq_last = min(q0 + PF_QT, len) - 1;   // last query of this block
    for (int j0 = 0; j0 <= tq_last; j0 += PF_KT) {
        __syncthreads();   // previous tile consumed (and qs written, first time)
        for (int i = threadIdx.x; i < PF_KT * HD; i += PF_THREADS) {
            const int kj = i / HD, e = i - kj * HD;
            const int j = j0 + kj;
            const bool in = j <= tq_last;
            ks[kj * (HD + 1) + e] = in ? K[(long long)j * dim + e] : 0.0f;
            vs[kj * (HD + 1) + e] = in ? Vv[(long long)j * dim + e] : 0.0f;
        }
        __syncthreads();
#pragma unroll
        for (int i = 0; i < PF_QW; i++) {
            const int qi = warp * PF_QW + i;
            const int t = q0 + qi;
            if (t >= len || j0 > t) continue;   // warp-uniform
            // score of key j0 + lane
            const float* qr = qs + qi * HD;
            const float* kr = ks + lane * (HD + 1);
            float sc = 0.0f;
#pragma unroll 8
            for (int e = 0; e < HD; e++) sc = fmaf(qr[e], kr[e], sc);
            sc = sc / denom;
            const bool valid = j0 + lane <= t;
            float tmax = valid ? sc : -3.402823466e38f;
#pragma unroll
            for (int off = 16; off >= 1; off >>= 1) tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, off));
            const float mnew = fmaxf(m[i], tmax);
            const float corr = expf(m[i] - mnew);
            const float p = valid ? expf(sc - mnew) : 0.0f;
            float psum = p;
#pragma unroll
            for (int off = 16; off >= 1; off >>= 1) psum += __shfl_xor_sync(0xffffffffu, psum, off);
            l[i] = l[i] * corr + psum;
            m[i] = mnew;
#pragma unroll
            for (int c = 0; c < HDW; c++) o[i][c] *= corr;
            const int nk = min(PF_KT, t - j0 + 1);
            for (int kj = 0; kj < nk; kj++) {
                const float pk = __shfl_sync(0xffffffffu, p, kj);
                const float* vr = vs + kj * (HD + 1);
#pragma unroll
                for (int c = 0; c < HDW; c++) o[i][c] = fmaf(pk, vr[lane + 32 * c], o[i][c]);
            }
        }
    }
#pragma unroll
    for (int i = 0; i < PF_QW; i++) {
        const int t = q0 + warp * PF_QW + i;
        if (t >= len) continue;
        const float inv = 1.0f / l[i];
        float* orow = out + (row0 + t) * dim + h * HD;
#pragma unroll
        for (int c = 0; c < HDW; c++) orow[lane + 32 * c] = o[i][c] * inv;
    }
}

// hidden rows of each sequence's last prompt position -> [S][dim].
__global__ void dz_prefill_gather_kernel(const float* __restrict__ rows, const int* __restrict__ lens, int T,
                                         int dim, float* __restrict__ out) {
    const int s = blockIdx.x;
    const int t = (lens ? lens[s] : T) - 1;
    const float* src = rows + ((long long)s * T + t) * dim;
    for (int i = threadIdx.x; i < dim; i += blockDim.x) out[(long long)s * dim + i] = src[i];
}

// Ring state after a prefill of len_s tokens into empty rings.
__global__ void dz_prefill_ring_kernel(int* __restrict__ start, int* __restrict__ length,
                                       long long* __restrict__ total, const int* __restrict__ lens, int T, int S) {
    const int s = blockIdx.x * blockDim.x + threadIdx.x;
    if (s >= S) return;
    const int len = lens ? lens[s] : T;
    start[s] = 0;
    length[s] = len;
    total[s] = len;
}

}  // namespace dz
