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
                                        long long pe_rows, float* __restrict__ hidden, int dim, int vocab,
                                        const int* __restrict__ lens, uint32_t* __restrict__ seen,
                                        int seen_words) {
    const long long r = blockIdx.x;
    const int s = (int)(r / T), t = (int)(r % T);
    uint32_t tok = tokens[(long long)s * ld_tok + t];
    if (tok >= (uint32_t)vocab) tok = 0;
    else if (seen && threadIdx.x == 0 && (!lens || t < lens[s]))   // the sequence's token history
        atomicOr(&seen[(long long)s * seen_words + (tok >> 5)], 1u << (tok & 31));
    const float* e = emb + (long long)tok * dim;
    float* h = hidden + r * dim;
    if (!pe) {   // rotary positions: no additive encoding (src/core/transformer.c:780-799)
        for (int i = threadIdx.x; i < dim; i += blockDim.x) h[i] = __fadd_rn(e[i], 0.0f);
    } else if (t < pe_rows) {
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
constexpr int PF_THREADS = 256;
constexpr int PF_PLD = PF_QT + 4;   // transposed probability tile row stride

// Shared memory of dz_attention_prefill_kernel for head dimension hd: the
// query tile, two K / V tile buffers, the probability tile, softmax state.
__host__ __device__ constexpr size_t dz_prefill_att_smem(int hd) {
    return ((size_t)PF_QT * (hd + 4) + 4 * (size_t)PF_KT * (hd + 4) + (size_t)PF_KT * PF_PLD + 3 * PF_QT) *
           sizeof(float);
}

__device__ __forceinline__ void pf_cp_async16(void* dst, const void* src, bool valid) {
    const uint32_t d = (uint32_t)__cvta_generic_to_shared(dst);
    const int n = valid ? 16 : 0;   // zero-fill rows past the block's last query
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(d), "l"(src), "r"(n) : "memory");
}
__device__ __forceinline__ void pf_cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void pf_cp_wait_all_but_one() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }
__device__ __forceinline__ void pf_cp_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

// Causal attention over one prompt, for queries [q0, q0 + PF_QT) of one
// (head, sequence): score_j = (q . k_j) / sqrtf(hd) for j <= t, softmax,
// o = sum_j p_j v_j, keys and values read from ring slots 0..T-1. K / V tiles
// of 32 rows are double-buffered with cp.async (the next tile loads while the
// current one is used). The score and P.V products of each tile are
// register-tiled SIMT GEMMs on shared memory (scores: 4 queries x 2 keys per
// thread, four head elements per 128-bit load; P.V: 8 queries x hd/32
// elements per thread), and the softmax runs online over the tiles (running
// max and sum, rescaled), so its rounding differs from the reference's
// two-pass form within fp32 noise.
//
// MASKED: the allowed edges of prepare_attention_mask (src/core/transformer.c:
// 366-390) instead of the prefix lengths: key j is scored for query t when
// j <= t, both positions are real (pad [S][T], null = all) and the custom
// mask allows it (att [S][T][T], null = all); a query with no allowed key
// gets a zero output (attention_head_forward, :80-131).
template <int HDW, bool MASKED = false>   // head_dim / 32
__global__ void __launch_bounds__(PF_THREADS) dz_attention_prefill_kernel(
    const float* __restrict__ q, const float* __restrict__ keys, const float* __restrict__ values,
    const int* __restrict__ lens, float* __restrict__ out, int T, int dim, int capacity,
    const uint8_t* __restrict__ pad = nullptr, const uint8_t* __restrict__ att = nullptr) {
    constexpr int HD = HDW * 32;
    constexpr int LD = HD + 4;               // row stride of the Q / K / V tiles (floats)
    constexpr int CH = HD / 4;               // 16-byte chunks per row
    extern __shared__ __align__(16) float pf_smem[];
    float* qs = pf_smem;                     // [PF_QT][LD]
    float* kb = qs + PF_QT * LD;             // [2][PF_KT][LD]
    float* vb = kb + 2 * PF_KT * LD;         // [2][PF_KT][LD]
    float* pt = vb + 2 * PF_KT * LD;         // [PF_KT][PF_PLD] probabilities transposed
    float* corr_s = pt + PF_KT * PF_PLD;     // [PF_QT]
    float* m_s = corr_s + PF_QT;             // [PF_QT]
    float* l_s = m_s + PF_QT;                // [PF_QT]
    const int q0 = blockIdx.x * PF_QT, h = blockIdx.y, s = blockIdx.z;
    const int len = (!MASKED && lens) ? lens[s] : T;
    if (q0 >= len) return;
    const uint8_t* pad_s = (MASKED && pad) ? pad + (long long)s * T : nullptr;
    const uint8_t* att_s = (MASKED && att) ? att + (long long)s * T * T : nullptr;
    auto allowed = [&](int t, int j) -> bool {
        if (!(j <= t && t < len)) return false;
        if (MASKED) {
            if (pad_s && !(pad_s[t] && pad_s[j])) return false;
            if (att_s && !att_s[(long long)t * T + j]) return false;
        }
        return true;
    };
    const int tid = threadIdx.x;
    const float* K = keys + (long long)s * capacity * dim + h * HD;
    const float* Vv = values + (long long)s * capacity * dim + h * HD;
    const long long row0 = (long long)s * T;
    const int tq_last = min(q0 + PF_QT, len) - 1;
    auto load_tile = [&](int j0, int buf) {
        for (int i = tid; i < PF_KT * CH; i += PF_THREADS) {
            const int kj = i / CH, c = i - kj * CH;
            const int j = j0 + kj;
            const bool in = j <= tq_last;
            const int jj = in ? j : 0;
            pf_cp_async16(kb + (buf * PF_KT + kj) * LD + 4 * c, K + (long long)jj * dim + 4 * c, in);
            pf_cp_async16(vb + (buf * PF_KT + kj) * LD + 4 * c, Vv + (long long)jj * dim + 4 * c, in);
        }
        pf_cp_commit();
    };
    load_tile(0, 0);
    for (int i = tid; i < PF_QT * CH; i += PF_THREADS) {
        const int qi = i / CH, c = i - qi * CH;
        const int t = q0 + qi;
        const float4 v = t < len ? *reinterpret_cast<const float4*>(q + (row0 + t) * dim + h * HD + 4 * c)
                                 : make_float4(0.f, 0.f, 0.f, 0.f);
        *reinterpret_cast<float4*>(qs + qi * LD + 4 * c) = v;
    }
    if (tid < PF_QT) {
        m_s[tid] = -3.402823466e38f;
        l_s[tid] = 0.0f;
    }
    const float denom = sqrtf((float)HD);
    const int sqg = tid >> 4, skg = tid & 15;          // scores: 16 x 4 queries, 16 x 2 keys
    const int oqg = tid >> 5, oe = (tid & 31) * HDW;   // P.V: 8 x 8 queries, 32 x HDW elements
    float o[8][HDW];
#pragma unroll
    for (int i = 0; i < 8; i++)
#pragma unroll
        for (int c = 0; c < HDW; c++) o[i][c] = 0.0f;
    int buf = 0;
    for (int j0 = 0; j0 <= tq_last; j0 += PF_KT, buf ^= 1) {
        if (j0 + PF_KT <= tq_last) {
            load_tile(j0 + PF_KT, buf ^ 1);   // prefetch the next tile
            pf_cp_wait_all_but_one();
        } else {
            pf_cp_wait_all();
        }
        __syncthreads();   // tile `buf` landed for everyone; qs, m_s, l_s written
        const float* ks = kb + buf * PF_KT * LD;
        const float* vs = vb + buf * PF_KT * LD;
        float sc[4][2];
#pragma unroll
        for (int i = 0; i < 4; i++) sc[i][0] = sc[i][1] = 0.0f;
#pragma unroll 4
        for (int e = 0; e < HD; e += 4) {
            float4 qv[4], kv[2];
#pragma unroll
            for (int i = 0; i < 4; i++) qv[i] = *reinterpret_cast<const float4*>(qs + (sqg * 4 + i) * LD + e);
#pragma unroll
            for (int kk = 0; kk < 2; kk++) kv[kk] = *reinterpret_cast<const float4*>(ks + (skg * 2 + kk) * LD + e);
#pragma unroll
            for (int i = 0; i < 4; i++)
#pragma unroll
                for (int kk = 0; kk < 2; kk++) {
                    float a2 = sc[i][kk];
                    a2 = fmaf(qv[i].x, kv[kk].x, a2);
                    a2 = fmaf(qv[i].y, kv[kk].y, a2);
                    a2 = fmaf(qv[i].z, kv[kk].z, a2);
                    a2 = fmaf(qv[i].w, kv[kk].w, a2);
                    sc[i][kk] = a2;
                }
        }
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const int qi = sqg * 4 + i;
            const int t = q0 + qi;
            float tmax = -3.402823466e38f;
#pragma unroll
            for (int kk = 0; kk < 2; kk++) {
                const int j = j0 + skg * 2 + kk;
                sc[i][kk] = sc[i][kk] / denom;
                if (allowed(t, j)) tmax = fmaxf(tmax, sc[i][kk]);
            }
#pragma unroll
            for (int off = 8; off >= 1; off >>= 1) tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, off));
            const float mold = m_s[qi];
            const float mnew = fmaxf(mold, tmax);
            float ps = 0.0f;
#pragma unroll
            for (int kk = 0; kk < 2; kk++) {
                const int j = j0 + skg * 2 + kk;
                const float p = allowed(t, j) ? expf(sc[i][kk] - mnew) : 0.0f;
                pt[(skg * 2 + kk) * PF_PLD + qi] = p;
                ps += p;
            }
#pragma unroll
            for (int off = 8; off >= 1; off >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, off);
            __syncwarp();
            if (skg == 0) {
                const float cf = expf(mold - mnew);
                corr_s[qi] = cf;
                l_s[qi] = l_s[qi] * cf + ps;
                m_s[qi] = mnew;
            }
        }
        __syncthreads();
        float cf[8];
#pragma unroll
        for (int i = 0; i < 8; i++) cf[i] = corr_s[oqg * 8 + i];
#pragma unroll
        for (int i = 0; i < 8; i++)
#pragma unroll
            for (int c = 0; c < HDW; c++) o[i][c] *= cf[i];
        const int nk = min(PF_KT, tq_last - j0 + 1);
        for (int k = 0; k < nk; k++) {
            const float4 pa = *reinterpret_cast<const float4*>(pt + k * PF_PLD + oqg * 8);
            const float4 pb = *reinterpret_cast<const float4*>(pt + k * PF_PLD + oqg * 8 + 4);
            const float pr[8] = {pa.x, pa.y, pa.z, pa.w, pb.x, pb.y, pb.z, pb.w};
            float vv[HDW];
#pragma unroll
            for (int c = 0; c < HDW; c++) vv[c] = vs[k * LD + oe + c];
#pragma unroll
            for (int i = 0; i < 8; i++)
#pragma unroll
                for (int c = 0; c < HDW; c++) o[i][c] = fmaf(pr[i], vv[c], o[i][c]);
        }
        __syncthreads();   // pt, corr_s and tile `buf` consumed before they are rewritten
    }
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const int qi = oqg * 8 + i;
        const int t = q0 + qi;
        if (t >= len) continue;
        float* orow = out + (row0 + t) * dim + h * HD;
        if (MASKED && l_s[qi] == 0.0f) {   // no allowed key: the row stays zero
#pragma unroll
            for (int c = 0; c < HDW; c++) orow[oe + c] = 0.0f;
            continue;
        }
        const float inv = 1.0f / l_s[qi];
#pragma unroll
        for (int c = 0; c < HDW; c++) orow[oe + c] = o[i][c] * inv;
    }
}

// zero_padded_rows (src/core/transformer.c:355-363): rows r of [R][dim] whose
// padding entry pad[r] is 0 are set to zero. One block per row.
__global__ void dz_zero_padded_rows_kernel(float* __restrict__ x, const uint8_t* __restrict__ pad, int dim) {
    const long long r = blockIdx.x;
    if (pad[r]) return;
    for (int i = threadIdx.x; i < dim; i += blockDim.x) x[r * dim + i] = 0.0f;
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
