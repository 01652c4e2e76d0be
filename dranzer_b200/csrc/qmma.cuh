// Tensor-core building blocks for the quantized matvec / skinny GEMM.
//
// Weights live in an MMA-fragment layout: the matrix W[k x n] (the reference's
// storage, src/core/quantize.c:213-270) is cut into n-tiles of 16 output
// columns and k-groups of 64 (INT4) or 32 (INT8) rows. One k-group of one
// n-tile is a 512-byte chunk; lane l = 4g + t of a warp loads bytes
// [16l, 16l+16) and holds exactly the A fragments (rows = output columns n,
// columns = k) of the m16n8k16 f16 MMAs it takes part in:
//   a0 = (n=g, k=2t..2t+1)  a1 = (n=g+8, k=2t..2t+1)
//   a2 = (n=g, k=2t+8..9)   a3 = (n=g+8, k=2t+8..9)
// INT4: one 32-bit word per 16-row k-tile (4 per chunk); nibble p sits at
// n = g + 8(p&1), k = 2t + 8((p>>1)&1) + (p>>2), so a_r is nibbles (r, r+4).
// INT8: two words per k-tile (2 k-tiles per chunk); byte b of word h sits at
// n = g + 8(b>>1), k = 2t + 8h + (b&1), so a0/a1 are bytes (0,1)/(2,3) of
// word 0 and a2/a3 those of word 1. Codes are the reference's bits, reordered.
//
// Dequantization to exact fp16 integers (the classic magic-number trick):
// INT8  prmt(word, 0x64646464) puts byte c under 0x64 -> 1024 + c; minus
//       1151 gives c - 127.
// INT4  (w & 0x000F000F) | 0x64006400 -> 1024 + c; minus 1031 gives c - 7.
//       The nibbles at bits 4..7 of each half give 1024 + 16c; minus 1136
//       gives 16 (c - 7): those are the a1 / a3 rows (n = g + 8), whose sums
//       are scaled by 1/16 (exactly) afterwards.
// Activations: each row x is scaled by 2^s (exact) so that max |x 2^s| lies
// in [2^14, 2^15), then split into fp16 hi + mid + lo (11 significant bits
// each; 33 >= 24, so the split is exact except below 2^-24 absolute, i.e.
// 2^-38 of the row maximum). Products of small integers and fp16 parts are
// exact in the fp32 accumulator, so results carry fp32-level error like the
// reference's fp32 multiply-add; the 2^-s and the per-column scale are applied
// after the k-sum.
#pragma once
#include <cstdint>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "qmv.cuh"

namespace dz {

// k rows covered by one 512-byte chunk
template <int BITS>
struct FragGeom {
    static constexpr int KG = BITS == 8 ? 32 : 64;   // rows per chunk
    static constexpr int KT = KG / 16;               // k-tiles per chunk
};

// Reference storage -> fragment layout; one thread per output word. The
// destination's columns are the concatenation of up to three sources (column
// offsets off[0..nsrc]); entries past the last column or past K hold code
// qmax (level 0).
struct FragSources {
    const uint8_t* ref[3];
    int off[4];
    int nsrc;
};

__global__ void dz_frag_repack_kernel(FragSources src, uint32_t* __restrict__ out, int K, int bits, int nkg,
                                      long long nwords) {
    const long long wid = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (wid >= nwords) return;
    const int j = (int)(wid & 3);
    const int lane = (int)((wid >> 2) & 31);
    const long long chunk = wid >> 7;
    const int kg = (int)(chunk % nkg);
    const long long nt = chunk / nkg;
    const int g = lane >> 2, t = lane & 3;
    const int ntot = src.off[src.nsrc];
    const int fields = bits == 4 ? 8 : 4;
    uint32_t word = 0;
    for (int p = 0; p < fields; p++) {
        long long n, k;
        if (bits == 4) {
            n = nt * 16 + g + 8 * (p & 1);
            k = (long long)(kg * 4 + j) * 16 + 2 * t + 8 * ((p >> 1) & 1) + (p >> 2);
        } else {
            n = nt * 16 + g + 8 * (p >> 1);
            k = (long long)(kg * 2 + (j >> 1)) * 16 + 2 * t + 8 * (j & 1) + (p & 1);
        }
        uint32_t code = bits == 8 ? 127u : 7u;
        if (n < ntot && k < K) {
            int i = 0;
            while (i + 1 < src.nsrc && n >= src.off[i + 1]) i++;
            const long long N = src.off[i + 1] - src.off[i];
            const long long idx = k * N + (n - src.off[i]);
            const uint8_t* ref = src.ref[i];
            code = bits == 8 ? ref[idx] : (uint32_t)((ref[idx >> 1] >> ((idx & 1) * 4)) & 0xF);
        }
        word |= code << ((bits == 4 ? 4 : 8) * p);
    }
    out[wid] = word;
}

// Code at (k, n) from the fragment layout.
__device__ __forceinline__ uint32_t dz_frag_code(const uint8_t* codes, int bits, int nkg, long long k, long long n) {
    const long long nt = n >> 4;
    const int nl = (int)(n & 15);
    const int kg = (int)(k / (bits == 8 ? 32 : 64));
    const int kin = (int)(k % (bits == 8 ? 32 : 64));
    const int kt = kin >> 4, kk = kin & 15;
    const int g = nl & 7, hi_row = nl >> 3;
    const int t = (kk & 7) >> 1, odd = kk & 1, hi_k = kk >> 3;
    const int lane = g * 4 + t;
    const uint32_t* chunk = reinterpret_cast<const uint32_t*>(codes) + ((nt * nkg + kg) * 128 + lane * 4);
    if (bits == 4) return (chunk[kt] >> (4 * (hi_row + 2 * hi_k + 4 * odd))) & 0xF;
    return (chunk[kt * 2 + hi_k] >> (8 * (hi_row * 2 + odd))) & 0xFF;
}

// Fragment layout -> reference storage (bit-exact inverse), one thread per byte.
__global__ void dz_frag_unrepack_kernel(const uint8_t* __restrict__ codes, uint8_t* __restrict__ ref, int K, int N,
                                        int bits, int nkg, long long nbytes) {
    const long long b = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= nbytes) return;
    const long long total = (long long)K * N;
    if (bits == 8) {
        ref[b] = (uint8_t)dz_frag_code(codes, 8, nkg, b / N, b % N);
    } else {
        const long long i0 = 2 * b, i1 = 2 * b + 1;
        const uint32_t lo = dz_frag_code(codes, 4, nkg, i0 / N, i0 % N);
        const uint32_t hi = i1 < total ? dz_frag_code(codes, 4, nkg, i1 / N, i1 % N) : 0u;
        ref[b] = (uint8_t)(lo | (hi << 4));
    }
}

// quantize_unpack (src/core/quantize.c:290-295) from the fragment layout.
__global__ void dz_frag_dequant_kernel(const uint8_t* __restrict__ codes, const float* __restrict__ scales, int gran,
                                       float* __restrict__ dst, int K, int N, int bits, int nkg) {
    const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= (long long)K * N) return;
    const long long k = idx / N, n = idx % N;
    const int qmax = bits == 8 ? 127 : 7;
    const uint32_t code = dz_frag_code(codes, bits, nkg, k, n);
    const float s = gran == 2 ? scales[n] : gran == 1 ? scales[k] : scales[0];
    dst[idx] = s * (float)((int)code - qmax);
}

// ---------------------------------------------------------------- math

__device__ __forceinline__ uint32_t dz_hsub2(uint32_t a, uint32_t b) {
    __half2 x = *reinterpret_cast<__half2*>(&a);
    __half2 y = *reinterpret_cast<__half2*>(&b);
    __half2 r = __hsub2(x, y);
    return *reinterpret_cast<uint32_t*>(&r);
}

constexpr uint32_t DZ_F16X2_1024 = 0x64006400u;   // 1024.0 in both halves
constexpr uint32_t DZ_F16X2_1031 = 0x64076407u;   // 1024 + 7
constexpr uint32_t DZ_F16X2_1136 = 0x64706470u;   // 1024 + 16 * 7
constexpr uint32_t DZ_F16X2_1151 = 0x647F647Fu;   // 1024 + 127

// The four A-fragment registers of one INT4 k-tile word; a1 and a3 carry 16x.
__device__ __forceinline__ void dz_deq4(uint32_t w, uint32_t (&a)[4]) {
    const uint32_t u = w >> 8;
    a[0] = dz_hsub2((w & 0x000F000Fu) | DZ_F16X2_1024, DZ_F16X2_1031);
    a[1] = dz_hsub2((w & 0x00F000F0u) | DZ_F16X2_1024, DZ_F16X2_1136);
    a[2] = dz_hsub2((u & 0x000F000Fu) | DZ_F16X2_1024, DZ_F16X2_1031);
    a[3] = dz_hsub2((u & 0x00F000F0u) | DZ_F16X2_1024, DZ_F16X2_1136);
}

// The four A-fragment registers of one INT8 k-tile (words w0, w1).
__device__ __forceinline__ void dz_deq8(uint32_t w0, uint32_t w1, uint32_t (&a)[4]) {
    a[0] = dz_hsub2(__byte_perm(w0, 0x64646464u, 0x4140), DZ_F16X2_1151);
    a[1] = dz_hsub2(__byte_perm(w0, 0x64646464u, 0x4342), DZ_F16X2_1151);
    a[2] = dz_hsub2(__byte_perm(w1, 0x64646464u, 0x4140), DZ_F16X2_1151);
    a[3] = dz_hsub2(__byte_perm(w1, 0x64646464u, 0x4342), DZ_F16X2_1151);
}

// D += A (16 x 16, f16, row) . B (16 x 8, f16, col), fp32 accumulate.
__device__ __forceinline__ void dz_mma_f16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Exponent shift s for a row whose largest magnitude is amax: max |x 2^s| in
// [2^14, 2^15). Zero, inf and NaN rows take s = 0.
__device__ __forceinline__ int dz_row_shift(float amax) {
    if (!(amax > 0.0f) || !(amax <= 3.402823466e38f)) return 0;
    return 14 - ilogbf(amax);
}

// fp16 hi / mid / lo of v (already scaled); hi + mid + lo == v exactly for
// |v| >= 2^-1 (and to 2^-25 absolute below).
struct DzSplit3 {
    __half h, m, l;
};
__device__ __forceinline__ DzSplit3 dz_split3(float v) {
    DzSplit3 r;
    r.h = __float2half_rn(v);
    const float r1 = v - __half2float(r.h);
    r.m = __float2half_rn(r1);
    r.l = __float2half_rn(r1 - __half2float(r.m));
    return r;
}

__device__ __forceinline__ uint32_t dz_pack_h2(__half lo, __half hi) {
    return (uint32_t)__half_as_ushort(lo) | ((uint32_t)__half_as_ushort(hi) << 16);
}

// ------------------------------------------------------ the global kernels

// Split activations in B-fragment order. For row pair u of the M rows and a
// k-group kg, lane l = 4g + t of a warp holds the words its m16n8k16 B
// fragments need: B column g is row 2u + g/4, part g%4 (hi, mid, lo; 3 = zero),
// and per k-tile kt the words are (k0+2t, k0+2t+1) and (k0+8+2t, k0+9+2t):
//   XF[((kg * nbt + u) * 32 + l) * 2KT + 2kt + j]
// so one chunk's B fragments are one (INT8) or two (INT4) 16-byte loads.
// One block per row: the row maximum sets the row's exponent shift (stored
// negated in row_shift, to undo after the k-sum), then every pair of elements
// is split. ROW-granularity scales (k_scale) are folded in first.
__global__ void __launch_bounds__(256) dz_split_rows_kernel(const float* __restrict__ X, long long ldx,
                                                            const float* __restrict__ k_scale, int M, int K, int KT,
                                                            int nkg, int nbt, uint32_t* __restrict__ XF,
                                                            int* __restrict__ row_shift) {
    const int r = blockIdx.x;
    const float* x = X + (long long)r * ldx;
    __shared__ float wmax[8];
    __shared__ int sh_s;
    float m = 0.0f;
    for (int k = threadIdx.x; k < K; k += blockDim.x) {
        float v = x[k];
        if (k_scale) v *= k_scale[k];
        m = fmaxf(m, fabsf(v));
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
    if ((threadIdx.x & 31) == 0) wmax[threadIdx.x >> 5] = m;
    __syncthreads();
    if (threadIdx.x == 0) {
        float a = 0.0f;
        for (int w = 0; w < (int)(blockDim.x >> 5); w++) a = fmaxf(a, wmax[w]);
        sh_s = dz_row_shift(a);
        row_shift[r] = -sh_s;
    }
    __syncthreads();
    const int sh = sh_s;
    const int u = r >> 1, rh = r & 1;
    const bool pad_next = (r == M - 1) && (M & 1);   // this block also zeroes the phantom row
    const long long pairs = (long long)nkg * KT * 8;
    for (long long q = threadIdx.x; q < pairs; q += blockDim.x) {
        const long long k = 2 * q;
        const int kg = (int)(k / (16 * KT));
        const int kt = (int)((k / 16) % KT);
        const int kk = (int)(k & 15);
        const int j = kk >> 3, t = (kk & 7) >> 1;
        float v0 = 0.0f, v1 = 0.0f;
        if (k < K) {
            v0 = x[k];
            if (k_scale) v0 *= k_scale[k];
        }
        if (k + 1 < K) {
            v1 = x[k + 1];
            if (k_scale) v1 *= k_scale[k + 1];
        }
        const DzSplit3 s0 = dz_split3(ldexpf(v0, sh)), s1 = dz_split3(ldexpf(v1, sh));
        const long long base = (((long long)kg * nbt + u) * 32) * 2 * KT + 2 * kt + j;
        const int g0 = rh * 4;
        XF[base + (long long)((g0 + 0) * 4 + t) * 2 * KT] = dz_pack_h2(s0.h, s1.h);
        XF[base + (long long)((g0 + 1) * 4 + t) * 2 * KT] = dz_pack_h2(s0.m, s1.m);
        XF[base + (long long)((g0 + 2) * 4 + t) * 2 * KT] = dz_pack_h2(s0.l, s1.l);
        XF[base + (long long)((g0 + 3) * 4 + t) * 2 * KT] = 0u;
        if (pad_next) {
#pragma unroll
            for (int sp = 0; sp < 4; sp++) XF[base + (long long)((4 + sp) * 4 + t) * 2 * KT] = 0u;
        }
    }
}

struct QmmArgs {
    const uint8_t* codes;     // fragment layout
    int K, N, nkg, ntiles;
    const uint32_t* XF;       // split activations in B-fragment order (dz_split_rows_kernel)
    int nbt;                  // row pairs in XF
    int M;
    int kparts;               // warps splitting the k-groups of one unit
    int kg_per_part;
    int n_groups;             // n-tile groups of NT tiles
    int m_passes;             // row passes of 2*NB rows
    QmvEpilogue ep;
};

// Combine one lane's accumulators for row pair u: the lane pair (t, t^1)
// holds hi+mid and lo of one row (t even: row 2u, t = 2: row 2u+1); outputs
// n+8 of INT4 carry 16x.
template <int BITS>
__device__ __forceinline__ void dz_combine(const float (&d)[4], float& lo_n, float& hi_n) {
    lo_n = d[0] + d[1];
    hi_n = d[2] + d[3];
    lo_n += __shfl_xor_sync(0xffffffffu, lo_n, 1);
    hi_n += __shfl_xor_sync(0xffffffffu, hi_n, 1);
    if (BITS == 4) hi_n *= 0.0625f;
}

// B fragment words (2kt, 2kt+1) from a lane's 16-byte XF loads.
__device__ __forceinline__ uint32_t dz_xw(const uint4* xv, int i) {
    const uint4 q = xv[i >> 2];
    switch (i & 3) {
        case 0: return q.x;
        case 1: return q.y;
        case 2: return q.z;
        default: return q.w;
    }
}

// Y = epilogue(X . deq(W)) on tensor cores for any M (used above the
// streaming kernel's row limit). A warp owns NT n-tiles x 2*NB rows over a
// range of k-groups; weight fragments are loaded one k-group ahead.
template <int BITS, int NB, int NT>
__global__ void __launch_bounds__(QMV_THREADS) dz_qmm_kernel(QmmArgs a) {
    constexpr int KT = FragGeom<BITS>::KT;
    constexpr int XV = KT / 2;                     // 16-byte B loads per (chunk, row pair)
    constexpr int NV = NT * NB * 2;                // combined outputs per lane
    __shared__ float red[QMV_WARPS][NV][32];

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, t = lane & 3;
    const int units_per_cta = QMV_WARPS / a.kparts;
    const int unit = blockIdx.x * units_per_cta + warp / a.kparts;
    const int kpart = warp % a.kparts;
    const bool active = unit < a.n_groups * a.m_passes;
    const int group = active ? unit % a.n_groups : 0;
    const int mpass = active ? unit / a.n_groups : 0;
    const int kg0 = kpart * a.kg_per_part;
    const int kg1 = min(kg0 + a.kg_per_part, a.nkg);

    float acc[NT][NB][4];
#pragma unroll
    for (int i = 0; i < NT; i++)
#pragma unroll
        for (int u = 0; u < NB; u++)
#pragma unroll
            for (int q = 0; q < 4; q++) acc[i][u][q] = 0.0f;

    const uint4* xf4 = reinterpret_cast<const uint4*>(a.XF);
    const uint4 pad = BITS == 8 ? make_uint4(0x7F7F7F7Fu, 0x7F7F7F7Fu, 0x7F7F7F7Fu, 0x7F7F7F7Fu)
                                : make_uint4(0x77777777u, 0x77777777u, 0x77777777u, 0x77777777u);
    auto load_group = [&](int kg, uint4 (&w)[NT]) {
#pragma unroll
        for (int i = 0; i < NT; i++) {
            const int nt = group * NT + i;
            w[i] = nt < a.ntiles
                       ? __ldg(reinterpret_cast<const uint4*>(a.codes + ((long long)nt * a.nkg + kg) * 512) + lane)
                       : pad;
        }
    };
    if (active && kg0 < kg1) {
        uint4 wcur[NT], wnext[NT];
        load_group(kg0, wcur);
        for (int kg = kg0; kg < kg1; kg++) {
            if (kg + 1 < kg1) load_group(kg + 1, wnext);
            uint4 xv[NB][XV];
#pragma unroll
            for (int u = 0; u < NB; u++) {
                const int ug = mpass * NB + u;
#pragma unroll
                for (int h = 0; h < XV; h++)
                    xv[u][h] = ug < a.nbt ? __ldg(xf4 + (((long long)kg * a.nbt + ug) * 32 + lane) * XV + h)
                                          : make_uint4(0u, 0u, 0u, 0u);
            }
#pragma unroll
            for (int kt = 0; kt < KT; kt++) {
#pragma unroll
                for (int i = 0; i < NT; i++) {
                    const uint32_t ww[4] = {wcur[i].x, wcur[i].y, wcur[i].z, wcur[i].w};
                    uint32_t af[4];
                    if (BITS == 4) dz_deq4(ww[kt], af);
                    else dz_deq8(ww[2 * kt], ww[2 * kt + 1], af);
#pragma unroll
                    for (int u = 0; u < NB; u++)
                        dz_mma_f16(acc[i][u], af, dz_xw(xv[u], 2 * kt), dz_xw(xv[u], 2 * kt + 1));
                }
            }
            if (kg + 1 < kg1) {
#pragma unroll
                for (int i = 0; i < NT; i++) wcur[i] = wnext[i];
            }
        }
    }

    float v[NV];
#pragma unroll
    for (int i = 0; i < NT; i++)
#pragma unroll
        for (int u = 0; u < NB; u++)
            dz_combine<BITS>(acc[i][u], v[(i * NB + u) * 2 + 0], v[(i * NB + u) * 2 + 1]);
    if (a.kparts > 1) {
#pragma unroll
        for (int q = 0; q < NV; q++) red[warp][q][lane] = v[q];
        __syncthreads();
        if (kpart != 0) return;
#pragma unroll
        for (int q = 0; q < NV; q++) {
            float s = 0.0f;
            for (int p = 0; p < a.kparts; p++) s += red[warp + p][q][lane];
            v[q] = s;
        }
    }
    if (!active || (t & 1)) return;
#pragma unroll
    for (int i = 0; i < NT; i++)
#pragma unroll
        for (int u = 0; u < NB; u++) {
            const int row = (mpass * NB + u) * 2 + (t >> 1);
            const int n = (group * NT + i) * 16 + g;
            dz_qmv_store_row(a.ep, a.M, a.N, row, n, v[(i * NB + u) * 2 + 0]);
            dz_qmv_store_row(a.ep, a.M, a.N, row, n + 8, v[(i * NB + u) * 2 + 1]);
        }
}

// ------------------------------------------------ streaming (TMA) kernel

__device__ __forceinline__ uint32_t dz_smem_addr(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ uint64_t dz_global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// mbarrier helpers (count-1 barriers completed by expect_tx + bulk copies)
__device__ __forceinline__ void dz_mbar_init(uint64_t* bar) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(dz_smem_addr(bar)) : "memory");
}
__device__ __forceinline__ void dz_mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(dz_smem_addr(bar)), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ bool dz_mbar_test(uint64_t* bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(dz_smem_addr(bar)), "r"(parity)
        : "memory");
    return done != 0;
}
// Bounded wait (about one second). False when it gave up.
__device__ __forceinline__ bool dz_mbar_wait(uint64_t* bar, uint32_t parity) {
    const uint64_t t0 = dz_global_ns();
    for (unsigned i = 0;; i++) {
        if (dz_mbar_test(bar, parity)) return true;
        if ((i & 255u) == 255u && dz_global_ns() - t0 > 1000000000ull) return false;
    }
}
__device__ __forceinline__ void dz_bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            dz_smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(dz_smem_addr(bar))
        : "memory");
}

constexpr int QMS_STAGES = 3;   // ring stages per warp

struct QmsArgs {
    const uint8_t* codes;     // fragment layout
    int N, nkg, ntiles;
    const uint32_t* XF;       // split activations in B-fragment order (dz_split_rows_kernel)
    int nbt;                  // row pairs in XF
    int M;
    int kparts;               // warps sharing one n-group's k-groups (1, 2, 4 or 8)
    int per;                  // k-groups per k-part
    int n_groups;             // groups of NT n-tiles
    int nrounds;              // rounds of QMV_WARPS / kparts n-groups
    int pk;                   // k-groups per piece (a stage holds NT * pk chunks)
    unsigned xf_bytes;        // XF bytes copied to shared memory (XSM kernels)
    int* status;              // set to 1 when a copy wait gave up (may be null)
    QmvEpilogue ep;
};

// One piece of a warp's stream: n-group ng (n-tiles NT*ng ..), k-groups
// [kg0, kg0 + nkg).
struct QmsPiece {
    int ng, kg0, nkg;
    bool first, last;
};

// Piece idx of warp `warp`: round r = blockIdx.x + (idx / ppr) * gridDim.x owns
// n-groups r * (QMV_WARPS / kparts) + [0, QMV_WARPS / kparts); the warp takes
// n-group warp / kparts, k-part warp % kparts, in pieces of pk k-groups.
__device__ __forceinline__ QmsPiece dz_qms_piece(const QmsArgs& a, int warp, int ppr, int idx) {
    QmsPiece p;
    const int j = idx / ppr, q = idx - j * ppr;
    const long long r = blockIdx.x + (long long)j * gridDim.x;
    p.ng = (int)(r * (QMV_WARPS / a.kparts) + warp / a.kparts);
    const int kstart = (warp % a.kparts) * a.per;
    const int kend = min(kstart + a.per, a.nkg);
    p.kg0 = kstart + q * a.pk;
    p.nkg = p.ng < a.n_groups ? max(0, min(a.pk, kend - p.kg0)) : 0;
    p.first = q == 0;
    p.last = q == ppr - 1;
    return p;
}

// Shared memory of dz_qms_kernel: the rings, the XF copy, the k-part
// reduction area and the barriers.
__host__ __device__ constexpr size_t dz_qms_ring_bytes(int pk, int NT) {
    return (size_t)QMV_WARPS * QMS_STAGES * NT * pk * 512;
}
__host__ __device__ constexpr size_t dz_qms_smem_bytes(int pk, int NT, int NB, unsigned xf_bytes) {
    return dz_qms_ring_bytes(pk, NT) + xf_bytes + (size_t)QMV_WARPS * NT * NB * 2 * 32 * 4 +
           ((size_t)QMV_WARPS * QMS_STAGES + 1) * 8;
}

// Y = epilogue(X . deq(W)) for M <= 2 * NB rows, streaming the weights. One
// persistent CTA per SM; each warp streams its pieces (NT n-tiles x pk
// k-groups) through its own QMS_STAGES-deep shared-memory ring with bulk
// copies, lane 0 keeping two pieces in flight. With XSM the activations'
// B fragments are copied to shared memory once per CTA; otherwise they are
// read through L1. Each chunk is dequantized from shared memory into fp16
// A fragments (dz_deq4 / dz_deq8) feeding NB MMAs per n-tile; CH independent
// accumulator chains per (n-tile, row pair) keep the tensor pipe busy when
// NT * NB is small. The k-parts of an n-group are summed in shared memory in
// k-part order, so results do not depend on the grid.
template <int BITS, int NB, int NT, bool XSM>
__global__ void __launch_bounds__(QMV_THREADS, 1) dz_qms_kernel(QmsArgs a) {
    constexpr int KT = FragGeom<BITS>::KT;
    constexpr int XV = KT / 2;
    constexpr int CH = NT * NB >= 4 ? 1 : (4 / (NT * NB) < KT ? 4 / (NT * NB) : KT);
    constexpr int NV = NT * NB * 2;
    extern __shared__ __align__(128) unsigned char qms_smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, t = lane & 3;
    const int stage_bytes = NT * a.pk * 512;
    uint8_t* ring = qms_smem + (size_t)warp * QMS_STAGES * stage_bytes;
    uint8_t* xf_sm = qms_smem + dz_qms_ring_bytes(a.pk, NT);
    float* red = reinterpret_cast<float*>(xf_sm + a.xf_bytes);
    uint64_t* bars = reinterpret_cast<uint64_t*>(red + QMV_WARPS * NV * 32);
    uint64_t* xbar = bars + QMV_WARPS * QMS_STAGES;
    bars += warp * QMS_STAGES;

    const int ppr = (a.per + a.pk - 1) / a.pk;
    const int rounds_here =
        (int)blockIdx.x < a.nrounds ? (a.nrounds - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
    const int npieces = rounds_here * ppr;

    if (lane == 0) {
        for (int st = 0; st < QMS_STAGES; st++) dz_mbar_init(&bars[st]);
        if (XSM && warp == 0) dz_mbar_init(xbar);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (XSM) {
        __syncthreads();   // xbar initialised before anyone waits on it
        if (threadIdx.x == 0) {
            dz_mbar_expect_tx(xbar, a.xf_bytes);
            for (unsigned off = 0; off < a.xf_bytes; off += 32768u) {
                const unsigned n = a.xf_bytes - off < 32768u ? a.xf_bytes - off : 32768u;
                dz_bulk_g2s(xf_sm + off, reinterpret_cast<const uint8_t*>(a.XF) + off, n, xbar);
            }
        }
    } else {
        __syncwarp();
    }

    // lane 0: put piece idx in flight into stage idx % QMS_STAGES
    auto issue = [&](int idx) {
        const QmsPiece pc = dz_qms_piece(a, warp, ppr, idx);
        uint64_t* bar = &bars[idx % QMS_STAGES];
        int tiles = 0;
        for (int i = 0; i < NT; i++) tiles += pc.ng * NT + i < a.ntiles ? 1 : 0;
        if (pc.nkg == 0 || tiles == 0) {
            asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(dz_smem_addr(bar)) : "memory");
            return;
        }
        const uint32_t bytes = (uint32_t)pc.nkg * 512u;
        dz_mbar_expect_tx(bar, bytes * tiles);
        uint8_t* dst = ring + (idx % QMS_STAGES) * stage_bytes;
        for (int i = 0; i < tiles; i++)
            dz_bulk_g2s(dst + (size_t)i * a.pk * 512,
                        a.codes + ((size_t)(pc.ng * NT + i) * a.nkg + pc.kg0) * 512, bytes, bar);
    };
    int issued = min(npieces, QMS_STAGES - 1);
    if (lane == 0)
        for (int i = 0; i < issued; i++) issue(i);

    bool failed = false;
    int failed_at = -1;   // first piece whose wait gave up
    if (XSM) {
        int ok = 1;
        if (lane == 0) ok = dz_mbar_wait(xbar, 0) ? 1 : 0;
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!ok) {
            failed = true;
            failed_at = 0;
            if (lane == 0 && a.status) atomicExch(a.status, 1);
        }
    }
    const uint4* xf4 = XSM ? reinterpret_cast<const uint4*>(xf_sm) : reinterpret_cast<const uint4*>(a.XF);

    float acc[CH][NT][NB][4];
    for (int idx = 0; idx < npieces; idx++) {
        const QmsPiece pc = dz_qms_piece(a, warp, ppr, idx);
        if (pc.first) {
#pragma unroll
            for (int c = 0; c < CH; c++)
#pragma unroll
                for (int i = 0; i < NT; i++)
#pragma unroll
                    for (int u = 0; u < NB; u++)
#pragma unroll
                        for (int q = 0; q < 4; q++) acc[c][i][u][q] = 0.0f;
        }
        // refill the stage every lane finished with in the previous iteration
        if (!failed && issued < npieces) {
            if (lane == 0) issue(issued);
            issued++;
        }
        const int stage = idx % QMS_STAGES;
        if (!failed) {
            int ok = 1;
            if (lane == 0) ok = dz_mbar_wait(&bars[stage], (uint32_t)((idx / QMS_STAGES) & 1)) ? 1 : 0;
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (!ok) {
                failed = true;
                failed_at = idx;
                if (lane == 0 && a.status) atomicExch(a.status, 1);
            }
        }
        if (!failed) {
            const uint4* w4 = reinterpret_cast<const uint4*>(ring + stage * stage_bytes);
            for (int c = 0; c < pc.nkg; c++) {
                const int kg = pc.kg0 + c;
                uint4 xv[NB][XV];
#pragma unroll
                for (int u = 0; u < NB; u++)
#pragma unroll
                    for (int h = 0; h < XV; h++) {
                        const long long at = (((long long)kg * a.nbt + u) * 32 + lane) * XV + h;
                        xv[u][h] = u < a.nbt ? (XSM ? xf4[at] : __ldg(xf4 + at)) : make_uint4(0u, 0u, 0u, 0u);
                    }
                uint4 w[NT];
#pragma unroll
                for (int i = 0; i < NT; i++) w[i] = w4[(i * a.pk + c) * 32 + lane];
#pragma unroll
                for (int kt = 0; kt < KT; kt++) {
#pragma unroll
                    for (int i = 0; i < NT; i++) {
                        const uint32_t ww[4] = {w[i].x, w[i].y, w[i].z, w[i].w};
                        uint32_t af[4];
                        if (BITS == 4) dz_deq4(ww[kt], af);
                        else dz_deq8(ww[2 * kt], ww[2 * kt + 1], af);
#pragma unroll
                        for (int u = 0; u < NB; u++)
                            dz_mma_f16(acc[kt % CH][i][u], af, dz_xw(xv[u], 2 * kt), dz_xw(xv[u], 2 * kt + 1));
                    }
                }
            }
        }
        __syncwarp();   // the stage is free for lane 0 to refill
        if (!pc.last) continue;

        // this round's n-group is done: combine chains and split columns, then k-parts
        float v[NV];
#pragma unroll
        for (int i = 0; i < NT; i++)
#pragma unroll
            for (int u = 0; u < NB; u++) {
                float d[4];
#pragma unroll
                for (int q = 0; q < 4; q++) {
                    d[q] = acc[0][i][u][q];
#pragma unroll
                    for (int c = 1; c < CH; c++) d[q] += acc[c][i][u][q];
                }
                dz_combine<BITS>(d, v[(i * NB + u) * 2], v[(i * NB + u) * 2 + 1]);
            }
        if (failed) {
#pragma unroll
            for (int q = 0; q < NV; q++) v[q] = __int_as_float(0x7fc00000);   // a failed tile reads NaN
        }
        bool owner = true;
        if (a.kparts > 1) {
#pragma unroll
            for (int q = 0; q < NV; q++) red[(warp * NV + q) * 32 + lane] = v[q];
            __syncthreads();
            owner = warp % a.kparts == 0;
            if (owner) {
#pragma unroll
                for (int q = 0; q < NV; q++) {
                    float sum = 0.0f;
                    for (int kp = 0; kp < a.kparts; kp++) sum += red[((warp + kp) * NV + q) * 32 + lane];
                    v[q] = sum;
                }
            }
            __syncthreads();
        }
        if (owner && pc.ng < a.n_groups && !(t & 1)) {
#pragma unroll
            for (int i = 0; i < NT; i++)
#pragma unroll
                for (int u = 0; u < NB; u++) {
                    const int row = 2 * u + (t >> 1);
                    const int n = (pc.ng * NT + i) * 16 + g;
                    if (n < a.ntiles * 16) {
                        dz_qmv_store_row(a.ep, a.M, a.N, row, n, v[(i * NB + u) * 2]);
                        dz_qmv_store_row(a.ep, a.M, a.N, row, n + 8, v[(i * NB + u) * 2 + 1]);
                    }
                }
        }
    }
    if (failed_at >= 0 && lane == 0) {
        // copies still in flight land before the shared memory is released
        if (XSM && warp == 0) dz_mbar_wait(xbar, 0);
        for (int i = failed_at; i < issued; i++)
            if (!dz_mbar_wait(&bars[i % QMS_STAGES], (uint32_t)((i / QMS_STAGES) & 1))) break;
    }
}

}  // namespace dz
