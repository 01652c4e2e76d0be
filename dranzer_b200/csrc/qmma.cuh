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

// Linkage of the non-template kernels defined in these headers: external in
// the translation unit that launches them (dz_cuda.cu); a unit that includes
// the headers only for their device helpers (qmvi.cu) defines it as static.
#ifndef DZ_KERNEL_LINKAGE
#define DZ_KERNEL_LINKAGE
#endif

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

DZ_KERNEL_LINKAGE __global__ void dz_frag_repack_kernel(FragSources src, uint32_t* __restrict__ out, int K, int bits, int nkg,
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
DZ_KERNEL_LINKAGE __global__ void dz_frag_unrepack_kernel(const uint8_t* __restrict__ codes, uint8_t* __restrict__ ref, int K, int N,
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
DZ_KERNEL_LINKAGE __global__ void dz_frag_dequant_kernel(const uint8_t* __restrict__ codes, const float* __restrict__ scales, int gran,
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

// floor(log2 |v|) of a finite non-zero float, read from its bit fields
// (normal: biased exponent - 127; subnormal: the mantissa's top bit - 149).
// Kept inline so that no kernel depends on how a library call is inlined.
__device__ __forceinline__ int dz_ilogb(float v) {
    const uint32_t u = __float_as_uint(v) & 0x7fffffffu;
    const int e = (int)(u >> 23);
    return e ? e - 127 : (31 - __clz((int)u)) - 149;
}

// Exponent shift s for a row whose largest magnitude is amax: max |x 2^s| in
// [2^14, 2^15). Zero, inf and NaN rows take s = 0.
__device__ __forceinline__ int dz_row_shift(float amax) {
    if (!(amax > 0.0f) || !(amax <= 3.402823466e38f)) return 0;
    return 14 - ilogbf(amax);
}

// v * 2^e, exact unless the result is subnormal (e in [-300, 300]).
__device__ __forceinline__ float dz_mul_pow2(float v, int e) {
    if (e >= -126 && e <= 127) return v * __int_as_float((e + 127) << 23);
    const int h = e / 2;
    return (v * __int_as_float((h + 127) << 23)) * __int_as_float((e - h + 127) << 23);
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
// ROW-granularity scales (k_scale) are folded in first.

// Largest |x k_scale| of a row, block-wide (every thread gets it); `wred`
// holds one float per warp.
__device__ __forceinline__ float dz_row_amax(const float* __restrict__ x, const float* __restrict__ k_scale, int K,
                                             float* wred) {
    float m = 0.0f;
#pragma unroll 8
    for (int k = threadIdx.x; k < K; k += blockDim.x) {
        float v = x[k];
        if (k_scale) v *= k_scale[k];
        m = fmaxf(m, fabsf(v));
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
    __syncthreads();   // wred may still be read by a previous call
    if ((threadIdx.x & 31) == 0) wred[threadIdx.x >> 5] = m;
    __syncthreads();
    float a = 0.0f;
    for (int w = 0; w < (int)(blockDim.x >> 5); w++) a = fmaxf(a, wred[w]);
    return a;
}

// Store the XF words of element pair q (k = 2q, 2q+1, values v0, v1 already
// scaled by k_scale) of row r with exponent shift sh.
template <int KT>
__device__ __forceinline__ void dz_split_store_pair(uint32_t* __restrict__ XF, int nbt, int M, int r, int q, float v0,
                                                    float v1, int sh) {
    const int k = 2 * q;
    const int kg = k / (16 * KT);   // KT is 2 or 4: shifts
    const int kt = (k >> 4) & (KT - 1);
    const int kk = k & 15;
    const int j = kk >> 3, t = (kk & 7) >> 1;
    const DzSplit3 s0 = dz_split3(dz_mul_pow2(v0, sh)), s1 = dz_split3(dz_mul_pow2(v1, sh));
    uint32_t* base = XF + ((size_t)kg * nbt + (r >> 1)) * 32 * 2 * KT + 2 * kt + j;
    const int g0 = (r & 1) * 4;
    base[((g0 + 0) * 4 + t) * 2 * KT] = dz_pack_h2(s0.h, s1.h);
    base[((g0 + 1) * 4 + t) * 2 * KT] = dz_pack_h2(s0.m, s1.m);
    base[((g0 + 2) * 4 + t) * 2 * KT] = dz_pack_h2(s0.l, s1.l);
    base[((g0 + 3) * 4 + t) * 2 * KT] = 0u;
    if (r == M - 1 && (M & 1)) {   // the phantom row after an odd last row reads zero
#pragma unroll
        for (int sp = 0; sp < 4; sp++) base[((4 + sp) * 4 + t) * 2 * KT] = 0u;
    }
}

// Element k of row x with its ROW-granularity scale, zero past K.
__device__ __forceinline__ float dz_x_at(const float* __restrict__ x, const float* __restrict__ k_scale, int K,
                                         int k) {
    if (k >= K) return 0.0f;
    float v = x[k];
    if (k_scale) v *= k_scale[k];
    return v;
}

// Block-wide split of a row into XF (shared or global memory) with every
// element pair held in registers: thread j takes pairs j + i * blockDim.x,
// i < PMAX, so the row is read once with all loads in flight. Needs
// pairs <= PMAX * blockDim.x. dz_split_row_load issues the loads;
// dz_split_row_store finds the row maximum and writes the parts (thread 0
// stores the negated shift).
template <int PMAX>
__device__ __forceinline__ void dz_split_row_load(const float* __restrict__ x, const float* __restrict__ k_scale,
                                                  int K, float (&v)[PMAX][2]) {
#pragma unroll
    for (int i = 0; i < PMAX; i++) {
        const int q = threadIdx.x + i * blockDim.x;
        v[i][0] = dz_x_at(x, k_scale, K, 2 * q);
        v[i][1] = dz_x_at(x, k_scale, K, 2 * q + 1);
    }
}

template <int PMAX, int KT>
__device__ __forceinline__ void dz_split_row_store(const float (&v)[PMAX][2], int r, int M, int pairs, int nbt,
                                                   uint32_t* __restrict__ XF, int* __restrict__ shifts, float* wred) {
    float m = 0.0f;
#pragma unroll
    for (int i = 0; i < PMAX; i++) m = fmaxf(m, fmaxf(fabsf(v[i][0]), fabsf(v[i][1])));
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
    __syncthreads();   // wred may still be read for the previous row
    if ((threadIdx.x & 31) == 0) wred[threadIdx.x >> 5] = m;
    __syncthreads();
    float amax = 0.0f;
    for (int w = 0; w < (int)(blockDim.x >> 5); w++) amax = fmaxf(amax, wred[w]);
    const int sh = dz_row_shift(amax);
    if (threadIdx.x == 0) shifts[r] = -sh;
#pragma unroll
    for (int i = 0; i < PMAX; i++) {
        const int q = threadIdx.x + i * blockDim.x;
        if (q < pairs) dz_split_store_pair<KT>(XF, nbt, M, r, q, v[i][0], v[i][1], sh);
    }
}

template <int PMAX, int KT>
__device__ __forceinline__ void dz_split_rows_block(const float* __restrict__ X, long long ldx,
                                                    const float* __restrict__ k_scale, int M, int K, int pairs,
                                                    int nbt, uint32_t* __restrict__ XF, int* __restrict__ shifts,
                                                    float* wred) {
    for (int r = 0; r < M; r++) {
        float v[PMAX][2];
        dz_split_row_load<PMAX>(X + (long long)r * ldx, k_scale, K, v);
        dz_split_row_store<PMAX, KT>(v, r, M, pairs, nbt, XF, shifts, wred);
    }
}

constexpr int DZ_SPLIT_PAIRS = 512;   // element pairs per block of dz_split_rows_kernel

// Grid (ceil(Kp / 2 / DZ_SPLIT_PAIRS), M): each block finds its row's maximum
// (the row's exponent shift, stored negated in row_shift) and splits its
// DZ_SPLIT_PAIRS pairs.
template <int KT>
__global__ void __launch_bounds__(256) dz_split_rows_kernel(const float* __restrict__ X, long long ldx,
                                                            const float* __restrict__ k_scale, int M, int K, int nkg,
                                                            int nbt, uint32_t* __restrict__ XF,
                                                            int* __restrict__ row_shift) {
    __shared__ float wred[8];
    const int r = blockIdx.y;
    const float* x = X + (long long)r * ldx;
    const int sh = dz_row_shift(dz_row_amax(x, k_scale, K, wred));
    if (blockIdx.x == 0 && threadIdx.x == 0) row_shift[r] = -sh;
    const int pairs = nkg * KT * 8;
    const int q0 = blockIdx.x * DZ_SPLIT_PAIRS;
    const int q1 = q0 + DZ_SPLIT_PAIRS < pairs ? q0 + DZ_SPLIT_PAIRS : pairs;
#pragma unroll 2
    for (int q = q0 + threadIdx.x; q < q1; q += blockDim.x)
        dz_split_store_pair<KT>(XF, nbt, M, r, q, dz_x_at(x, k_scale, K, 2 * q), dz_x_at(x, k_scale, K, 2 * q + 1),
                                sh);
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
// Bounded wait (about one second). False when it gave up. The timer is read
// only once the phase has not completed on the first tries (a global-timer
// read costs far more than a try_wait that succeeds).
__device__ __forceinline__ bool dz_mbar_wait(uint64_t* bar, uint32_t parity) {
#pragma unroll 1
    for (int i = 0; i < 4; i++)
        if (dz_mbar_test(bar, parity)) return true;
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

// L2 policy for streamed weights: read once per product, so they should not
// evict activations and other reused data.
__device__ __forceinline__ uint64_t dz_policy_evict_first() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}
__device__ __forceinline__ void dz_bulk_g2s_stream(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                                   uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
            dz_smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(dz_smem_addr(bar)), "l"(policy)
        : "memory");
}

constexpr int QMS_STAGES = 3;      // ring stages per warp
constexpr int QMS_XIN_PAIRS = 8;   // element pairs per thread of the in-kernel split

struct QmsArgs {
    const uint8_t* codes;     // fragment layout
    int N, nkg, ntiles;
    // activations: XIN kernels split X themselves into shared memory; the
    // others read XF / row_shift (dz_split_rows_kernel)
    const float* X;
    long long ldx;
    const float* k_scale;
    int K;
    const uint32_t* XF;
    const int* row_shift;
    int nbt;                  // row pairs
    int M;
    int kparts;               // warps sharing one n-group's k-groups
    int per;                  // k-groups per k-part
    int n_groups;             // groups of NT n-tiles
    int nrounds;              // rounds of W / kparts n-groups
    int pk;                   // k-groups per piece (a stage holds NT * pk chunks)
    unsigned xf_bytes;        // XF bytes in shared memory (XIN kernels)
    int* status;              // set to 1 when a copy wait gave up (may be null)
    QmvEpilogue ep;           // row_shift is applied by the kernel, ep.row_shift unused
};

// One piece of a warp's stream: n-group ng (n-tiles NT*ng ..), k-groups
// [kg0, kg0 + nkg).
struct QmsPiece {
    int ng, kg0, nkg;
    bool first, last;
};

// Piece idx of warp `warp` of W: round r = blockIdx.x + (idx / ppr) * gridDim.x
// owns n-groups r * (W / kparts) + [0, W / kparts); the warp takes n-group
// warp / kparts, k-part warp % kparts, in pieces of pk k-groups.
template <int W>
__device__ __forceinline__ QmsPiece dz_qms_piece(const QmsArgs& a, int warp, int ppr, int idx) {
    QmsPiece p;
    const int j = idx / ppr, q = idx - j * ppr;
    const long long r = blockIdx.x + (long long)j * gridDim.x;
    p.ng = (int)(r * (W / a.kparts) + warp / a.kparts);
    const int kstart = (warp % a.kparts) * a.per;
    const int kend = min(kstart + a.per, a.nkg);
    p.kg0 = kstart + q * a.pk;
    p.nkg = p.ng < a.n_groups ? max(0, min(a.pk, kend - p.kg0)) : 0;
    p.first = q == 0;
    p.last = q == ppr - 1;
    return p;
}

// Shared memory of dz_qms_kernel: the rings, the XF copy, the k-part
// reduction area, the barriers, row shifts and a per-warp scratch float.
__host__ __device__ constexpr size_t dz_qms_ring_bytes(int pk, int NT, int W) {
    return (size_t)W * QMS_STAGES * NT * pk * 512;
}
__host__ __device__ constexpr size_t dz_qms_smem_bytes(int pk, int NT, int NB, int W, unsigned xf_bytes) {
    return dz_qms_ring_bytes(pk, NT, W) + xf_bytes + (size_t)W * NT * NB * 2 * 32 * 4 +
           (size_t)W * QMS_STAGES * 8 + 16 * 4 + 32 * 4;
}

__device__ __forceinline__ void dz_named_sync(int id, int threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// Y = epilogue(X . deq(W)) for M <= 2 * NB rows, streaming the weights. One
// persistent CTA of W warps per SM; each warp streams its pieces (NT n-tiles
// x pk k-groups) through its own QMS_STAGES-deep shared-memory ring with bulk
// copies, lane 0 keeping two pieces in flight. XIN kernels split the
// activations into B-fragment order in shared memory themselves (while the
// first weight pieces are in flight); the others read XF through L1. Each
// chunk is dequantized from shared memory into fp16 A fragments (dz_deq4 /
// dz_deq8) feeding NB MMAs per n-tile; CH independent accumulator chains per
// (n-tile, row pair) keep the tensor pipe fed when NT * NB is small. The
// k-parts of an n-group are summed in shared memory in k-part order (named
// barrier per group), so results do not depend on the grid.
template <int BITS, int NB, int NT, int W, bool XIN>
__global__ void __launch_bounds__(W * 32, 1) dz_qms_kernel(QmsArgs a) {
    constexpr int KT = FragGeom<BITS>::KT;
    constexpr int XV = KT / 2;
    constexpr int CH = NT * NB >= 4 ? 1 : (4 / (NT * NB) < KT ? 4 / (NT * NB) : KT);
    constexpr int NV = NT * NB * 2;
    extern __shared__ __align__(128) unsigned char qms_smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, t = lane & 3;
    const int stage_bytes = NT * a.pk * 512;
    uint8_t* ring = qms_smem + (size_t)warp * QMS_STAGES * stage_bytes;
    uint8_t* xf_sm = qms_smem + dz_qms_ring_bytes(a.pk, NT, W);
    float* red = reinterpret_cast<float*>(xf_sm + a.xf_bytes);
    uint64_t* bars = reinterpret_cast<uint64_t*>(red + W * NV * 32) + warp * QMS_STAGES;
    int* rsh = reinterpret_cast<int*>(reinterpret_cast<uint64_t*>(red + W * NV * 32) + W * QMS_STAGES);
    float* wred = reinterpret_cast<float*>(rsh + 16);

    const int ppr = (a.per + a.pk - 1) / a.pk;
    const int rounds_here =
        (int)blockIdx.x < a.nrounds ? (a.nrounds - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
    const int npieces = rounds_here * ppr;

    if (lane == 0) {
        for (int st = 0; st < QMS_STAGES; st++) dz_mbar_init(&bars[st]);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncwarp();

    const uint64_t wpolicy = dz_policy_evict_first();
    // lane 0: put piece idx in flight into stage idx % QMS_STAGES
    auto issue = [&](int idx) {
        const QmsPiece pc = dz_qms_piece<W>(a, warp, ppr, idx);
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
            dz_bulk_g2s_stream(dst + (size_t)i * a.pk * 512,
                               a.codes + ((size_t)(pc.ng * NT + i) * a.nkg + pc.kg0) * 512, bytes, bar, wpolicy);
    };
    int issued = min(npieces, QMS_STAGES - 1);
    if (lane == 0)
        for (int i = 0; i < issued; i++) issue(i);

    const int* shifts = a.row_shift;
    if (XIN) {
        // split the activations into shared memory while the weights stream in
        // (pairs <= QMS_XIN_PAIRS * W * 32, checked by the host)
        dz_split_rows_block<QMS_XIN_PAIRS, KT>(a.X, a.ldx, a.k_scale, a.M, a.K, a.nkg * KT * 8, a.nbt,
                                               reinterpret_cast<uint32_t*>(xf_sm), rsh, wred);
        __syncthreads();
        shifts = rsh;
    }
    const uint4* xl = (XIN ? reinterpret_cast<const uint4*>(xf_sm) : reinterpret_cast<const uint4*>(a.XF)) + lane * XV;
    const long long xkg = (long long)a.nbt * 32 * XV;   // uint4 per k-group

    bool failed = false;
    int failed_at = -1;   // first piece whose wait gave up
    float acc[CH][NT][NB][4];
    for (int idx = 0; idx < npieces; idx++) {
        const QmsPiece pc = dz_qms_piece<W>(a, warp, ppr, idx);
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
            const uint4* w4 = reinterpret_cast<const uint4*>(ring + stage * stage_bytes) + lane;
            const uint4* xk = xl + pc.kg0 * xkg;
#pragma unroll 2
            for (int c = 0; c < pc.nkg; c++, xk += xkg) {
                uint4 xv[NB][XV];
#pragma unroll
                for (int u = 0; u < NB; u++)
#pragma unroll
                    for (int h = 0; h < XV; h++)
                        xv[u][h] = u < a.nbt ? (XIN ? xk[u * 32 * XV + h] : __ldg(xk + u * 32 * XV + h))
                                             : make_uint4(0u, 0u, 0u, 0u);
                uint4 w[NT];
#pragma unroll
                for (int i = 0; i < NT; i++) w[i] = w4[(i * a.pk + c) * 32];
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
            const int grp = warp / a.kparts;
#pragma unroll
            for (int q = 0; q < NV; q++) red[(warp * NV + q) * 32 + lane] = v[q];
            dz_named_sync(1 + grp, 32 * a.kparts);
            owner = warp % a.kparts == 0;
            if (owner) {
#pragma unroll
                for (int q = 0; q < NV; q++) {
                    float sum = 0.0f;
                    for (int kp = 0; kp < a.kparts; kp++) sum += red[((warp + kp) * NV + q) * 32 + lane];
                    v[q] = sum;
                }
            }
            dz_named_sync(1 + grp, 32 * a.kparts);
        }
        if (owner && pc.ng < a.n_groups && !(t & 1)) {
#pragma unroll
            for (int u = 0; u < NB; u++) {
                const int row = 2 * u + (t >> 1);
                if (row >= a.M) continue;
                const int e = shifts[row];
#pragma unroll
                for (int i = 0; i < NT; i++) {
                    const int n = (pc.ng * NT + i) * 16 + g;
                    if (n < a.ntiles * 16) {
                        dz_qmv_store_row(a.ep, a.M, a.N, row, n, dz_mul_pow2(v[(i * NB + u) * 2], e));
                        dz_qmv_store_row(a.ep, a.M, a.N, row, n + 8, dz_mul_pow2(v[(i * NB + u) * 2 + 1], e));
                    }
                }
            }
        }
    }
    if (failed_at >= 0 && lane == 0) {
        // copies still in flight land before the shared memory is released
        for (int i = failed_at; i < issued; i++)
            if (!dz_mbar_wait(&bars[i % QMS_STAGES], (uint32_t)((i / QMS_STAGES) & 1))) break;
    }
}

// ------------------------------------------- stream-K matvec for M <= 2

struct Qmv1Args {
    const uint8_t* codes;     // fragment layout
    int N, nkg, ntiles;
    const float* X;           // XIN: rows split in the kernel
    long long ldx;
    const float* k_scale;
    int K;
    const uint32_t* XF;       // otherwise: dz_split_rows_kernel output
    const int* row_shift;
    int M;                    // 1 or 2
    int pk;                   // chunks per piece
    int max_tiles;            // n-tiles per CTA at most
    int max_parts;            // warps sharing one n-tile at most
    unsigned xf_bytes;        // XIN: XF bytes in shared memory
    int* status;              // set to 1 when a copy wait gave up (may be null)
    QmvEpilogue ep;           // row shifts are applied by the kernel
};

__host__ __device__ constexpr size_t dz_qmv1_smem_bytes(int pk, int W, unsigned xf_bytes, int max_tiles,
                                                        int max_parts) {
    return (size_t)W * QMS_STAGES * pk * 512 + xf_bytes + (size_t)max_tiles * max_parts * 32 * 4 +
           (size_t)((max_tiles + 3) & ~3) * 4 + (size_t)W * QMS_STAGES * 8 + 16 * 4 + 32 * 4;
}

// Y = epilogue(X . deq(W)) for M <= 2 rows. The weights are one array of
// 512-byte chunks, n-tile major. CTA c takes the whole n-tiles
// [c * ntiles / G, (c+1) * ntiles / G); its W warps split that run's chunks
// into W equal contiguous ranges (stream-K), so every warp streams the same
// number of bytes whatever the tile count. A warp streams its range through
// its own QMS_STAGES-deep shared-memory ring with bulk copies (pieces never
// cross an n-tile end), accumulating on the tensor cores as dz_qms_kernel
// does. An n-tile covered by one warp is stored directly; one shared by
// several warps is combined in shared memory: each warp deposits its part and
// the last to arrive (a shared-memory counter) adds the parts in warp order,
// so results do not depend on timing.
template <int BITS, int W, bool XIN>
__global__ void __launch_bounds__(W * 32, 1) dz_qmv1_kernel(Qmv1Args a) {
    constexpr int KT = FragGeom<BITS>::KT;
    constexpr int XV = KT / 2;
    constexpr int CH = KT;   // one accumulator chain per k-tile
    extern __shared__ __align__(128) unsigned char qmv1_smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, t = lane & 3;
    const int stage_bytes = a.pk * 512;
    uint8_t* ring = qmv1_smem + (size_t)warp * QMS_STAGES * stage_bytes;
    uint8_t* xf_sm = qmv1_smem + (size_t)W * QMS_STAGES * stage_bytes;
    float* slots = reinterpret_cast<float*>(xf_sm + a.xf_bytes);
    int* cnt = reinterpret_cast<int*>(slots + (size_t)a.max_tiles * a.max_parts * 32);
    uint64_t* bars = reinterpret_cast<uint64_t*>(cnt + ((a.max_tiles + 3) & ~3)) + warp * QMS_STAGES;
    int* rsh = reinterpret_cast<int*>(reinterpret_cast<uint64_t*>(cnt + ((a.max_tiles + 3) & ~3)) + W * QMS_STAGES);
    float* wred = reinterpret_cast<float*>(rsh + 16);

    // chunk indices fit 32 bits (2^31 chunks = 1 TB of codes)
    const int G = gridDim.x;
    const int t0 = (int)((long long)blockIdx.x * a.ntiles / G), t1 = (int)(((long long)blockIdx.x + 1) * a.ntiles / G);
    const int C0 = t0 * a.nkg, L = (t1 - t0) * a.nkg;
    auto wstart = [&](int w) { return C0 + (int)((long long)w * L / W); };
    const int my0 = wstart(warp), my1 = wstart(warp + 1);
    // a position in this warp's range: chunk pos = tile * nkg + kg
    struct Cursor {
        int pos, tile, kg;
    };
    auto cursor_at = [&](int p) {
        Cursor c;
        c.pos = p;
        c.tile = p / a.nkg;
        c.kg = p - c.tile * a.nkg;
        return c;
    };
    // the piece at c: up to pk chunks, not past the n-tile or the range
    auto piece_len = [&](const Cursor& c) { return min(a.pk, min(a.nkg - c.kg, my1 - c.pos)); };
    auto advance = [&](Cursor& c, int n) {
        c.pos += n;
        c.kg += n;
        if (c.kg == a.nkg) {
            c.kg = 0;
            c.tile++;
        }
    };

    for (int i = threadIdx.x; i < a.max_tiles; i += blockDim.x) cnt[i] = 0;
    if (lane == 0) {
        for (int st = 0; st < QMS_STAGES; st++) dz_mbar_init(&bars[st]);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncwarp();

    // Launched as a programmatic dependent of the previous kernel, and lets the
    // next one launch: its CTAs take SMs as this kernel's CTAs finish. Only
    // the weight copies (constant for the launch) go out before
    // griddepcontrol.wait; activations are read and every global write made
    // after it, i.e. after the previous kernel completed.
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    // lane 0 keeps two pieces in flight: piece i -> stage i % QMS_STAGES
    Cursor ic = cursor_at(my0);
    int issued = 0, istage = 0;
    const uint64_t wpolicy = dz_policy_evict_first();
    auto issue = [&]() {
        const int n = piece_len(ic);
        uint64_t* bar = &bars[istage];
        dz_mbar_expect_tx(bar, (uint32_t)n * 512u);
        dz_bulk_g2s_stream(ring + istage * stage_bytes, a.codes + (size_t)ic.pos * 512, (uint32_t)n * 512u, bar,
                           wpolicy);
        advance(ic, n);
        issued++;
        istage = istage == QMS_STAGES - 1 ? 0 : istage + 1;
    };
    // the first weight piece goes out before the wait; the activation rows
    // are requested before the second, so they do not queue behind both
    if (lane == 0 && ic.pos < my1) issue();
    asm volatile("griddepcontrol.wait;" ::: "memory");
    float xr[2][QMS_XIN_PAIRS][2];
    if (XIN) {
        dz_split_row_load<QMS_XIN_PAIRS>(a.X, a.k_scale, a.K, xr[0]);
        if (a.M > 1) dz_split_row_load<QMS_XIN_PAIRS>(a.X + a.ldx, a.k_scale, a.K, xr[1]);
    }
    if (lane == 0)
        for (int i = 1; i < QMS_STAGES - 1 && ic.pos < my1; i++) issue();

    const int* shifts = a.row_shift;
    if (XIN) {
        uint32_t* xf32 = reinterpret_cast<uint32_t*>(xf_sm);
        dz_split_row_store<QMS_XIN_PAIRS, KT>(xr[0], 0, a.M, a.nkg * KT * 8, 1, xf32, rsh, wred);
        if (a.M > 1) dz_split_row_store<QMS_XIN_PAIRS, KT>(xr[1], 1, a.M, a.nkg * KT * 8, 1, xf32, rsh, wred);
        shifts = rsh;
    }
    __syncthreads();   // counters zeroed, XF written
    const uint4* xl = (XIN ? reinterpret_cast<const uint4*>(xf_sm) : reinterpret_cast<const uint4*>(a.XF)) + lane * XV;

    // warp owning chunk x of this CTA's run (ranges may be empty when L < W)
    auto owner_of = [&](int x) {
        int w = (int)(((long long)(x - C0) * W) / (L > 0 ? L : 1));
        if (w > W - 1) w = W - 1;
        while (w < W - 1 && wstart(w + 1) <= x) w++;
        while (w > 0 && wstart(w) > x) w--;
        return w;
    };

    bool failed = false;
    int failed_at = -1;   // first piece whose wait gave up
    Cursor cc = cursor_at(my0);
    int consumed = 0, cstage = 0;
    uint32_t cphase = 0;
    float acc[CH][4];
#pragma unroll
    for (int c = 0; c < CH; c++)
#pragma unroll
        for (int q = 0; q < 4; q++) acc[c][q] = 0.0f;
    while (cc.pos < my1) {
        const int n = piece_len(cc);
        if (!failed && lane == 0 && ic.pos < my1) issue();
        const int stage = cstage;
        if (!failed) {
            int ok = 1;
            if (lane == 0) ok = dz_mbar_wait(&bars[stage], cphase) ? 1 : 0;
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (!ok) {
                failed = true;
                failed_at = consumed;
                if (lane == 0 && a.status) atomicExch(a.status, 1);
            }
        }
        const int tile = cc.tile;
        const int kg0 = cc.kg;
        if (!failed) {
            const uint4* w4 = reinterpret_cast<const uint4*>(ring + stage * stage_bytes) + lane;
            const uint4* xk = xl + (long long)kg0 * 32 * XV;
#pragma unroll 2
            for (int c = 0; c < n; c++, xk += 32 * XV) {
                uint4 xv[XV];
#pragma unroll
                for (int h = 0; h < XV; h++) xv[h] = XIN ? xk[h] : __ldg(xk + h);
                const uint4 w = w4[c * 32];
                const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
                for (int kt = 0; kt < KT; kt++) {
                    uint32_t af[4];
                    if (BITS == 4) dz_deq4(ww[kt], af);
                    else dz_deq8(ww[2 * kt], ww[2 * kt + 1], af);
                    dz_mma_f16(acc[kt % CH], af, dz_xw(xv, 2 * kt), dz_xw(xv, 2 * kt + 1));
                }
            }
        }
        __syncwarp();   // the stage is free for lane 0 to refill
        consumed++;
        if (++cstage == QMS_STAGES) {
            cstage = 0;
            cphase ^= 1u;
        }
        advance(cc, n);
        const int tile_start = tile * a.nkg, tile_end = tile_start + a.nkg;
        if (cc.pos != tile_end && cc.pos != my1) continue;

        // this warp's share of the n-tile is done
        float d[4];
#pragma unroll
        for (int q = 0; q < 4; q++) {
            d[q] = acc[0][q];
#pragma unroll
            for (int c = 1; c < CH; c++) d[q] += acc[c][q];
        }
        float v0, v1;
        dz_combine<BITS>(d, v0, v1);
        if (failed) v0 = v1 = __int_as_float(0x7fc00000);   // a failed tile reads NaN
#pragma unroll
        for (int c = 0; c < CH; c++)
#pragma unroll
            for (int q = 0; q < 4; q++) acc[c][q] = 0.0f;
        const int row = t >> 1;
        const int n0 = tile * 16 + g;
        const bool whole = my0 <= tile_start && my1 >= tile_end;
        if (whole) {
            if (!(t & 1) && row < a.M) {
                const int e = shifts[row];
                dz_qmv_store_row(a.ep, a.M, a.N, row, n0, dz_mul_pow2(v0, e));
                dz_qmv_store_row(a.ep, a.M, a.N, row, n0 + 8, dz_mul_pow2(v1, e));
            }
            continue;
        }
        // shared n-tile: parts are the non-empty warp ranges meeting it, in warp order
        const int wf = owner_of(tile_start > C0 ? tile_start : C0);
        const int wl = owner_of((tile_end < C0 + L ? tile_end : C0 + L) - 1);
        int part = 0, nparts = 0;
        for (int w = wf; w <= wl; w++) {
            if (wstart(w + 1) > wstart(w)) {
                if (w < warp) part++;
                nparts++;
            }
        }
        const int lt = tile - t0;
        float* mine = slots + ((size_t)lt * a.max_parts + part) * 32;
        if (!(t & 1)) {
            mine[row * 16 + g] = v0;
            mine[row * 16 + g + 8] = v1;
        }
        __syncwarp();
        int last = 0;
        if (lane == 0) {
            __threadfence_block();
            last = atomicAdd(&cnt[lt], 1) == nparts - 1 ? 1 : 0;
        }
        last = __shfl_sync(0xffffffffu, last, 0);
        if (last) {
            __threadfence_block();
            if (!(t & 1) && row < a.M) {
                float s0 = 0.0f, s1 = 0.0f;
                for (int pp = 0; pp < nparts; pp++) {
                    const float* sl = slots + ((size_t)lt * a.max_parts + pp) * 32;
                    s0 += sl[row * 16 + g];
                    s1 += sl[row * 16 + g + 8];
                }
                const int e = shifts[row];
                dz_qmv_store_row(a.ep, a.M, a.N, row, n0, dz_mul_pow2(s0, e));
                dz_qmv_store_row(a.ep, a.M, a.N, row, n0 + 8, dz_mul_pow2(s1, e));
            }
        }
    }
    if (failed_at >= 0 && lane == 0) {
        // copies still in flight land before the shared memory is released
        for (int i = failed_at; i < issued; i++)
            if (!dz_mbar_wait(&bars[i % QMS_STAGES], (uint32_t)((i / QMS_STAGES) & 1))) break;
    }
}

}  // namespace dz
