// Tensor-core building blocks for the quantized matvec / skinny GEMM.
//
// Weights live in an MMA-fragment layout: the matrix W[k x n] (the reference's
// storage, src/core/quantize.c:213-270) is cut into n-tiles of 16 output
// columns and k-groups of 64 (INT4) or 32 (INT8) rows. One k-group of one
// n-tile is a 512-byte chunk; lane l of a warp loads bytes [16l, 16l+16) and
// holds exactly the A-fragments of the m16n8k16 MMAs it takes part in: with
// g = l/4, t = l%4 and k0 the k-tile base, an A fragment is the 8 values
//   (n=g, k=2t) (n=g+8, k=2t) (n=g, k=2t+8) (n=g+8, k=2t+8)
//   (n=g, k=2t+1) (n=g+8, k=2t+1) (n=g, k=2t+9) (n=g+8, k=2t+9)
// stored as the nibbles 0..7 of one 32-bit word. INT4: a chunk holds 4 k-tiles,
// one word each. INT8: a code c = 16h + l splits into a high and a low nibble
// plane, level = c - 127 = 16*(h - 8) + (l + 1); a k-tile is two words (low
// plane, high plane), a chunk holds 2 k-tiles. Codes are the reference's bits,
// reordered.
//
// Dequantization: (word >> 4p) & 0x000F000F | 0x43004300 is the bf16 pair
// (128 + c_a, 128 + c_b); subtracting 135 (INT4: c - 7), 136 (INT8 high
// plane: h - 8) or 127 (INT8 low plane: l + 1) gives exact small integers. Activations enter as three bf16 columns hi, mid, lo
// with hi + mid + lo = x to 24 mantissa bits (hi = bf16(x), mid =
// bf16(x - hi), lo = bf16(x - hi - mid)); the products are exact and the
// tensor core accumulates in fp32, so the result carries fp32-level error like
// the reference's fp32 multiply-add, with the per-column scale applied after
// the k-sum.
#pragma once
#include <cstdint>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

namespace dz {

// k rows covered by one 512-byte chunk
template <int BITS>
struct FragGeom {
    static constexpr int KG = BITS == 8 ? 32 : 64;   // rows per chunk
    static constexpr int KT = KG / 16;               // k-tiles per chunk
};

// Reference storage -> fragment layout; one thread per output word. The
// destination's columns are the concatenation of up to three sources (column
// offsets off[0..nsrc]); words past the last column or past K hold code qmax
// (level 0).
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
    // position p of the 8 nibbles -> (n offset, k offset) inside the k-tile
    const int pn[8] = {g, g + 8, g, g + 8, g, g + 8, g, g + 8};
    const int pk[8] = {2 * t, 2 * t, 2 * t + 8, 2 * t + 8, 2 * t + 1, 2 * t + 1, 2 * t + 9, 2 * t + 9};
    int ktile, plane;
    if (bits == 4) {
        ktile = kg * 4 + j;
        plane = -1;
    } else {
        ktile = kg * 2 + (j >> 1);
        plane = j & 1;   // 0 low nibbles, 1 high nibbles
    }
    const int ntot = src.off[src.nsrc];
    uint32_t word = 0;
    for (int p = 0; p < 8; p++) {
        const long long n = nt * 16 + pn[p];
        const long long k = (long long)ktile * 16 + pk[p];
        uint32_t code = bits == 8 ? 127u : 7u;
        if (n < ntot && k < K) {
            int i = 0;
            while (i + 1 < src.nsrc && n >= src.off[i + 1]) i++;
            const long long N = src.off[i + 1] - src.off[i];
            const long long idx = k * N + (n - src.off[i]);
            const uint8_t* ref = src.ref[i];
            code = bits == 8 ? ref[idx] : (uint32_t)((ref[idx >> 1] >> ((idx & 1) * 4)) & 0xF);
        }
        const uint32_t nib = bits == 4 ? code : (plane == 0 ? (code & 0xF) : (code >> 4));
        word |= nib << (4 * p);
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
    // invert the position table: n offset g or g+8, k offset 2t(+1)(+8)
    const int g = nl & 7, hi_row = nl >> 3;
    const int t = (kk & 7) >> 1, odd = kk & 1, hi_k = kk >> 3;
    const int p = hi_row + 2 * hi_k + 4 * odd;
    const int lane = g * 4 + t;
    const uint32_t* chunk = reinterpret_cast<const uint32_t*>(codes) + ((nt * nkg + kg) * 128 + lane * 4);
    if (bits == 4) return (chunk[kt] >> (4 * p)) & 0xF;
    const uint32_t lo = (chunk[kt * 2] >> (4 * p)) & 0xF;
    const uint32_t hi = (chunk[kt * 2 + 1] >> (4 * p)) & 0xF;
    return lo | (hi << 4);
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

__device__ __forceinline__ uint32_t dz_bf16x2_sub(uint32_t a, uint32_t b) {
    __nv_bfloat162 x = *reinterpret_cast<__nv_bfloat162*>(&a);
    __nv_bfloat162 y = *reinterpret_cast<__nv_bfloat162*>(&b);
    __nv_bfloat162 r = __hsub2(x, y);
    return *reinterpret_cast<uint32_t*>(&r);
}

// The four A-fragment registers of one plane word; `off` = bf16x2 of
// (128 + offset) in both halves.
__device__ __forceinline__ void dz_frag_dequant(uint32_t w, uint32_t off, uint32_t (&a)[4]) {
    a[0] = dz_bf16x2_sub((w & 0x000F000Fu) | 0x43004300u, off);
    a[1] = dz_bf16x2_sub(((w >> 4) & 0x000F000Fu) | 0x43004300u, off);
    a[2] = dz_bf16x2_sub(((w >> 8) & 0x000F000Fu) | 0x43004300u, off);
    a[3] = dz_bf16x2_sub(((w >> 12) & 0x000F000Fu) | 0x43004300u, off);
}

constexpr uint32_t DZ_BF16X2_135 = 0x43074307u;   // 135.0 in both halves
constexpr uint32_t DZ_BF16X2_136 = 0x43084308u;   // 136.0
constexpr uint32_t DZ_BF16X2_127 = 0x42FE42FEu;   // 127.0

// D += A (16 x 16, bf16, row) . B (16 x 8, bf16, col), fp32 accumulate.
__device__ __forceinline__ void dz_mma_bf16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Component s (0 hi, 1 mid, 2 lo, 3 zero) of the exact three-way bf16 split of x.
__device__ __forceinline__ __nv_bfloat16 dz_split(float x, int s) {
    const __nv_bfloat16 h = __float2bfloat16_rn(x);
    if (s == 0) return h;
    const float r1 = x - __bfloat162float(h);
    const __nv_bfloat16 m = __float2bfloat16_rn(r1);
    if (s == 1) return m;
    if (s == 2) return __float2bfloat16_rn(r1 - __bfloat162float(m));
    return __float2bfloat16_rn(0.0f);
}

__device__ __forceinline__ uint32_t dz_pack_bf16x2(__nv_bfloat16 lo, __nv_bfloat16 hi) {
    return (uint32_t)__bfloat16_as_ushort(lo) | ((uint32_t)__bfloat16_as_ushort(hi) << 16);
}


// ------------------------------------------------------ the global kernels

// X[M][K] (fp32, ROW-granularity scales folded in) -> Xs[M][3][Kp] bf16: the
// hi / mid / lo split the MMAs take as B columns, zero past K.
__global__ void dz_split_rows_kernel(const float* __restrict__ X, long long ldx, const float* __restrict__ k_scale,
                                     int M, int K, int Kp, __nv_bfloat16* __restrict__ Xs) {
    const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= (long long)M * Kp) return;
    const int m = (int)(idx / Kp), k = (int)(idx % Kp);
    float v = 0.0f;
    if (k < K) {
        v = X[(long long)m * ldx + k];
        if (k_scale) v *= k_scale[k];
    }
    const __nv_bfloat16 h = __float2bfloat16_rn(v);
    const float r1 = v - __bfloat162float(h);
    const __nv_bfloat16 mid = __float2bfloat16_rn(r1);
    __nv_bfloat16* row = Xs + (long long)m * 3 * Kp;
    row[k] = h;
    row[Kp + k] = mid;
    row[2 * Kp + k] = __float2bfloat16_rn(r1 - __bfloat162float(mid));
}

struct QmmArgs {
    const uint8_t* codes;     // fragment layout
    int K, N, nkg, ntiles;
    const __nv_bfloat16* Xs;  // [M][3][Kp] split activations (dz_split_rows_kernel)
    int Kp;                   // nkg * rows per k-group
    int M;
    int kparts;               // warps splitting the k-groups of one unit
    int kg_per_part;
    int n_groups;             // n-tile groups of NT tiles
    int m_passes;             // row passes of 2*NB rows
    QmvEpilogue ep;
};

// Y = epilogue(X . deq(W)) on tensor cores. A warp owns NT n-tiles x 2*NB rows
// over a range of k-groups. Weight fragments are loaded one k-group ahead
// (registers double-buffered); per k-tile the lane fetches its B fragments
// (two 32-bit loads per 8-column tile of rows x {hi, mid, lo, 0}), and each
// n-tile's dequantized A fragment feeds NB MMAs (x2 planes for INT8).
template <int BITS, int NB, int NT>
__global__ void __launch_bounds__(QMV_THREADS) dz_qmm_kernel(QmmArgs a) {
    constexpr int KT = FragGeom<BITS>::KT;
    constexpr int PL = BITS == 8 ? 2 : 1;          // nibble planes
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
    const int m0 = mpass * 2 * NB;
    const int kg0 = kpart * a.kg_per_part;
    const int kg1 = min(kg0 + a.kg_per_part, a.nkg);

    float acc[PL][NT][NB][4];
#pragma unroll
    for (int p = 0; p < PL; p++)
#pragma unroll
        for (int i = 0; i < NT; i++)
#pragma unroll
            for (int u = 0; u < NB; u++)
#pragma unroll
                for (int q = 0; q < 4; q++) acc[p][i][u][q] = 0.0f;

    // B column 8u + g of this lane = row m0 + 2u + g/4, split g%4 (3: zero column)
    const uint32_t* xs32 = reinterpret_cast<const uint32_t*>(a.Xs);
    long long xbase[NB];
    bool xvalid[NB];
#pragma unroll
    for (int u = 0; u < NB; u++) {
        const int row = m0 + 2 * u + (g >> 2);
        xvalid[u] = row < a.M && (g & 3) < 3;
        xbase[u] = xvalid[u] ? (((long long)row * 3 + (g & 3)) * a.Kp) / 2 + t : 0;
    }
    const uint4 pad = make_uint4(0x77777777u, 0x77777777u, 0x77777777u, 0x77777777u);
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
#pragma unroll
            for (int kt = 0; kt < KT; kt++) {
                const int kh = (kg * KT + kt) * 8;   // k0 / 2
                uint32_t b0[NB], b1[NB];
#pragma unroll
                for (int u = 0; u < NB; u++) {
                    b0[u] = xvalid[u] ? __ldg(xs32 + xbase[u] + kh) : 0u;
                    b1[u] = xvalid[u] ? __ldg(xs32 + xbase[u] + kh + 4) : 0u;
                }
#pragma unroll
                for (int i = 0; i < NT; i++) {
                    const uint32_t ww[4] = {wcur[i].x, wcur[i].y, wcur[i].z, wcur[i].w};
                    uint32_t af[4];
                    if (BITS == 4) {
                        dz_frag_dequant(ww[kt], DZ_BF16X2_135, af);
#pragma unroll
                        for (int u = 0; u < NB; u++) dz_mma_bf16(acc[0][i][u], af, b0[u], b1[u]);
                    } else {
                        dz_frag_dequant(ww[2 * kt], DZ_BF16X2_127, af);
#pragma unroll
                        for (int u = 0; u < NB; u++) dz_mma_bf16(acc[0][i][u], af, b0[u], b1[u]);
                        dz_frag_dequant(ww[2 * kt + 1], DZ_BF16X2_136, af);
#pragma unroll
                        for (int u = 0; u < NB; u++) dz_mma_bf16(acc[PL - 1][i][u], af, b0[u], b1[u]);
                    }
                }
            }
            if (kg + 1 < kg1) {
#pragma unroll
                for (int i = 0; i < NT; i++) wcur[i] = wnext[i];
            }
        }
    }

    // combine the split columns: lane pair (t, t^1) holds hi+mid and lo of one row
    float v[NV];
#pragma unroll
    for (int i = 0; i < NT; i++)
#pragma unroll
        for (int u = 0; u < NB; u++) {
            float lo_n, hi_n;
            if (BITS == 4) {
                lo_n = acc[0][i][u][0] + acc[0][i][u][1];
                hi_n = acc[0][i][u][2] + acc[0][i][u][3];
            } else {
                lo_n = 16.0f * (acc[1][i][u][0] + acc[1][i][u][1]) + (acc[0][i][u][0] + acc[0][i][u][1]);
                hi_n = 16.0f * (acc[1][i][u][2] + acc[1][i][u][3]) + (acc[0][i][u][2] + acc[0][i][u][3]);
            }
            lo_n += __shfl_xor_sync(0xffffffffu, lo_n, 1);
            hi_n += __shfl_xor_sync(0xffffffffu, hi_n, 1);
            v[(i * NB + u) * 2 + 0] = lo_n;   // output column nt*16 + g
            v[(i * NB + u) * 2 + 1] = hi_n;   // output column nt*16 + g + 8
        }
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
            const int row = m0 + 2 * u + (t >> 1);
            const int n = (group * NT + i) * 16 + g;
            dz_qmv_store_row(a.ep, a.M, a.N, row, n, v[(i * NB + u) * 2 + 0]);
            dz_qmv_store_row(a.ep, a.M, a.N, row, n + 8, v[(i * NB + u) * 2 + 1]);
        }
}

}  // namespace dz
