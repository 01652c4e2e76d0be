// Quantized weight-streaming matvec / skinny GEMM for sm_100a (CUDA cores).
//
// Computes Y[m][n] = epilogue( sum_k X[m][k] * level(k, n) ) for the weight
// matrix W[k x n] of the reference's storage form (src/core/quantize.c:213-270;
// C = A . deq(W) as in matmul_quantized_weight, src/core/quantized_matmul.c:
// 253-295), with the per-column scale factored out of the k-sum and applied in
// the epilogue (COLUMN/TENSOR granularity) or folded into the activation as it
// is loaded (ROW granularity).
//
// Device layout ("strips"): columns are grouped in strips of 4; a strip is a
// contiguous run of 16-byte chunks ascending in k. One chunk holds 4 columns
// x KC rows (KC = 4 for INT8, 8 for INT4): 32-bit word j of the chunk is
// column 4s+j, its bytes (INT8) or nibbles (INT4) are consecutive k. Codes are
// bit-identical to the reference's; only their order changes. K is padded to
// a multiple of KC and N to a multiple of 16 with code qmax (level 0).
//
// A warp streams one strip group over a k-range: each lane issues one 128-bit
// load per strip per 32 chunks, so a warp instruction reads 512 contiguous
// bytes. Codes are unpacked in registers by building the float 2^23 + code
// with one byte-permute / mask and subtracting 2^23 + qmax (exact), then FMA'd
// against fp32 activations. Lanes hold partial sums for ST strips x MT rows;
// a butterfly shuffle reduction leaves one total per lane group, warps that
// split K combine through shared memory, and the epilogue writes each output
// once.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace dz {

constexpr int QMV_THREADS = 256;
constexpr int QMV_WARPS = QMV_THREADS / 32;

struct QmvEpilogue {
    const float* col_scale;   // [Np] per-column scale, or nullptr (scale 1)
    const float* bias;        // [N] or nullptr
    const float* residual;    // [M][ld_res] or nullptr, added after bias
    long long ld_res;
    int relu;                 // apply max(0, .) last
    // Output column segments: columns [seg_start[i], seg_start[i+1]) go to
    // seg_ptr[i] + row*seg_ld[i] + (seg_row_off ? seg_row_off[row] : 0) + (n - seg_start[i]).
    int nseg;
    int seg_start[4];
    float* seg_ptr[3];
    long long seg_ld[3];
    const int* seg_row_off[3];
};

struct QmvArgs {
    const uint8_t* codes;     // strip layout
    int K, N, nchunks;        // nchunks = Kp / KC
    const float* k_scale;     // [K] ROW-granularity scales folded into x, or nullptr
    const float* X;           // [M][ldx]
    long long ldx;
    int M;
    int kparts;               // warps splitting K for one unit (1, 2, 4, 8)
    int chunks_per_part;
    int n_groups;             // strip groups (Np / (4*ST))
    int m_tiles;
    QmvEpilogue ep;
};

__device__ __forceinline__ float dz_level8(uint32_t w, int i) {
    // float 2^23 + byte i of w, exact; minus 2^23 + 127 gives the level
    const uint32_t b = __byte_perm(w, 0x4B000000u, 0x7440u | (uint32_t)i);
    return __uint_as_float(b) - 8388735.0f;
}

__device__ __forceinline__ float dz_level4(uint32_t w, int i) {
    const uint32_t b = ((w >> (4 * i)) & 0xFu) | 0x4B000000u;
    return __uint_as_float(b) - 8388615.0f;  // 2^23 + 7
}

// Butterfly reduce-scatter over a warp: NV values per lane in, afterwards the
// lanes whose low (5 - log2 NV) bits are zero hold the warp total of value
// index (lane >> (5 - log2 NV)).
template <int NV>
__device__ __forceinline__ float dz_warp_reduce_scatter(float (&v)[NV], int lane) {
    static_assert(NV >= 1 && NV <= 32 && (NV & (NV - 1)) == 0, "NV power of two <= 32");
#pragma unroll
    for (int half = NV / 2, off = 16; half >= 1; half /= 2, off /= 2) {
        const bool upper = (lane & off) != 0;
#pragma unroll
        for (int i = 0; i < half; i++) {
            const float send = upper ? v[i] : v[i + half];
            const float keep = upper ? v[i + half] : v[i];
            v[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
        }
    }
    float t = v[0];
    constexpr int done = (NV == 1) ? 0 : (NV == 2 ? 1 : NV == 4 ? 2 : NV == 8 ? 3 : NV == 16 ? 4 : 5);
#pragma unroll
    for (int off = 16 >> done; off >= 1; off >>= 1) t += __shfl_xor_sync(0xffffffffu, t, off);
    return t;
}

__device__ __forceinline__ void dz_qmv_store(const QmvArgs& a, int m, int n, float acc) {
    const QmvEpilogue& e = a.ep;
    if (m >= a.M || n >= a.N) return;
    float y = e.col_scale ? acc * e.col_scale[n] : acc;
    if (e.bias) y = y + e.bias[n];
    if (e.residual) y = y + e.residual[(long long)m * e.ld_res + n];
    if (e.relu) y = y > 0.0f ? y : 0.0f;
    int s = 0;
    while (s + 1 < e.nseg && n >= e.seg_start[s + 1]) s++;
    long long off = (long long)m * e.seg_ld[s] + (n - e.seg_start[s]);
    if (e.seg_row_off[s]) off += e.seg_row_off[s][m];
    e.seg_ptr[s][off] = y;
}

// BITS: 8 or 4. MT rows per tile, ST strips per warp, VEC: x rows 16-byte
// aligned with K % KC == 0 (vector x loads).
template <int BITS, int MT, int ST, bool VEC>
__global__ void __launch_bounds__(QMV_THREADS) dz_qmv_kernel(QmvArgs a) {
    constexpr int KC = (BITS == 8) ? 4 : 8;
    constexpr int NV = MT * ST * 4;
    static_assert(NV <= 32, "per-lane accumulators bounded by the butterfly width");
    __shared__ float red[QMV_WARPS][32];

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int units_per_cta = QMV_WARPS / a.kparts;
    const int unit = blockIdx.x * units_per_cta + warp / a.kparts;
    const int kpart = warp % a.kparts;
    const int total_units = a.n_groups * a.m_tiles;
    const bool active = unit < total_units;

    const int group = active ? unit % a.n_groups : 0;
    const int mtile = active ? unit / a.n_groups : 0;
    const int m0 = mtile * MT;
    const int c_begin = kpart * a.chunks_per_part;
    int c_end = c_begin + a.chunks_per_part;
    if (c_end > a.nchunks) c_end = a.nchunks;

    float acc[NV];
#pragma unroll
    for (int i = 0; i < NV; i++) acc[i] = 0.0f;

    if (active) {
        const uint4* strip_base[ST];
#pragma unroll
        for (int s = 0; s < ST; s++)
            strip_base[s] = reinterpret_cast<const uint4*>(a.codes) +
                            (long long)(group * ST + s) * a.nchunks;
        for (int c = c_begin + lane; c < c_end; c += 32) {
            uint4 w[ST];
#pragma unroll
            for (int s = 0; s < ST; s++) w[s] = __ldg(strip_base[s] + c);
            const int k0 = c * KC;
#pragma unroll
            for (int m = 0; m < MT; m++) {
                float x[KC];
                const int row = m0 + m;
                if (row < a.M) {
                    const float* xr = a.X + (long long)row * a.ldx + k0;
                    if (VEC) {
#pragma unroll
                        for (int q = 0; q < KC / 4; q++) {
                            const float4 v = __ldg(reinterpret_cast<const float4*>(xr) + q);
                            x[4 * q + 0] = v.x; x[4 * q + 1] = v.y; x[4 * q + 2] = v.z; x[4 * q + 3] = v.w;
                        }
                        if (k0 + KC > a.K) {
#pragma unroll
                            for (int i = 0; i < KC; i++) if (k0 + i >= a.K) x[i] = 0.0f;
                        }
                    } else {
#pragma unroll
                        for (int i = 0; i < KC; i++) x[i] = (k0 + i < a.K) ? __ldg(xr + i) : 0.0f;
                    }
                    if (a.k_scale) {
#pragma unroll
                        for (int i = 0; i < KC; i++) x[i] = (k0 + i < a.K) ? x[i] * __ldg(a.k_scale + k0 + i) : 0.0f;
                    }
                } else {
#pragma unroll
                    for (int i = 0; i < KC; i++) x[i] = 0.0f;
                }
#pragma unroll
                for (int s = 0; s < ST; s++) {
                    const uint32_t ww[4] = {w[s].x, w[s].y, w[s].z, w[s].w};
#pragma unroll
                    for (int j = 0; j < 4; j++) {
                        float t = acc[(m * ST + s) * 4 + j];
#pragma unroll
                        for (int i = 0; i < KC; i++) {
                            const float lv = (BITS == 8) ? dz_level8(ww[j], i) : dz_level4(ww[j], i);
                            t = fmaf(x[i], lv, t);
                        }
                        acc[(m * ST + s) * 4 + j] = t;
                    }
                }
            }
        }
    }

    const float total = dz_warp_reduce_scatter<NV>(acc, lane);
    constexpr int shift = (NV == 1) ? 5 : (NV == 2 ? 4 : NV == 4 ? 3 : NV == 8 ? 2 : NV == 16 ? 1 : 0);
    const int idx = lane >> shift;
    const bool owner = (lane & ((1 << shift) - 1)) == 0;

    if (a.kparts == 1) {
        if (active && owner) {
            const int m = m0 + idx / (ST * 4);
            const int n = (group * ST + (idx / 4) % ST) * 4 + (idx & 3);
            dz_qmv_store(a, m, n, total);
        }
        return;
    }
    if (owner) red[warp][idx] = total;
    __syncthreads();
    if (active && kpart == 0 && lane < NV) {
        float sum = 0.0f;
        for (int p = 0; p < a.kparts; p++) sum += red[warp + p][lane];
        const int m = m0 + lane / (ST * 4);
        const int n = (group * ST + (lane / 4) % ST) * 4 + (lane & 3);
        dz_qmv_store(a, m, n, sum);
    }
}

// Reference storage -> strip layout. One thread per 32-bit output word.
__global__ void dz_repack_kernel(const uint8_t* __restrict__ ref, uint32_t* __restrict__ out, int K,
                                 int N, int bits, int nchunks, long long nwords) {
    const long long wid = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (wid >= nwords) return;
    const int KC = bits == 8 ? 4 : 8;
    const int qmax = bits == 8 ? 127 : 7;
    const int j = (int)(wid & 3);
    const long long chunk = wid >> 2;
    const int c = (int)(chunk % nchunks);
    const long long strip = chunk / nchunks;
    const long long n = strip * 4 + j;
    uint32_t word = 0;
    for (int i = 0; i < KC; i++) {
        const long long k = (long long)c * KC + i;
        uint32_t code = (uint32_t)qmax;
        if (k < K && n < N) {
            const long long idx = k * N + n;
            code = bits == 8 ? ref[idx] : (uint32_t)((ref[idx >> 1] >> ((idx & 1) * 4)) & 0xF);
        }
        word |= code << (bits == 8 ? 8 * i : 4 * i);
    }
    out[wid] = word;
}

// Strip layout -> reference storage (bit-exact inverse of the repack), one
// thread per reference byte. Padding bits of a final half byte are zero.
__global__ void dz_unrepack_kernel(const uint8_t* __restrict__ codes, uint8_t* __restrict__ ref, int K,
                                   int N, int bits, int nchunks, long long nbytes) {
    const long long b = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= nbytes) return;
    const int KC = bits == 8 ? 4 : 8;
    const long long total = (long long)K * N;
    auto code_at = [&](long long idx) -> uint32_t {
        const long long k = idx / N, n = idx % N;
        const long long strip = n >> 2;
        const int j = (int)(n & 3);
        const long long c = k / KC;
        const int i = (int)(k % KC);
        const uint32_t* w = reinterpret_cast<const uint32_t*>(codes) + ((strip * nchunks + c) * 4 + j);
        return bits == 8 ? ((*w >> (8 * i)) & 0xFF) : ((*w >> (4 * i)) & 0xF);
    };
    if (bits == 8) {
        ref[b] = (uint8_t)code_at(b);
    } else {
        uint32_t lo = code_at(2 * b);
        uint32_t hi = (2 * b + 1 < total) ? code_at(2 * b + 1) : 0u;
        ref[b] = (uint8_t)(lo | (hi << 4));
    }
}

// quantize_unpack on the device: dst[k][n] = scale * (code - qmax), the
// reference's decode (src/core/quantize.c:290-295), from the strip layout.
__global__ void dz_dequant_kernel(const uint8_t* __restrict__ codes, const float* __restrict__ scales,
                                  int gran, float* __restrict__ dst, int K, int N, int bits,
                                  int nchunks) {
    const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= (long long)K * N) return;
    const int KC = bits == 8 ? 4 : 8;
    const int qmax = bits == 8 ? 127 : 7;
    const long long k = idx / N, n = idx % N;
    const uint32_t* w = reinterpret_cast<const uint32_t*>(codes) + (((n >> 2) * nchunks + k / KC) * 4 + (n & 3));
    const int i = (int)(k % KC);
    const uint32_t code = bits == 8 ? ((*w >> (8 * i)) & 0xFF) : ((*w >> (4 * i)) & 0xF);
    const float s = gran == 2 ? scales[n] : gran == 1 ? scales[k] : scales[0];
    dst[idx] = s * (float)((int)code - qmax);
}

}  // namespace dz
