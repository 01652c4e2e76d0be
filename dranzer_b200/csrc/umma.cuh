// Quantized GEMM on the 5th-generation tensor cores (tcgen05 / UMMA) for
// many activation rows (batched prefill and large-batch decode):
//   C[m, n] = epilogue(scale[n] * sum_k x[m, k] * level[k, n]).
//
// Integer formulation, exact in every product and sum:
// - each activation row is scaled by 2^s (exact) so that max |x 2^s| lies in
//   [2^21, 2^22), rounded to an integer X (|X| <= 2^22) and cut into three
//   signed 8-bit limbs X = 65536 * top + 256 * mid + low (balanced base-256
//   digits: mid, low in [-128, 127], top in [-64, 64]);
// - weights enter the tensor core as their signed levels q = code - qmax
//   (src/core/quantize.c:213-221 stores code = level + qmax; INT4 nibbles are
//   widened to bytes), converted once at upload, so there is no
//   dequantization at all;
// - one kind::i8 MMA per limb accumulates int32 in tensor memory (exact for
//   K <= UG_MAX_K); the epilogue combines the limbs in int64, converts to
//   fp32 once and applies 2^-s and the column scale.
// Rounding differs from the reference's fp32 multiply-add only in the
// activation's 24-bit fixed-point representation (relative to the row's
// largest element) and the final conversions.
//
// Tiles: 128 rows x 128 columns per CTA, k in steps of 128 bytes. A (the
// limbs) and B (the codes, 16 KB blocks) are K-major, both loaded by TMA with
// the 128-byte swizzle; a 3-stage ring of 64 KB stages. Warp 0 issues the TMA
// loads, warp 1 (one thread) the MMAs and commits, warps 4-7 drain the
// accumulators (tcgen05.ld) and run the epilogue. Every wait is bounded.
#pragma once
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

#include "qmma.cuh"

namespace dz {

constexpr int UG_BM = 128;
constexpr int UG_BN = 128;
constexpr int UG_BK = 128;
constexpr int UG_STAGES = 3;
constexpr int UG_LIMBS = 3;
constexpr int UG_THREADS = 256;
constexpr uint32_t UG_A_BYTES = UG_BM * UG_BK;   // one limb tile
constexpr uint32_t UG_B_BYTES = UG_BK * UG_BN;
constexpr uint32_t UG_STAGE_BYTES = UG_LIMBS * UG_A_BYTES + UG_B_BYTES;
constexpr uint32_t UG_TMEM_COLS = 512;           // three 128-column int32 accumulators
// + alignment slack, the barriers and progress words, and the tile's column
// scales and biases (2 x UG_BN floats)
constexpr size_t UG_SMEM_BYTES = (size_t)UG_STAGES * UG_STAGE_BYTES + 1024 + 256 + 2 * UG_BN * 4;
constexpr int UG_ROW_NONFINITE = -0x40000000;    // row exponent marking a non-finite input row
constexpr int UG_TILE_LD = UG_BN + 4;            // staging tile row stride (floats): 16-byte rows, spread banks
constexpr int UG_PART_LD = UG_BN + 2;            // split-K int64 staging row stride: 65 16-byte units
// Largest K for which the int32 limb sums are exact: |q| <= 127, |limb| <=
// 128, and 131072 * 128 * 127 < 2^31.
constexpr int UG_MAX_K = 131072;
constexpr int UG_X_BITS = 22;                    // |X| <= 2^22 after scaling

struct UgArgs {
    int M, N, K, nkb;             // nkb: k blocks of UG_BK
    const int* shift;             // [M] -s, or UG_ROW_NONFINITE
    int* status;                  // set to 1 when a wait gave up (may be null)
    QmvEpilogue ep;               // col_scale etc.; row_shift unused
    // split-K (kparts > 1, grid z = kparts): CTA z takes k blocks
    // [z nkb / kparts, (z + 1) nkb / kparts) of its tile and stores the
    // tile's int64 totals as partial[tile][z][UG_BM][UG_BN]; the per-tile
    // counter (zero between launches) finds the last part, which adds the
    // parts, finishes the tile and resets the counter
    int kparts;
    long long* partial;
    int* counters;
};

// ------------------------------------------------------------ PTX wrappers

__device__ __forceinline__ void ug_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void ug_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// K-major operand, 128-byte swizzle: rows of 128 bytes, 8-row groups 1024
// bytes apart (stride byte offset), leading byte offset unused (1).
__device__ __forceinline__ uint64_t ug_desc_kmajor(uint32_t saddr) {
    uint64_t d = (uint64_t)((saddr >> 4) & 0x3FFFu);
    d |= (uint64_t)1u << 16;
    d |= (uint64_t)(1024u >> 4) << 32;
    d |= (uint64_t)1u << 46;   // descriptor version (sm_100)
    d |= (uint64_t)2u << 61;   // SWIZZLE_128B
    return d;
}

// Instruction descriptor for kind::i8, int32 accumulate, A = limb K-major
// (s8), B = codes K-major s8, M = UG_BM, N = UG_BN.
__device__ __forceinline__ uint32_t ug_idesc() {
    uint32_t d = 2u << 4;                   // D format S32
    d |= 1u << 7;                           // A: s8 (balanced limbs)
    d |= 1u << 10;                          // B: s8 (signed codes)
    d |= 0u << 16;                          // B K-major
    d |= (uint32_t)(UG_BN >> 3) << 17;
    d |= (uint32_t)(UG_BM >> 4) << 24;
    return d;
}

__device__ __forceinline__ void ug_mma(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                       uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Arrive on `bar` once every MMA this thread issued so far has completed.
__device__ __forceinline__ void ug_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(dz_smem_addr(bar))
                 : "memory");
}

__device__ __forceinline__ void ug_tma_3d(void* dst, const CUtensorMap* tm, int c0, int c1, int c2, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(
            dz_smem_addr(dst)),
        "l"(reinterpret_cast<uint64_t>(tm)), "r"(c0), "r"(c1), "r"(c2), "r"(dz_smem_addr(bar))
        : "memory");
}

__device__ __forceinline__ void ug_tma_4d(void* dst, const CUtensorMap* tm, int c0, int c1, int c2, int c3,
                                          uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], "
        "[%6];" ::"r"(dz_smem_addr(dst)),
        "l"(reinterpret_cast<uint64_t>(tm)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(dz_smem_addr(bar))
        : "memory");
}

// The same with an L2 cache policy (createpolicy), for streamed weights.
__device__ __forceinline__ void ug_tma_4d_hint(void* dst, const CUtensorMap* tm, int c0, int c1, int c2, int c3,
                                               uint64_t* bar, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint "
        "[%0], [%1, {%2, %3, %4, %5}], [%6], %7;" ::"r"(dz_smem_addr(dst)),
        "l"(reinterpret_cast<uint64_t>(tm)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(dz_smem_addr(bar)), "l"(policy)
        : "memory");
}

// 32 consecutive int32 columns of this warp's 32 TMEM lanes (one per thread).
__device__ __forceinline__ void ug_tmem_ld32(uint32_t taddr, int32_t (&v)[32]) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 32; i++) v[i] = (int32_t)r[i];
}

// ------------------------------------------------------- weight bytes

// INT4 codes (two per byte, even index in the low nibble, src/core/
// quantize.c:213-221) of a k x cols matrix -> one byte per code in rows of
// `ld` bytes.
// The code copy for the tensor-core kernels: the signed levels q = code - qmax
// (in [-qmax, qmax]: loaded blobs hold no code above 2 * qmax) as s8 in
// K-major 16 KB blocks, codes[tile][kb][n % 128][k % 128] with tile = n / 128
// and kb = k / 128, so one TMA box (128 n x 128 k) is one contiguous read and
// lands as the K-major operand the 8-bit MMA reads at full rate. Source: the
// reference's k x cols order (INT8 bytes or packed nibbles, low nibble first)
// placed at columns [off, off + cols). Padding (n >= N, k >= K) stays as the
// caller zeroed it (q = 0).
DZ_KERNEL_LINKAGE __global__ void dz_code_blocks_kernel(const uint8_t* __restrict__ packed, int bits, long long cols, long long total,
                                      int8_t* __restrict__ codes, int nkb, int off) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= total) return;
    const long long k = i / cols, n = off + (i - k * cols);
    const int c = bits == 8 ? (int)packed[i] - 127 : (int)((packed[i >> 1] >> ((i & 1) * 4)) & 0xF) - 7;
    const long long blk = (n / UG_BN) * nkb + k / UG_BK;
    codes[(blk * UG_BN + n % UG_BN) * UG_BK + k % UG_BK] = (int8_t)c;
}

// ------------------------------------------------------- activation limbs

// X of one element: rint(v * 2^s) (|X| <= 2^22 for finite v), 0 for a
// non-finite v (the row is flagged separately).
__device__ __forceinline__ int ug_fixed(float v, int s) {
    if (!(fabsf(v) <= 3.402823466e38f)) return 0;
    const float f = rintf(dz_mul_pow2(v, s));
    const float lim = (float)(1 << UG_X_BITS);
    return f >= lim ? (1 << UG_X_BITS) : f <= -lim ? -(1 << UG_X_BITS) : (int)f;
}
// Balanced base-256 digits of X: X = 65536 * t + 256 * m + l, l, m in
// [-128, 127], |t| <= 64; each returned as its byte.
__device__ __forceinline__ void ug_digits(int X, uint32_t& t, uint32_t& m, uint32_t& l) {
    const int d0 = (int)(int8_t)(X & 0xFF);
    const int x1 = (X - d0) >> 8;
    const int d1 = (int)(int8_t)(x1 & 0xFF);
    const int d2 = (x1 - d1) >> 8;
    l = (uint32_t)d0 & 0xFFu;
    m = (uint32_t)d1 & 0xFFu;
    t = (uint32_t)d2 & 0xFFu;
}

// One pass over a row of K <= UG_SPLIT_REG_K elements (K % 4 == 0, row and
// k_scale 16-byte aligned): thread t holds the float4s 4 (j * 256 + t) of the
// row in registers, so the row is read once; the maximum, exponent and limbs
// are those of the two-pass form below.
constexpr int UG_SPLIT_REG_V = 8;                          // float4s per thread
constexpr int UG_SPLIT_REG_K = 256 * 4 * UG_SPLIT_REG_V;   // 8192
__device__ __forceinline__ void ug_limb_split_row_regs(const float* __restrict__ x, const float* __restrict__ k_scale,
                                                       int r, int M, int K, int Kp, int8_t* __restrict__ L,
                                                       int* __restrict__ shift, float* wred, int* wbad) {
    float4 v[UG_SPLIT_REG_V];
    float m = 0.0f;
    int bad = 0;
#pragma unroll
    for (int j = 0; j < UG_SPLIT_REG_V; j++) {
        const int k0 = (j * 256 + (int)threadIdx.x) * 4;
        v[j] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        if (k0 < K) {
            v[j] = *reinterpret_cast<const float4*>(x + k0);
            if (k_scale) {
                const float4 w = *reinterpret_cast<const float4*>(k_scale + k0);
                v[j].x *= w.x;
                v[j].y *= w.y;
                v[j].z *= w.z;
                v[j].w *= w.w;
            }
        }
        const float e[4] = {v[j].x, v[j].y, v[j].z, v[j].w};
#pragma unroll
        for (int c = 0; c < 4; c++) {
            if (!(fabsf(e[c]) <= 3.402823466e38f)) bad = 1;
            else m = fmaxf(m, fabsf(e[c]));
        }
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) {
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
        bad |= __shfl_xor_sync(0xffffffffu, bad, off);
    }
    if ((threadIdx.x & 31) == 0) {
        wred[threadIdx.x >> 5] = m;
        wbad[threadIdx.x >> 5] = bad;
    }
    __syncthreads();
    float amax = 0.0f;
    for (int w = 0; w < (int)(blockDim.x >> 5); w++) {
        amax = fmaxf(amax, wred[w]);
        bad |= wbad[w];
    }
    const int s = amax > 0.0f ? (UG_X_BITS - 1) - dz_ilogb(amax) : 0;
    const size_t plane = (size_t)M * Kp;
#pragma unroll
    for (int j = 0; j < UG_SPLIT_REG_V; j++) {
        const int k0 = (j * 256 + (int)threadIdx.x) * 4;
        if (k0 >= Kp) continue;
        const float e[4] = {v[j].x, v[j].y, v[j].z, v[j].w};   // zero past K
        uint32_t t4 = 0, m4 = 0, l4 = 0;
#pragma unroll
        for (int c = 0; c < 4; c++) {
            uint32_t dt, dm, dl;
            ug_digits(ug_fixed(e[c], s), dt, dm, dl);
            t4 |= dt << (8 * c);
            m4 |= dm << (8 * c);
            l4 |= dl << (8 * c);
        }
        const size_t at = (size_t)r * Kp + k0;
        *reinterpret_cast<uint32_t*>(L + at) = t4;
        *reinterpret_cast<uint32_t*>(L + plane + at) = m4;
        *reinterpret_cast<uint32_t*>(L + 2 * plane + at) = l4;
    }
    if (threadIdx.x == 0) shift[r] = bad ? UG_ROW_NONFINITE : -s;
}

// One block per row: X = rint(x * k_scale * 2^s), stored as three signed limb
// planes L[limb][M][Kp] (zero past K), and -s.
DZ_KERNEL_LINKAGE __global__ void __launch_bounds__(256) dz_limb_split_kernel(const float* __restrict__ X, long long ldx,
                                                            const float* __restrict__ k_scale, int M, int K, int Kp,
                                                            int8_t* __restrict__ L, int* __restrict__ shift) {
    __shared__ float wred[8];
    __shared__ int wbad[8];
    // launched as a programmatic dependent of the previous kernel (a GEMM
    // that may still read this scratch's limbs): the GEMM after this split
    // may launch now, and nothing here is read or written before the
    // previous kernel completed
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const int r = blockIdx.x;
    const float* x = X + (long long)r * ldx;
    if (blockDim.x == 256 && K <= UG_SPLIT_REG_K && (K & 3) == 0 &&
        ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(k_scale)) & 15u) == 0) {
        ug_limb_split_row_regs(x, k_scale, r, M, K, Kp, L, shift, wred, wbad);
        return;
    }
    float m = 0.0f;
    int bad = 0;
#pragma unroll 8
    for (int k = threadIdx.x; k < K; k += blockDim.x) {
        float v = x[k];
        if (k_scale) v *= k_scale[k];
        if (!(fabsf(v) <= 3.402823466e38f)) bad = 1;
        else m = fmaxf(m, fabsf(v));
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) {
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
        bad |= __shfl_xor_sync(0xffffffffu, bad, off);
    }
    if ((threadIdx.x & 31) == 0) {
        wred[threadIdx.x >> 5] = m;
        wbad[threadIdx.x >> 5] = bad;
    }
    __syncthreads();
    float amax = 0.0f;
    for (int w = 0; w < (int)(blockDim.x >> 5); w++) {
        amax = fmaxf(amax, wred[w]);
        bad |= wbad[w];
    }
    const int s = amax > 0.0f ? (UG_X_BITS - 1) - dz_ilogb(amax) : 0;
    const size_t plane = (size_t)M * Kp;
    for (int k0 = threadIdx.x * 4; k0 < Kp; k0 += blockDim.x * 4) {
        uint32_t t4 = 0, m4 = 0, l4 = 0;
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const int k = k0 + j;
            int xi = 0;
            if (k < K) {
                float v = x[k];
                if (k_scale) v *= k_scale[k];
                xi = ug_fixed(v, s);
            }
            uint32_t dt, dm, dl;
            ug_digits(xi, dt, dm, dl);
            t4 |= dt << (8 * j);
            m4 |= dm << (8 * j);
            l4 |= dl << (8 * j);
        }
        const size_t at = (size_t)r * Kp + k0;
        *reinterpret_cast<uint32_t*>(L + at) = t4;
        *reinterpret_cast<uint32_t*>(L + plane + at) = m4;
        *reinterpret_cast<uint32_t*>(L + 2 * plane + at) = l4;
    }
    if (threadIdx.x == 0) shift[r] = bad ? UG_ROW_NONFINITE : -s;
}

// The limb split for many rows: one warp per row, eight rows per block, no
// block barriers. Pass 1 finds the row's maximum (and non-finite elements)
// with 16-byte loads; pass 2 reads the row again (from L1/L2) and writes the
// three limb planes, 4 bytes per lane per plane per step (128-byte coalesced
// stores), zero past K. The same limbs and exponents as dz_limb_split_kernel.
constexpr int UG_SPLIT_WARP_ROWS = 8;
DZ_KERNEL_LINKAGE __global__ void __launch_bounds__(256) dz_limb_split_warp_kernel(const float* __restrict__ X, long long ldx,
                                                                 const float* __restrict__ k_scale, int M, int K,
                                                                 int Kp, int8_t* __restrict__ L,
                                                                 int* __restrict__ shift) {
    // a programmatic dependent, as dz_limb_split_kernel
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const int lane = threadIdx.x & 31;
    const int r = blockIdx.x * UG_SPLIT_WARP_ROWS + (threadIdx.x >> 5);
    if (r >= M) return;
    const float* x = X + (long long)r * ldx;
    const bool vec = (K & 3) == 0 &&
                     ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(k_scale)) & 15u) == 0;
    auto load4 = [&](int k0, float (&v)[4]) {
        if (vec && k0 + 3 < K) {
            const float4 q = *reinterpret_cast<const float4*>(x + k0);
            v[0] = q.x; v[1] = q.y; v[2] = q.z; v[3] = q.w;
            if (k_scale) {
                const float4 w = *reinterpret_cast<const float4*>(k_scale + k0);
                v[0] *= w.x; v[1] *= w.y; v[2] *= w.z; v[3] *= w.w;
            }
        } else {
#pragma unroll
            for (int j = 0; j < 4; j++) {
                v[j] = 0.0f;
                if (k0 + j < K) {
                    v[j] = x[k0 + j];
                    if (k_scale) v[j] *= k_scale[k0 + j];
                }
            }
        }
    };
    float m = 0.0f;
    int bad = 0;
#pragma unroll 4
    for (int k0 = lane * 4; k0 < K; k0 += 128) {
        float v[4];
        load4(k0, v);
#pragma unroll
        for (int j = 0; j < 4; j++) {
            if (!(fabsf(v[j]) <= 3.402823466e38f)) bad = 1;
            else m = fmaxf(m, fabsf(v[j]));
        }
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) {
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
        bad |= __shfl_xor_sync(0xffffffffu, bad, off);
    }
    const int s = m > 0.0f ? (UG_X_BITS - 1) - dz_ilogb(m) : 0;
    const size_t plane = (size_t)M * Kp;
#pragma unroll 4
    for (int k0 = lane * 4; k0 < Kp; k0 += 128) {
        float v[4];
        load4(k0, v);   // zero past K
        uint32_t t4 = 0, m4 = 0, l4 = 0;
#pragma unroll
        for (int j = 0; j < 4; j++) {
            uint32_t dt, dm, dl;
            ug_digits(ug_fixed(v[j], s), dt, dm, dl);
            t4 |= dt << (8 * j);
            m4 |= dm << (8 * j);
            l4 |= dl << (8 * j);
        }
        const size_t at = (size_t)r * Kp + k0;
        *reinterpret_cast<uint32_t*>(L + at) = t4;
        *reinterpret_cast<uint32_t*>(L + plane + at) = m4;
        *reinterpret_cast<uint32_t*>(L + 2 * plane + at) = l4;
    }
    if (lane == 0) shift[r] = bad ? UG_ROW_NONFINITE : -s;
}

// Columns [n0, n0 + UG_BN) of rows [m0, m0 + UG_BM) through the epilogue
// (column scale, bias, residual, activation, segment routing), a warp per
// row and four columns per lane, float4 accesses where the addresses allow.
// get4(r0, y) gives this lane's four values of tile rows r0 .. r0 + 3 (a
// warp takes four rows at a time, so their loads can be in flight together).
// The bias / residual / activation choice is a template argument: the
// generic form with all three decided per element at run time measured about
// three times slower over a tile (3.4 against 1.1 us) than the specialised
// one. Every field is read once, with constant indices, into registers (see
// dz_seg_of).
template <bool HB, bool HR, int ACT, typename Get4>
__device__ __forceinline__ void ug_store_rows_t(const UgArgs& a, int m0, int n0, const float* cols, Get4 get4) {
    const QmvEpilogue& e = a.ep;
    const int M = a.M, N = a.N;
    const int c4 = (threadIdx.x & 31) * 4;   // fixed per thread: blockDim.x is a multiple of 32
    const int n = n0 + c4;
    if (n >= N) return;
    const int nv = N - n < 4 ? N - n : 4;
    const float* col_scale = e.col_scale;
    const float* residual = e.residual;
    const long long ld_res = e.ld_res;
    // column scales and biases: from the tile's shared table (loaded by the
    // idle warps during the main loop) when there is one
    float sc[4], bi[4];
#pragma unroll
    for (int j = 0; j < 4; j++) {
        sc[j] = (j < nv && col_scale) ? (cols ? cols[c4 + j] : col_scale[n + j]) : 1.0f;
        bi[j] = (HB && j < nv) ? (cols ? cols[UG_BN + c4 + j] : e.bias[n + j]) : 0.0f;
    }
    const DzSeg sg = dz_seg_of(e, n);
    const bool one_seg = nv == 4 && n + 3 < sg.end;
    // this lane's four columns of one segment: row r goes to base + r * ld
    // (+ row_off[r]); 16-byte stores when base and ld keep them aligned
    float* const base = sg.ptr + (n - sg.start);
    const long long ld = sg.ld;
    const int* const row_off = sg.row_off;
    const bool vec = one_seg && ((reinterpret_cast<uintptr_t>(base) & 15) == 0) && (ld & 3) == 0;
    for (int r0 = (threadIdx.x >> 5) * 4; r0 < UG_BM && m0 + r0 < M; r0 += (UG_THREADS / 32) * 4) {
        float yy[4][4];
        get4(r0, yy);
        // the four rows' residuals and ring-row offsets, loaded before any store
        float rs[4][4];
        int ro[4] = {0, 0, 0, 0};
        if (row_off) {
#pragma unroll
            for (int i = 0; i < 4; i++) ro[i] = m0 + r0 + i < M ? row_off[m0 + r0 + i] : 0;
        }
        if (HR) {
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const int row = m0 + r0 + i;
#pragma unroll
                for (int j = 0; j < 4; j++)
                    rs[i][j] = (row < M && j < nv) ? residual[(long long)row * ld_res + n + j] : 0.0f;
            }
        }
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const int row = m0 + r0 + i;
            if (row >= M) break;
            float y0 = yy[i][0], y1 = yy[i][1], y2 = yy[i][2], y3 = yy[i][3];
            if (col_scale) {
                y0 = y0 * sc[0]; y1 = y1 * sc[1]; y2 = y2 * sc[2]; y3 = y3 * sc[3];
            }
            if (HB) {
                y0 = y0 + bi[0]; y1 = y1 + bi[1]; y2 = y2 + bi[2]; y3 = y3 + bi[3];
            }
            if (HR) {
                y0 = y0 + rs[i][0]; y1 = y1 + rs[i][1]; y2 = y2 + rs[i][2]; y3 = y3 + rs[i][3];
            }
            if (ACT) {
                y0 = dz_act(y0, ACT); y1 = dz_act(y1, ACT); y2 = dz_act(y2, ACT); y3 = dz_act(y3, ACT);
            }
            if (vec) {
                *reinterpret_cast<float4*>(base + (long long)row * ld + ro[i]) = make_float4(y0, y1, y2, y3);
                continue;
            }
            if (one_seg) {
                float* dst = base + (long long)row * ld + ro[i];
                dst[0] = y0; dst[1] = y1; dst[2] = y2; dst[3] = y3;
                continue;
            }
            const float yv[4] = {y0, y1, y2, y3};
            for (int j = 0; j < nv; j++) {
                const DzSeg sj = dz_seg_of(e, n + j);
                long long off = (long long)row * sj.ld + (n + j - sj.start);
                if (sj.row_off) off += sj.row_off[row];
                sj.ptr[off] = yv[j];
            }
        }
    }
}

template <typename Get4>
__device__ __forceinline__ void ug_store_rows(const UgArgs& a, int m0, int n0, const float* cols, Get4 get4) {
    const bool hb = a.ep.bias != nullptr, hr = a.ep.residual != nullptr;
    const int act = a.ep.act;
    if (act == DZ_ACT_RELU) {
        if (hr) hb ? ug_store_rows_t<true, true, DZ_ACT_RELU>(a, m0, n0, cols, get4)
                   : ug_store_rows_t<false, true, DZ_ACT_RELU>(a, m0, n0, cols, get4);
        else hb ? ug_store_rows_t<true, false, DZ_ACT_RELU>(a, m0, n0, cols, get4)
                : ug_store_rows_t<false, false, DZ_ACT_RELU>(a, m0, n0, cols, get4);
    } else if (act == DZ_ACT_GELU) {
        if (hr) hb ? ug_store_rows_t<true, true, DZ_ACT_GELU>(a, m0, n0, cols, get4)
                   : ug_store_rows_t<false, true, DZ_ACT_GELU>(a, m0, n0, cols, get4);
        else hb ? ug_store_rows_t<true, false, DZ_ACT_GELU>(a, m0, n0, cols, get4)
                : ug_store_rows_t<false, false, DZ_ACT_GELU>(a, m0, n0, cols, get4);
    } else {
        if (hr) hb ? ug_store_rows_t<true, true, DZ_ACT_NONE>(a, m0, n0, cols, get4)
                   : ug_store_rows_t<false, true, DZ_ACT_NONE>(a, m0, n0, cols, get4);
        else hb ? ug_store_rows_t<true, false, DZ_ACT_NONE>(a, m0, n0, cols, get4)
                : ug_store_rows_t<false, false, DZ_ACT_NONE>(a, m0, n0, cols, get4);
    }
}

// The same from the fp32 staging tile ([UG_BM][UG_TILE_LD]); a failed tile reads NaN.
__device__ __forceinline__ void ug_store_tile(const UgArgs& a, const float* tile, int m0, int n0, bool failed,
                                              const float* cols) {
    const int c4 = (threadIdx.x & 31) * 4;
    ug_store_rows(a, m0, n0, cols, [&](int r0, float (*y)[4]) {
#pragma unroll
        for (int i = 0; i < 4; i++) {
            float4 t = *reinterpret_cast<const float4*>(tile + (r0 + i) * UG_TILE_LD + c4);
            if (failed) t.x = t.y = t.z = t.w = __int_as_float(0x7fc00000);
            y[i][0] = t.x; y[i][1] = t.y; y[i][2] = t.z; y[i][3] = t.w;
        }
    });
}

constexpr int UG_SPLIT_CHUNK = 1024;   // k per block of dz_limb_split_chunk_kernel

// The limb split for few rows: grid (ceil(Kp / UG_SPLIT_CHUNK), M). Every
// block reads its whole row once (thread t holds elements c * 1024 + 4t ..
// + 3 of every chunk c; float4 loads when the row and k_scale are 16-byte
// aligned and K % 4 == 0), keeps its own chunk's four in registers, finds the
// row's maximum (the same exponent in every block) and converts those four:
// one global round trip. It lets the GEMV launched after it start at once
// (programmatic dependent launch): the GEMV streams weights and waits for
// this grid only before it reads the limbs.
DZ_KERNEL_LINKAGE __global__ void __launch_bounds__(256) dz_limb_split_chunk_kernel(const float* __restrict__ X, long long ldx,
                                                                  const float* __restrict__ k_scale, int M, int K,
                                                                  int Kp, int8_t* __restrict__ L,
                                                                  int* __restrict__ shift) {
    __shared__ float wred[8];
    __shared__ int wbad[8];
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    // launched as a programmatic dependent of the previous kernel (a GEMV
    // that may still read this scratch's limbs): nothing is read or written
    // before that kernel completed
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const int r = blockIdx.y, ch = blockIdx.x;
    const float* x = X + (long long)r * ldx;
    const bool vec = (K & 3) == 0 &&
                     ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(k_scale)) & 15u) == 0;
    const int nch = (K + UG_SPLIT_CHUNK - 1) / UG_SPLIT_CHUNK;
    float mine[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    float m = 0.0f;
    int bad = 0;
#pragma unroll 4
    for (int c = 0; c < nch; c++) {
        const int k0 = c * UG_SPLIT_CHUNK + threadIdx.x * 4;
        float v[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        if (vec) {
            if (k0 < K) {
                const float4 q = *reinterpret_cast<const float4*>(x + k0);
                v[0] = q.x;
                v[1] = q.y;
                v[2] = q.z;
                v[3] = q.w;
                if (k_scale) {
                    const float4 w = *reinterpret_cast<const float4*>(k_scale + k0);
                    v[0] *= w.x;
                    v[1] *= w.y;
                    v[2] *= w.z;
                    v[3] *= w.w;
                }
            }
        } else {
#pragma unroll
            for (int j = 0; j < 4; j++)
                if (k0 + j < K) {
                    v[j] = x[k0 + j];
                    if (k_scale) v[j] *= k_scale[k0 + j];
                }
        }
#pragma unroll
        for (int j = 0; j < 4; j++) {
            if (!(fabsf(v[j]) <= 3.402823466e38f)) bad = 1;
            else m = fmaxf(m, fabsf(v[j]));
            if (c == ch) mine[j] = v[j];
        }
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) {
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
        bad |= __shfl_xor_sync(0xffffffffu, bad, off);
    }
    if ((threadIdx.x & 31) == 0) {
        wred[threadIdx.x >> 5] = m;
        wbad[threadIdx.x >> 5] = bad;
    }
    __syncthreads();
    float amax = 0.0f;
    for (int w = 0; w < (int)(blockDim.x >> 5); w++) {
        amax = fmaxf(amax, wred[w]);
        bad |= wbad[w];
    }
    const int s = amax > 0.0f ? (UG_X_BITS - 1) - dz_ilogb(amax) : 0;
    const size_t plane = (size_t)M * Kp;
    const int k0 = ch * UG_SPLIT_CHUNK + threadIdx.x * 4;
    if (k0 < Kp) {
        uint32_t t4 = 0, m4 = 0, l4 = 0;
#pragma unroll
        for (int j = 0; j < 4; j++) {
            uint32_t dt, dm, dl;
            ug_digits(ug_fixed(mine[j], s), dt, dm, dl);   // zero past K
            t4 |= dt << (8 * j);
            m4 |= dm << (8 * j);
            l4 |= dl << (8 * j);
        }
        const size_t at = (size_t)r * Kp + k0;
        *reinterpret_cast<uint32_t*>(L + at) = t4;
        *reinterpret_cast<uint32_t*>(L + plane + at) = m4;
        *reinterpret_cast<uint32_t*>(L + 2 * plane + at) = l4;
    }
    if (threadIdx.x == 0 && ch == 0) shift[r] = bad ? UG_ROW_NONFINITE : -s;
}

// ------------------------------------------------------------------- GEMM

DZ_KERNEL_LINKAGE __global__ void __launch_bounds__(UG_THREADS, 1)
    dz_ugemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, UgArgs a) {
    // launched as a programmatic dependent of its limb split: the weight
    // tiles of the first stages load before the split grid completes; the
    // limbs, row exponents and epilogue inputs are read only after
    // griddepcontrol.wait. The next call's split may launch now (it waits for
    // this grid before touching memory).
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    extern __shared__ __align__(1024) uint8_t ug_raw[];
    const uint32_t raw = dz_smem_addr(ug_raw);
    uint8_t* sm = ug_raw + ((1024u - (raw & 1023u)) & 1023u);
    uint64_t* full = reinterpret_cast<uint64_t*>(sm + (size_t)UG_STAGES * UG_STAGE_BYTES);
    uint64_t* empty = full + UG_STAGES;
    uint64_t* accum = empty + UG_STAGES;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accum + 1);
    // [0] stages issued, [1] stages consumed, [2] failed, [3] last split-K part
    int* progress = reinterpret_cast<int*>(tmem_slot + 1);
    // the tile's column scales [UG_BN] and biases [UG_BN]
    float* cols = reinterpret_cast<float*>(sm + (size_t)UG_STAGES * UG_STAGE_BYTES + 256);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n0 = blockIdx.x * UG_BN, m0 = blockIdx.y * UG_BM;
    // this CTA's k blocks (all of them unless split-K)
    const int kb0 = (int)(((long long)a.nkb * blockIdx.z) / a.kparts);
    const int nkb = (int)(((long long)a.nkb * (blockIdx.z + 1)) / a.kparts) - kb0;
    auto stage_a = [&](int s, int limb) { return sm + (size_t)s * UG_STAGE_BYTES + (size_t)limb * UG_A_BYTES; };
    auto stage_b = [&](int s) { return sm + (size_t)s * UG_STAGE_BYTES + (size_t)UG_LIMBS * UG_A_BYTES; };

    if (threadIdx.x == 0) {
        for (int s = 0; s < UG_STAGES; s++) {
            dz_mbar_init(&full[s]);
            dz_mbar_init(&empty[s]);
        }
        dz_mbar_init(accum);
        progress[0] = progress[1] = progress[2] = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dz_smem_addr(tmem_slot)),
                     "r"(UG_TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    ug_fence_before();
    __syncthreads();
    ug_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
      if (lane == 0) {
        // producer: TMA loads of the three limb tiles and the code tile per k block
        // the first stages' weight tiles go out before the split is waited for
        const int pre = nkb < UG_STAGES ? nkb : UG_STAGES;
        for (int kb = 0; kb < pre; kb++) {
            dz_mbar_expect_tx(&full[kb], UG_STAGE_BYTES);
            ug_tma_4d(stage_b(kb), &tmB, 0, 0, kb0 + kb, blockIdx.x, &full[kb]);
        }
        asm volatile("griddepcontrol.wait;" ::: "memory");
        int kb = 0;
        for (; kb < nkb; kb++) {
            const int s = kb % UG_STAGES;
            if (kb >= UG_STAGES && !dz_mbar_wait(&empty[s], (uint32_t)(((kb / UG_STAGES) - 1) & 1))) {
                progress[2] = 1;
                break;
            }
            if (kb >= pre) {
                dz_mbar_expect_tx(&full[s], UG_STAGE_BYTES);
                ug_tma_4d(stage_b(s), &tmB, 0, 0, kb0 + kb, blockIdx.x, &full[s]);
            }
            for (int limb = 0; limb < UG_LIMBS; limb++)
                ug_tma_3d(stage_a(s, limb), &tmA, (kb0 + kb) * UG_BK, m0, limb, &full[s]);
        }
        progress[0] = kb;
      }
      __syncwarp();   // the warp reconverges before the block barriers below
    } else if (warp == 1) {
      if (lane == 0) {
        // MMA issuer: 3 limbs x 4 k-steps of 32 per stage
        int kb = 0;
        const uint32_t idesc = ug_idesc();
        for (; kb < nkb; kb++) {
            const int s = kb % UG_STAGES;
            if (!dz_mbar_wait(&full[s], (uint32_t)((kb / UG_STAGES) & 1))) {
                progress[2] = 1;
                break;
            }
            ug_fence_after();
            const uint32_t b_addr = dz_smem_addr(stage_b(s));
#pragma unroll
            for (int limb = 0; limb < UG_LIMBS; limb++) {
                const uint32_t a_addr = dz_smem_addr(stage_a(s, limb));
#pragma unroll
                for (int kk = 0; kk < UG_BK / 32; kk++) {
                    const uint64_t ad = ug_desc_kmajor(a_addr + kk * 32);
                    const uint64_t bd = ug_desc_kmajor(b_addr + kk * 32);
                    ug_mma(tmem + (uint32_t)(limb * UG_BN), ad, bd, idesc, (kb > 0 || kk > 0) ? 1u : 0u);
                }
            }
            ug_commit(&empty[s]);
        }
        progress[1] = kb;
        ug_commit(accum);   // completes once every MMA issued above has
      }
      __syncwarp();
    } else if (warp == 2 || warp == 3) {
        // the epilogue's column scales and biases, read while the main loop
        // runs (kernel inputs that no earlier grid writes)
        const int t = (warp - 2) * 32 + lane;
        for (int c = t; c < UG_BN; c += 64) {
            const int n = n0 + c;
            cols[c] = (n < a.N && a.ep.col_scale) ? a.ep.col_scale[n] : 1.0f;
            cols[UG_BN + c] = (n < a.N && a.ep.bias) ? a.ep.bias[n] : 0.0f;
        }
    } else if (warp >= 4) {
        // epilogue, part 1: thread = row; drain the three accumulators into a
        // staging tile in the pipeline buffers (free once the accumulator
        // barrier completes): fp32 [128][UG_TILE_LD], or with split-K the
        // int64 totals [128][UG_PART_LD] (exact, so the parts add in any order)
        const int ew = warp - 4;
        bool ok = dz_mbar_wait(accum, 0);
        ug_fence_after();
        asm volatile("griddepcontrol.wait;" ::: "memory");   // the split's exponents (and epilogue inputs)
        const int rl = ew * 32 + lane;
        const int row = m0 + rl;
        const uint32_t lane_base = (uint32_t)(ew * 32) << 16;
        const int e = row < a.M ? a.shift[row] : 0;
        if (!ok || progress[2]) {
            if (a.status && lane == 0) atomicExch(a.status, 1);
            ok = false;
            progress[2] = 1;
        }
        float* tile = reinterpret_cast<float*>(sm);
        long long* srow = reinterpret_cast<long long*>(sm) + (size_t)rl * UG_PART_LD;
        for (int c0 = 0; c0 < UG_BN; c0 += 32) {
            int32_t top[32], mid[32], low[32];
            ug_tmem_ld32(tmem + lane_base + (uint32_t)c0, top);
            ug_tmem_ld32(tmem + lane_base + (uint32_t)(UG_BN + c0), mid);
            ug_tmem_ld32(tmem + lane_base + (uint32_t)(2 * UG_BN + c0), low);
            if (a.kparts > 1) {
#pragma unroll
                for (int c = 0; c < 32; c += 2) {
                    longlong2 v;
                    v.x = (long long)top[c] * 65536 + (long long)mid[c] * 256 + (long long)low[c];
                    v.y = (long long)top[c + 1] * 65536 + (long long)mid[c + 1] * 256 + (long long)low[c + 1];
                    *reinterpret_cast<longlong2*>(srow + c0 + c) = v;
                }
                continue;
            }
#pragma unroll
            for (int q = 0; q < 8; q++) {
                float y[4];
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    const int c = 4 * q + j;
                    const long long v = (long long)top[c] * 65536 + (long long)mid[c] * 256 + (long long)low[c];
                    y[j] = dz_mul_pow2(__ll2float_rn(v), e);
                    if (!ok || e == UG_ROW_NONFINITE) y[j] = __int_as_float(0x7fc00000);
                }
                *reinterpret_cast<float4*>(tile + rl * UG_TILE_LD + c0 + 4 * q) = make_float4(y[0], y[1], y[2], y[3]);
            }
        }
    }

    asm volatile("griddepcontrol.wait;" ::: "memory");   // every thread: the split grid's writes are visible
    ug_fence_before();
    __syncthreads();
    bool finish = true;
    if (a.kparts > 1) {
        // split-K: every part stores its totals (all warps, a warp per row,
        // 32 bytes per lane: 1 KB contiguous per store pair); the part that
        // arrives last adds the parts and finishes
        int* last = progress + 3;
        const int tile_id = blockIdx.y * gridDim.x + blockIdx.x;
        const int c4 = lane * 4;
        long long* part = a.partial + ((size_t)tile_id * a.kparts + blockIdx.z) * UG_BM * UG_BN;
        const long long* stile = reinterpret_cast<const long long*>(sm);
        for (int r = warp; r < UG_BM; r += UG_THREADS / 32) {
            const longlong2 u0 = *reinterpret_cast<const longlong2*>(stile + (size_t)r * UG_PART_LD + c4);
            const longlong2 u1 = *reinterpret_cast<const longlong2*>(stile + (size_t)r * UG_PART_LD + c4 + 2);
            *reinterpret_cast<longlong2*>(part + (size_t)r * UG_BN + c4) = u0;
            *reinterpret_cast<longlong2*>(part + (size_t)r * UG_BN + c4 + 2) = u1;
        }
        __threadfence();
        __syncthreads();
        if (threadIdx.x == 0) {
            const int old = atomicAdd(&a.counters[tile_id], 1);
            *last = old == a.kparts - 1;
            if (*last) a.counters[tile_id] = 0;   // zero again for the next launch
        }
        __syncthreads();
        finish = *last != 0;
        if (finish) {
            __threadfence();
            // the parts' totals added (this part's from shared memory, the
            // others' from global), converted to fp32 once and 2^-s applied,
            // straight into the epilogue: a warp per row, four rows at a time
            const long long* base = a.partial + (size_t)tile_id * a.kparts * UG_BM * UG_BN;
            const int own = (int)blockIdx.z;
            ug_store_rows(a, m0, n0, cols, [&](int r0, float (*y)[4]) {
                long long v[4][4];
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    const longlong2 u0 = *reinterpret_cast<const longlong2*>(stile + (size_t)(r0 + i) * UG_PART_LD + c4);
                    const longlong2 u1 =
                        *reinterpret_cast<const longlong2*>(stile + (size_t)(r0 + i) * UG_PART_LD + c4 + 2);
                    v[i][0] = u0.x; v[i][1] = u0.y; v[i][2] = u1.x; v[i][3] = u1.y;
                }
                // the other parts three at a time, their loads issued together
                // (one round trip to L2 per batch instead of one per part)
                const int nother = a.kparts - 1;
                for (int b0 = 0; b0 < nother; b0 += 3) {
                    longlong2 w[3][4][2];
#pragma unroll
                    for (int q = 0; q < 3; q++) {
                        const int idx = b0 + q;
                        const int z = idx < own ? idx : idx + 1;
                        const long long* pz = base + (size_t)z * UG_BM * UG_BN + c4;
#pragma unroll
                        for (int i = 0; i < 4; i++) {
                            if (idx < nother) {
                                w[q][i][0] = *reinterpret_cast<const longlong2*>(pz + (size_t)(r0 + i) * UG_BN);
                                w[q][i][1] = *reinterpret_cast<const longlong2*>(pz + (size_t)(r0 + i) * UG_BN + 2);
                            } else {
                                w[q][i][0] = make_longlong2(0, 0);
                                w[q][i][1] = make_longlong2(0, 0);
                            }
                        }
                    }
#pragma unroll
                    for (int q = 0; q < 3; q++)
#pragma unroll
                        for (int i = 0; i < 4; i++) {
                            v[i][0] += w[q][i][0].x; v[i][1] += w[q][i][0].y;
                            v[i][2] += w[q][i][1].x; v[i][3] += w[q][i][1].y;
                        }
                }
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    const int row = m0 + r0 + i;
                    const int e = row < a.M ? a.shift[row] : 0;
#pragma unroll
                    for (int j = 0; j < 4; j++) {
                        y[i][j] = dz_mul_pow2(__ll2float_rn(v[i][j]), e);
                        if (e == UG_ROW_NONFINITE || progress[2]) y[i][j] = __int_as_float(0x7fc00000);
                    }
                }
            });
            finish = false;   // stored
        }
    }
    // epilogue, part 2, all warps: one warp per output row, lane = 4 columns,
    // so each store instruction writes 512 contiguous bytes
    if (finish) ug_store_tile(a, reinterpret_cast<const float*>(sm), m0, n0, progress[2] != 0, cols);

    // teardown: copies and MMAs in flight finish before the shared memory and
    // the tensor memory are released
    if (threadIdx.x == 0 && progress[2]) {
        for (int kb = progress[1]; kb < progress[0]; kb++)
            if (!dz_mbar_wait(&full[kb % UG_STAGES], (uint32_t)((kb / UG_STAGES) & 1))) break;
        dz_mbar_wait(accum, 0);
    }
    __syncthreads();
    if (warp == 1) {
        ug_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(UG_TMEM_COLS) : "memory");
    }
}

// ------------------------------------------------------------------- GEMV

// The same integer formulation for M <= 16 rows (decode matvecs), with the
// roles turned round so the tensor core's 128-row side holds output columns:
// D[128 n x 48] += codes[128 n x k] . limbs[k x 48], the code blocks as the
// K-major A operand (no dequantization) and the three limbs' 16 rows each
// (rows past M zero-filled by TMA) as one 48-row K-major B operand, so one
// MMA per 32 k serves all three limbs.
//
// Work is split stream-K: the ntiles x nkb (n-tile, k block) stages, tile
// major, are cut into gridDim.x equal contiguous ranges, one per CTA, so every
// CTA streams the same number of weight bytes. A CTA's range holds whole tiles
// and at most two pieces of tiles shared with its neighbours. A piece's three
// limb accumulators become int64 partials (exact, so order does not matter),
// stored in the CTA's slot 0 (the first segment of its range) or slot 1 (the
// last); the per-tile counter adds k blocks and the piece that completes the
// tile (counter reaches nkb) adds the other pieces and finishes: convert to
// fp32 once, apply 2^-s and the epilogue. That CTA resets the counter for the
// next launch. The codes are signed levels, so the products need no offset
// correction.
//
// The kernel is launched as a programmatic dependent of the limb split: the
// weight loads of the first UV_STAGES stages go out at once, and only the
// limb loads and the row exponents wait for the split grid
// (griddepcontrol.wait); every output store comes after that wait.
constexpr int UV_N = 16;                          // rows (tokens) per UMMA
constexpr int UV_STAGES = 9;
constexpr uint32_t UV_A_BYTES = UG_BN * UG_BK;    // 128 n x 128 k codes
constexpr uint32_t UV_B_BYTES = UV_N * UG_BK;     // 16 rows x 128 k, one limb
constexpr uint32_t UV_B_PITCH = (UV_B_BYTES + 1023) & ~1023u;
static_assert(UV_B_PITCH == UV_B_BYTES, "the three limb boxes of a stage form one 48-row operand");
constexpr uint32_t UV_STAGE_BYTES = UV_A_BYTES + UG_LIMBS * UV_B_PITCH;
constexpr uint32_t UV_ACC_COLS = UG_LIMBS * UV_N; // one accumulator set: 48 columns
constexpr uint32_t UV_TMEM_COLS = 128;            // two sets
constexpr size_t UV_SMEM_BYTES = (size_t)UV_STAGES * UV_STAGE_BYTES + 1024 + 512;
constexpr size_t UV_SLOT_ELEMS = (size_t)UG_BN * UV_N;   // int64 per partial slot
constexpr int UV_MIN_STAGES_PER_CTA = 4;

struct UvArgs {
    int M, N, K, nkb;             // nkb: k blocks of UG_BK per tile
    int ntiles;
    long long total;              // ntiles * nkb
    const int* shift;             // [M] -s, or UG_ROW_NONFINITE
    long long* partial;           // [gridDim.x][2][UV_SLOT_ELEMS]
    int* counter;                 // [ntiles], zero between launches
    int* status;
    QmvEpilogue ep;               // row_shift unused
};

// First stage of CTA c's range, and the CTA whose range holds stage p.
__device__ __forceinline__ long long uv_range_start(long long total, int c, int G) {
    return total * c / G;
}
__device__ __forceinline__ int uv_owner(long long total, long long p, int G) {
    return (int)(((p + 1) * G - 1) / total);
}

// Next segment of a CTA's range: the tile holding stage `pos`, its first k
// block and the k blocks up to the tile's or the range's end.
struct UvSeg {
    int tile, kb0, nk;
};
__device__ __forceinline__ UvSeg uv_segment(long long pos, long long end, int nkb) {
    UvSeg g;
    g.tile = (int)(pos / nkb);
    g.kb0 = (int)(pos - (long long)g.tile * nkb);
    g.nk = (int)min((long long)(nkb - g.kb0), end - pos);
    return g;
}

// Epilogue of one output column for rows 0..M-1 (M <= R): the column's scale,
// bias and output segment are looked up once and the residuals are loaded
// before any store, so the rows do not wait on one another.
template <int R>
__device__ __forceinline__ void dz_qmv_store_col(const QmvEpilogue& e, int M, int N, int n, const float (&acc)[R]) {
    if (n >= N) return;
    const float cs = e.col_scale ? e.col_scale[n] : 0.0f;
    const float bi = e.bias ? e.bias[n] : 0.0f;
    const DzSeg sg = dz_seg_of(e, n);   // constant indices only (see dz_seg_of)
    float res[R];
#pragma unroll
    for (int m = 0; m < R; m++) res[m] = (e.residual && m < M) ? e.residual[(long long)m * e.ld_res + n] : 0.0f;
    int roff[R];
#pragma unroll
    for (int m = 0; m < R; m++) roff[m] = (sg.row_off && m < M) ? sg.row_off[m] : 0;
#pragma unroll
    for (int m = 0; m < R; m++) {
        if (m >= M) break;
        float y = e.col_scale ? acc[m] * cs : acc[m];
        if (e.bias) y = y + bi;
        if (e.residual) y = y + res[m];
        if (e.act) y = dz_act(y, e.act);
        sg.ptr[(long long)m * sg.ld + (n - sg.start) + roff[m]] = y;
    }
}

__device__ __forceinline__ void ug_tmem_ld16(uint32_t taddr, int32_t (&v)[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; i++) v[i] = (int32_t)r[i];
}

// Instruction descriptor: A = codes (s8, K-major), B = the three limbs' rows
// (s8, K-major), M = 128 output columns, N = 3 x 16 limb rows, int32
// accumulate.
__device__ __forceinline__ uint32_t uv_idesc() {
    uint32_t d = 2u << 4;                 // D format S32
    d |= 1u << 7;                         // A: s8
    d |= 1u << 10;                        // B: s8
    d |= 0u << 15;                        // A K-major
    d |= 0u << 16;                        // B K-major
    d |= (uint32_t)((UG_LIMBS * UV_N) >> 3) << 17;
    d |= (uint32_t)(UG_BN >> 4) << 24;
    return d;
}

// Warp 0 lane 0 streams the stages by TMA through a UV_STAGES ring that runs
// across segments; warp 1 lane 0 issues the MMAs into one of two accumulator
// sets (segments alternate, so a segment's epilogue overlaps the next
// segment's MMAs); warps 4-7 drain a set (one output column per thread).
DZ_KERNEL_LINKAGE __global__ void __launch_bounds__(UG_THREADS, 1)
    dz_ugemv_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmL, UvArgs a) {
    // the next kernel (the next call's limb split) may launch now; it waits
    // for this grid before touching memory
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    extern __shared__ __align__(1024) uint8_t uv_raw[];
    const uint32_t raw = dz_smem_addr(uv_raw);
    uint8_t* sm = uv_raw + ((1024u - (raw & 1023u)) & 1023u);
    uint64_t* full = reinterpret_cast<uint64_t*>(sm + (size_t)UV_STAGES * UV_STAGE_BYTES);
    uint64_t* empty = full + UV_STAGES;
    uint64_t* tfull = empty + UV_STAGES;      // [2] accumulator set ready
    uint64_t* tempty = tfull + 2;             // [2] accumulator set drained (4 epilogue warps arrive)
    int* row_e = reinterpret_cast<int*>(tempty + 2);   // [UV_N] -s or UG_ROW_NONFINITE
    int* pend_kb = row_e + UV_N;                        // [UV_STAGES] k block of a stage whose limbs wait
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(pend_kb + UV_STAGES);
    int* flags = reinterpret_cast<int*>(tmem_slot + 1);   // [0] stages issued, [1] consumed, [2] failed, [3] last
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int G = gridDim.x;
    const long long s0 = uv_range_start(a.total, blockIdx.x, G), s1 = uv_range_start(a.total, blockIdx.x + 1, G);
    auto stage_a = [&](int s) { return sm + (size_t)s * UV_STAGE_BYTES; };
    auto stage_b = [&](int s, int limb) { return sm + (size_t)s * UV_STAGE_BYTES + UV_A_BYTES + (size_t)limb * UV_B_PITCH; };

    if (threadIdx.x == 0) {
        for (int s = 0; s < UV_STAGES; s++) {
            dz_mbar_init(&full[s]);
            dz_mbar_init(&empty[s]);
        }
        for (int b = 0; b < 2; b++) {
            dz_mbar_init(&tfull[b]);
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 4;" ::"r"(dz_smem_addr(&tempty[b])) : "memory");
        }
        flags[0] = flags[1] = flags[2] = flags[3] = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dz_smem_addr(tmem_slot)),
                     "r"(UV_TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    ug_fence_before();
    __syncthreads();
    ug_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            // the weights are read once per product: they should not push
            // the activations and other reused data out of L2
            const uint64_t wpol = dz_policy_evict_first();
            int i = 0;   // stage counter over the range
            bool stop = false, limbs_ready = false;
            auto load_limbs = [&](int s, int kb) {
                for (int limb = 0; limb < UG_LIMBS; limb++)
                    ug_tma_3d(stage_b(s, limb), &tmL, kb * UG_BK, 0, limb, &full[s]);
            };
            auto release_pending = [&]() {   // the split grid is done: its limbs can be read
                asm volatile("griddepcontrol.wait;" ::: "memory");
                for (int q = 0; q < i && q < UV_STAGES; q++) load_limbs(q, pend_kb[q]);
                limbs_ready = true;
            };
            for (long long pos = s0; pos < s1 && !stop;) {
                const UvSeg g = uv_segment(pos, s1, a.nkb);
                for (int j = 0; j < g.nk; j++, i++) {
                    const int s = i % UV_STAGES;
                    if (i >= UV_STAGES) {
                        if (!limbs_ready) release_pending();
                        if (!dz_mbar_wait(&empty[s], (uint32_t)(((i / UV_STAGES) - 1) & 1))) {
                            flags[2] = 1;
                            stop = true;
                            break;
                        }
                    }
                    const int kb = g.kb0 + j;
                    dz_mbar_expect_tx(&full[s], UV_A_BYTES + UG_LIMBS * UV_B_BYTES);
                    ug_tma_4d_hint(stage_a(s), &tmW, 0, 0, kb, g.tile, &full[s], wpol);
                    if (limbs_ready) load_limbs(s, kb);
                    else pend_kb[s] = kb;
                }
                pos += g.nk;
            }
            if (!limbs_ready) release_pending();
            flags[0] = i;
        }
        __syncwarp();
    } else if (warp == 1) {
        if (lane == 0) {
            const uint32_t idesc = uv_idesc();
            int i = 0, t = 0;   // stage counter, segment counter
            bool stop = false;
            for (long long pos = s0; pos < s1 && !stop; t++) {
                const UvSeg g = uv_segment(pos, s1, a.nkb);
                pos += g.nk;
                const int buf = t & 1;
                // the accumulator set of segment t-2 has been drained
                if (t >= 2 && !dz_mbar_wait(&tempty[buf], (uint32_t)(((t >> 1) - 1) & 1))) {
                    flags[2] = 1;
                    break;
                }
                ug_fence_after();
                const uint32_t acc = tmem + (uint32_t)(buf * UV_ACC_COLS);
                for (int j = 0; j < g.nk; j++, i++) {
                    const int s = i % UV_STAGES;
                    if (!dz_mbar_wait(&full[s], (uint32_t)((i / UV_STAGES) & 1))) {
                        flags[2] = 1;
                        stop = true;
                        break;
                    }
                    ug_fence_after();
                    // one MMA per 32 k covers the three limbs: B is the
                    // stage's 48 limb rows (limb-major, 16 rows each)
                    const uint32_t a_addr = dz_smem_addr(stage_a(s)), b_addr = dz_smem_addr(stage_b(s, 0));
#pragma unroll
                    for (int kk = 0; kk < UG_BK / 32; kk++) {
                        const uint64_t ad = ug_desc_kmajor(a_addr + kk * 32);
                        const uint64_t bd = ug_desc_kmajor(b_addr + kk * 32);
                        ug_mma(acc, ad, bd, idesc, (j > 0 || kk > 0) ? 1u : 0u);
                    }
                    ug_commit(&empty[s]);
                }
                ug_commit(&tfull[buf]);   // this segment's accumulator set is complete
            }
            flags[1] = i;
        }
        __syncwarp();
    } else if (warp == 2) {
        // row exponents: written by the split grid, read after it completed
        asm volatile("griddepcontrol.wait;" ::: "memory");
        if (lane < UV_N) row_e[lane] = lane < a.M ? a.shift[lane] : 0;
        __syncwarp();
        asm volatile("bar.arrive 2, 160;" ::: "memory");
    } else if (warp >= 4) {
        // thread = output column n0 + nl: 16 rows x 3 limbs -> int64
        asm volatile("bar.sync 2, 160;" ::: "memory");   // row exponents are in place
        const int ew = warp - 4;
        const int nl = ew * 32 + lane;
        const uint32_t lane_base = (uint32_t)(ew * 32) << 16;
        int t = 0;
        for (long long pos = s0; pos < s1; t++) {
            const bool first = pos == s0;
            const UvSeg g = uv_segment(pos, s1, a.nkb);
            pos += g.nk;
            const int buf = t & 1;
            bool ok = dz_mbar_wait(&tfull[buf], (uint32_t)((t >> 1) & 1));
            ug_fence_after();
            if (!ok || flags[2]) {
                ok = false;
                flags[2] = 1;
                if (a.status && lane == 0) atomicExch(a.status, 1);
            }
            const uint32_t acc = tmem + lane_base + (uint32_t)(buf * UV_ACC_COLS);
            int32_t top[UV_N], mid[UV_N], low[UV_N];
            ug_tmem_ld16(acc, top);
            ug_tmem_ld16(acc + UV_N, mid);
            ug_tmem_ld16(acc + 2 * UV_N, low);
            ug_fence_before();
            __syncwarp();
            if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(dz_smem_addr(&tempty[buf])) : "memory");
            long long v[UV_N];
#pragma unroll
            for (int r = 0; r < UV_N; r++) v[r] = (long long)top[r] * 65536 + (long long)mid[r] * 256 + (long long)low[r];
            bool finish = true;
            if (g.nk < a.nkb) {   // a piece of a tile shared with neighbouring ranges
                long long* mine = a.partial + ((size_t)blockIdx.x * 2 + (first ? 0 : 1)) * UV_SLOT_ELEMS + (size_t)nl * UV_N;
#pragma unroll
                for (int r = 0; r < UV_N; r++) __stcg(mine + r, v[r]);
                // one release by one thread after the barrier covers the
                // group's stores; its acquire covers the reads below
                dz_named_sync(1, 128);
                if (threadIdx.x == 128) {
                    int prev;
                    asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], %2;"
                                 : "=r"(prev)
                                 : "l"(a.counter + g.tile), "r"(g.nk)
                                 : "memory");
                    flags[3] = prev + g.nk == a.nkb ? 1 : 0;
                    if (flags[3]) a.counter[g.tile] = 0;   // ready for the next launch
                }
                dz_named_sync(1, 128);
                finish = flags[3] != 0;
                dz_named_sync(1, 128);   // everyone read flags[3] before the next piece rewrites it
                if (finish) {
                    const long long t0 = (long long)g.tile * a.nkb;
                    const int c0 = uv_owner(a.total, t0, G), c1 = uv_owner(a.total, t0 + a.nkb - 1, G);
                    for (int c = c0; c <= c1; c++) {
                        if (c == (int)blockIdx.x) continue;
                        const int slot = uv_range_start(a.total, c, G) >= t0 ? 0 : 1;
                        const long long* pp = a.partial + ((size_t)c * 2 + slot) * UV_SLOT_ELEMS + (size_t)nl * UV_N;
                        long long q[UV_N];
#pragma unroll
                        for (int r = 0; r < UV_N; r++) q[r] = __ldcg(pp + r);
#pragma unroll
                        for (int r = 0; r < UV_N; r++) v[r] += q[r];
                    }
                }
            }
            if (finish) {
                float y[UV_N];
#pragma unroll
                for (int r = 0; r < UV_N; r++) {
                    const int e = row_e[r];
                    y[r] = dz_mul_pow2(__ll2float_rn(v[r]), e);
                    if (!ok || e == UG_ROW_NONFINITE) y[r] = __int_as_float(0x7fc00000);
                }
                dz_qmv_store_col<UV_N>(a.ep, a.M, a.N, g.tile * UG_BN + nl, y);
            }
        }
    }

    ug_fence_before();
    __syncthreads();
    if (threadIdx.x == 0 && flags[2]) {
        // copies in flight land before the shared memory goes away
        for (int i = flags[1]; i < flags[0]; i++)
            if (!dz_mbar_wait(&full[i % UV_STAGES], (uint32_t)((i / UV_STAGES) & 1))) break;
    }
    __syncthreads();
    if (warp == 1) {
        ug_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(UV_TMEM_COLS) : "memory");
    }
}

}  // namespace dz
