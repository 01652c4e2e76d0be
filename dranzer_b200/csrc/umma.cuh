// Quantized GEMM on the 5th-generation tensor cores (tcgen05 / UMMA) for
// many activation rows (batched prefill and large-batch decode):
//   C[m, n] = epilogue(scale[n] * sum_k x[m, k] * level[k, n]).
//
// Integer formulation, exact in every product and sum:
// - each activation row is scaled by 2^s (exact) so that max |x 2^s| lies in
//   [2^22, 2^23), rounded to a 24-bit integer X and cut into three 8-bit
//   limbs X = 65536 * top + 256 * mid + low (top signed, mid / low unsigned);
// - weights enter the tensor core as their unsigned codes c = level + qmax
//   (INT8: the reference's k x n bytes as stored, src/core/quantize.c:
//   213-221; INT4: the nibbles widened to bytes once at upload), so there is
//   no dequantization at all: sum_k X level = sum_k X c - qmax * sum_k X;
// - one kind::i8 MMA per limb accumulates int32 in tensor memory (exact for
//   K up to 33k); the epilogue combines the limbs in int64, subtracts the
//   code bias times the row sum, converts to fp32 once and applies 2^-s and
//   the column scale.
// Rounding differs from the reference's fp32 multiply-add only in the
// activation's 24-bit fixed-point representation (relative to the row's
// largest element) and the final conversions.
//
// Tiles: 128 rows x 128 columns per CTA, k in steps of 128 bytes. A (the
// limbs) is K-major and B (the codes) MN-major, both loaded by TMA with the
// 128-byte swizzle; a 3-stage ring of 64 KB stages. Warp 0 issues the TMA
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
constexpr size_t UG_SMEM_BYTES = (size_t)UG_STAGES * UG_STAGE_BYTES + 1024 + 256;
constexpr int UG_ROW_NONFINITE = -0x40000000;    // row exponent marking a non-finite input row
constexpr int UG_TILE_LD = UG_BN + 4;            // staging tile row stride (floats): 16-byte rows, spread banks

struct UgArgs {
    int M, N, K, nkb;             // nkb: k blocks of UG_BK
    const long long* rowsum;      // [M] sum_k X
    const int* shift;             // [M] -s, or UG_ROW_NONFINITE
    int code_bias;                // qmax: 127 (INT8) or 7 (INT4)
    int* status;                  // set to 1 when a wait gave up (may be null)
    QmvEpilogue ep;               // col_scale etc.; row_shift unused
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

// MN-major operand, 128-byte swizzle: 128 consecutive n per 128-byte row, one
// row per k; 8-row groups 1024 bytes apart along k (stride byte offset);
// 128-column atoms `lbo` bytes apart along n (a single atom here).
__device__ __forceinline__ uint64_t ug_desc_mnmajor(uint32_t saddr, uint32_t lbo) {
    uint64_t d = (uint64_t)((saddr >> 4) & 0x3FFFu);
    d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
    d |= (uint64_t)(1024u >> 4) << 32;
    d |= (uint64_t)1u << 46;
    d |= (uint64_t)2u << 61;
    return d;
}

// Instruction descriptor for kind::i8, int32 accumulate, A K-major (s8 or
// u8), B MN-major u8, M = UG_BM, N = UG_BN.
__device__ __forceinline__ uint32_t ug_idesc(bool a_signed) {
    uint32_t d = 2u << 4;                   // D format S32
    d |= (a_signed ? 1u : 0u) << 7;         // A: 1 = s8, 0 = u8
    d |= 0u << 10;                          // B: u8
    d |= 1u << 16;                          // B MN-major
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

__device__ __forceinline__ void ug_tma_2d(void* dst, const CUtensorMap* tm, int c0, int c1, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            dz_smem_addr(dst)),
        "l"(reinterpret_cast<uint64_t>(tm)), "r"(c0), "r"(c1), "r"(dz_smem_addr(bar))
        : "memory");
}

__device__ __forceinline__ void ug_tma_3d(void* dst, const CUtensorMap* tm, int c0, int c1, int c2, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(
            dz_smem_addr(dst)),
        "l"(reinterpret_cast<uint64_t>(tm)), "r"(c0), "r"(c1), "r"(c2), "r"(dz_smem_addr(bar))
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
__global__ void dz_widen_nibbles_kernel(const uint8_t* __restrict__ packed, long long cols, long long total,
                                        uint8_t* __restrict__ out, int ld) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= total) return;
    const long long k = i / cols, n = i - k * cols;
    out[k * ld + n] = (packed[i >> 1] >> ((i & 1) * 4)) & 0xF;
}

// ------------------------------------------------------- activation limbs

// One block per row: X = rint(x * k_scale * 2^s) clamped to 24 bits, stored
// as three limb planes L[limb][M][Kp] (zero past K), the row sum of X and -s.
__global__ void __launch_bounds__(256) dz_limb_split_kernel(const float* __restrict__ X, long long ldx,
                                                            const float* __restrict__ k_scale, int M, int K, int Kp,
                                                            int8_t* __restrict__ L, long long* __restrict__ rowsum,
                                                            int* __restrict__ shift) {
    __shared__ float wred[8];
    __shared__ long long wsum[8];
    __shared__ int wbad[8];
    const int r = blockIdx.x;
    const float* x = X + (long long)r * ldx;
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
    const int s = amax > 0.0f ? 22 - ilogbf(amax) : 0;
    long long sum = 0;
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
                if (fabsf(v) <= 3.402823466e38f) {
                    const float f = rintf(dz_mul_pow2(v, s));
                    xi = f >= 8388607.0f ? 8388607 : f <= -8388608.0f ? -8388608 : (int)f;
                }
            }
            sum += xi;
            t4 |= ((uint32_t)(xi >> 16) & 0xFFu) << (8 * j);
            m4 |= ((uint32_t)(xi >> 8) & 0xFFu) << (8 * j);
            l4 |= ((uint32_t)xi & 0xFFu) << (8 * j);
        }
        const size_t at = (size_t)r * Kp + k0;
        *reinterpret_cast<uint32_t*>(L + at) = t4;
        *reinterpret_cast<uint32_t*>(L + plane + at) = m4;
        *reinterpret_cast<uint32_t*>(L + 2 * plane + at) = l4;
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
    if ((threadIdx.x & 31) == 0) wsum[threadIdx.x >> 5] = sum;
    __syncthreads();
    if (threadIdx.x == 0) {
        long long t = 0;
        for (int w = 0; w < (int)(blockDim.x >> 5); w++) t += wsum[w];
        rowsum[r] = t;
        shift[r] = bad ? UG_ROW_NONFINITE : -s;
    }
}

// Columns [n0, n0 + UG_BN) of rows [m0, m0 + UG_BM) from the staging tile
// through the epilogue (column scale, bias, residual, ReLU, segment routing),
// four columns per thread with float4 accesses where the addresses allow.
__device__ __forceinline__ void ug_store_tile(const UgArgs& a, const float* tile, int m0, int n0, bool failed) {
    const QmvEpilogue& e = a.ep;
    const int c4 = (threadIdx.x & 31) * 4;   // fixed per thread: blockDim.x is a multiple of 32
    const int n = n0 + c4;
    if (n >= a.N) return;
    const int nv = a.N - n < 4 ? a.N - n : 4;
    float sc[4], bi[4];
#pragma unroll
    for (int j = 0; j < 4; j++) {
        sc[j] = (j < nv && e.col_scale) ? e.col_scale[n + j] : 1.0f;
        bi[j] = (j < nv && e.bias) ? e.bias[n + j] : 0.0f;
    }
    int sg = 0;
    while (sg + 1 < e.nseg && n >= e.seg_start[sg + 1]) sg++;
    const bool one_seg = nv == 4 && (sg + 1 >= e.nseg || n + 3 < e.seg_start[sg + 1]);
    for (int r = threadIdx.x >> 5; r < UG_BM; r += UG_THREADS / 32) {
        const int row = m0 + r;
        if (row >= a.M) break;
        float4 t = *reinterpret_cast<const float4*>(tile + r * UG_TILE_LD + c4);
        if (failed) t.x = t.y = t.z = t.w = __int_as_float(0x7fc00000);   // a failed tile reads NaN
        float y[4] = {t.x, t.y, t.z, t.w};
#pragma unroll
        for (int j = 0; j < 4; j++) {
            y[j] = (e.col_scale ? y[j] * sc[j] : y[j]);
            if (e.bias) y[j] = y[j] + bi[j];
        }
        if (e.residual) {
            const float* rp = e.residual + (long long)row * e.ld_res + n;
#pragma unroll
            for (int j = 0; j < 4; j++)
                if (j < nv) y[j] = y[j] + rp[j];
        }
        if (e.relu) {
#pragma unroll
            for (int j = 0; j < 4; j++) y[j] = y[j] > 0.0f ? y[j] : 0.0f;
        }
        if (one_seg) {
            long long off = (long long)row * e.seg_ld[sg] + (n - e.seg_start[sg]);
            if (e.seg_row_off[sg]) off += e.seg_row_off[sg][row];
            float* dst = e.seg_ptr[sg] + off;
            if ((reinterpret_cast<uintptr_t>(dst) & 15) == 0) {
                *reinterpret_cast<float4*>(dst) = make_float4(y[0], y[1], y[2], y[3]);
                continue;
            }
#pragma unroll
            for (int j = 0; j < 4; j++) dst[j] = y[j];
            continue;
        }
        for (int j = 0; j < nv; j++) {
            int s2 = 0;
            while (s2 + 1 < e.nseg && n + j >= e.seg_start[s2 + 1]) s2++;
            long long off = (long long)row * e.seg_ld[s2] + (n + j - e.seg_start[s2]);
            if (e.seg_row_off[s2]) off += e.seg_row_off[s2][row];
            e.seg_ptr[s2][off] = y[j];
        }
    }
}

// ------------------------------------------------------------------- GEMM

__global__ void __launch_bounds__(UG_THREADS, 1)
    dz_ugemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, UgArgs a) {
    extern __shared__ __align__(1024) uint8_t ug_raw[];
    const uint32_t raw = dz_smem_addr(ug_raw);
    uint8_t* sm = ug_raw + ((1024u - (raw & 1023u)) & 1023u);
    uint64_t* full = reinterpret_cast<uint64_t*>(sm + (size_t)UG_STAGES * UG_STAGE_BYTES);
    uint64_t* empty = full + UG_STAGES;
    uint64_t* accum = empty + UG_STAGES;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accum + 1);
    int* progress = reinterpret_cast<int*>(tmem_slot + 1);   // [0] stages issued, [1] stages consumed, [2] failed
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n0 = blockIdx.x * UG_BN, m0 = blockIdx.y * UG_BM;
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
        int kb = 0;
        for (; kb < a.nkb; kb++) {
            const int s = kb % UG_STAGES;
            if (kb >= UG_STAGES && !dz_mbar_wait(&empty[s], (uint32_t)(((kb / UG_STAGES) - 1) & 1))) {
                progress[2] = 1;
                break;
            }
            dz_mbar_expect_tx(&full[s], UG_STAGE_BYTES);
            for (int limb = 0; limb < UG_LIMBS; limb++) ug_tma_3d(stage_a(s, limb), &tmA, kb * UG_BK, m0, limb, &full[s]);
            ug_tma_2d(stage_b(s), &tmB, n0, kb * UG_BK, &full[s]);
        }
        progress[0] = kb;
      }
      __syncwarp();   // the warp reconverges before the block barriers below
    } else if (warp == 1) {
      if (lane == 0) {
        // MMA issuer: 3 limbs x 4 k-steps of 32 per stage
        int kb = 0;
        const uint32_t id_top = ug_idesc(true), id_low = ug_idesc(false);
        for (; kb < a.nkb; kb++) {
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
                    const uint64_t bd = ug_desc_mnmajor(b_addr + kk * 32 * UG_BN, UG_B_BYTES);
                    ug_mma(tmem + (uint32_t)(limb * UG_BN), ad, bd, limb == 0 ? id_top : id_low,
                           (kb > 0 || kk > 0) ? 1u : 0u);
                }
            }
            ug_commit(&empty[s]);
        }
        progress[1] = kb;
        ug_commit(accum);   // completes once every MMA issued above has
      }
      __syncwarp();
    } else if (warp >= 4) {
        // epilogue, part 1: thread = row; drain the three accumulators into a
        // [128][UG_TILE_LD] fp32 staging tile in the pipeline buffers (free
        // once the accumulator barrier completes)
        const int ew = warp - 4;
        bool ok = dz_mbar_wait(accum, 0);
        ug_fence_after();
        const int rl = ew * 32 + lane;
        const int row = m0 + rl;
        const uint32_t lane_base = (uint32_t)(ew * 32) << 16;
        const bool live = row < a.M;
        const long long bias = live ? (long long)a.code_bias * a.rowsum[row] : 0;
        const int e = live ? a.shift[row] : 0;
        if (!ok || progress[2]) {
            if (a.status && lane == 0) atomicExch(a.status, 1);
            ok = false;
            progress[2] = 1;
        }
        float* tile = reinterpret_cast<float*>(sm);
        for (int c0 = 0; c0 < UG_BN; c0 += 32) {
            int32_t top[32], mid[32], low[32];
            ug_tmem_ld32(tmem + lane_base + (uint32_t)c0, top);
            ug_tmem_ld32(tmem + lane_base + (uint32_t)(UG_BN + c0), mid);
            ug_tmem_ld32(tmem + lane_base + (uint32_t)(2 * UG_BN + c0), low);
#pragma unroll
            for (int q = 0; q < 8; q++) {
                float y[4];
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    const int c = 4 * q + j;
                    const long long v = (long long)top[c] * 65536 + (long long)mid[c] * 256 + (long long)low[c] - bias;
                    y[j] = dz_mul_pow2(__ll2float_rn(v), e);
                    if (!ok || e == UG_ROW_NONFINITE) y[j] = __int_as_float(0x7fc00000);
                }
                *reinterpret_cast<float4*>(tile + rl * UG_TILE_LD + c0 + 4 * q) = make_float4(y[0], y[1], y[2], y[3]);
            }
        }
    }

    ug_fence_before();
    __syncthreads();
    // epilogue, part 2, all warps: one warp per output row, lane = 4 columns,
    // so each store instruction writes 512 contiguous bytes
    ug_store_tile(a, reinterpret_cast<const float*>(sm), m0, n0, progress[2] != 0);

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

}  // namespace dz
