// The decode matvec (M <= 2 activation rows) with the codes as they are: the
// weights stream from HBM in the MMA-fragment layout of qmma.cuh (bulk-copied
// shared-memory stages, one 16-byte load per lane per chunk), are widened to
// bytes in registers with one logic op per word (no dequantization), and
// meet the activation limbs in the 8-bit integer MMA (m16n8k32, u8 codes x
// s8 limbs, int32 accumulate): two MMAs per INT4 chunk and one per INT8
// chunk, half and a quarter of the fp16 kernel's per-chunk MMA count.
//
// Integer formulation (the same as the tensor-core GEMM of umma.cuh):
// - each activation row is scaled by 2^s (exact) so that max |x 2^s| lies in
//   [2^21, 2^22), rounded to an integer X and cut into three balanced
//   base-256 digits X = 65536 * top + 256 * mid + low (signed bytes);
// - codes enter as the reference's biased values c = level + qmax
//   (src/core/quantize.c:213-221): sum_k c X = sum_k level X + qmax sum_k X,
//   and qmax sum_k X is subtracted once per column;
// - the int32 sums are exact (|sum| <= K * 254 * 128 < 2^31 for INT8, and
//   16 * K * 14 * 128 < 2^31 for INT4, K <= 65536); the three limb sums
//   combine in int64, convert to fp32 once, and 2^-s and the column scale
//   are applied after.
//
// Operand mapping. In the fragment layout lane l = 4g + t holds, per 16-row
// k-tile, columns g and g + 8 at k in {2t, 2t+1, 2t+8, 2t+9}. INT4:
// (w & 0x0F0F0F0F) is column g and (w & 0xF0F0F0F0) is 16x column g + 8,
// bytes in the k order (2t, 2t+8, 2t+1, 2t+9); INT8: the two words of a
// k-tile give column g with one byte permute (0x5140) and column g + 8 with
// another (0x7362), in the same order. Those four words are exactly the A
// fragment of m16n8k32 (rows = output columns) for two k-tiles, with the
// MMA's k indices 4t..4t+3 standing for that lane's four k; the MMA sums over
// k, so any permutation shared with B is the same sum. B column j is limb
// j % 3 of row j / 3 (columns 3M..7 zero); the limb table holds, per pair of
// k-tiles and lane, the B fragment words in the same k order.
#pragma once
#include <cstdint>
#include <cstring>
#include <cuda_runtime.h>

#include "umma.cuh"

namespace dz {

constexpr int QMV1I_WARPS = 16;

struct Qmv1iArgs {
    const uint8_t* codes;     // fragment layout
    int N, nkg, ntiles;
    const float* X;
    long long ldx;
    const float* k_scale;
    int K;
    int M;                    // rows, <= the kernel's MR
    int pk;                   // chunks per piece
    int max_tiles;            // n-tiles per CTA at most
    int max_parts;            // warps sharing one n-tile at most
    unsigned tab_bytes;       // limb table bytes in shared memory
    int* status;              // set to 1 when a copy wait gave up (may be null)
    QmvEpilogue ep;           // row shifts are applied by the kernel
};

// Largest K for which the int32 limb sums of biased codes are exact.
constexpr int QI_MAX_K = 65536;

// The B-fragment table: per pair of k-tiles, 32 lanes x two words.
__host__ __device__ constexpr unsigned dz_qmv1i_tab_bytes(int nkg, int KT) {
    return (unsigned)nkg * KT / 2 * 256;
}

__host__ __device__ constexpr size_t dz_qmv1i_smem_bytes(int pk, int W, unsigned tab_bytes, int max_tiles,
                                                         int max_parts) {
    return (size_t)W * QMS_STAGES * pk * 512 + tab_bytes + (size_t)max_tiles * max_parts * 32 * 8 +
           (size_t)((max_tiles + 3) & ~3) * 4 + (size_t)W * QMS_STAGES * 8 + 16 * 4 + 2 * 8 + 32 * 4 + 32 * 4 +
           32 * 8;
}

// D += A (16 x 32, u8 codes, row) . B (32 x 8, s8 limbs, col), int32.
__device__ __forceinline__ void dz_imma(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                        uint2 b) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b.x), "r"(b.y));
}

// Limbs of row r of M into the B-fragment table: for k-tile kt and t, the
// limb words of k = 16 kt + (2t, 2t+8, 2t+1, 2t+9) (zero past K) go to lanes
// g = 3r + limb, word kt & 1 of pair kt / 2; the last row also zeroes lanes
// g >= 3M. Sets rsh[r] (-s, or UG_ROW_NONFINITE) and sumx[r] = sum_k X.
__device__ __forceinline__ void dz_qmv1i_split_row(const float* __restrict__ x, const float* __restrict__ k_scale,
                                                   int K, int nkt, int r, int M, uint32_t* __restrict__ tab,
                                                   int* __restrict__ rsh, long long* __restrict__ sumx, float* wred,
                                                   int* wbad, long long* wsum) {
    float m = 0.0f;
    int bad = 0;
#pragma unroll 4
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
    __syncthreads();   // wred / wsum may still be read for the previous row
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
    long long sx = 0;
    for (int e = threadIdx.x; e < nkt * 4; e += blockDim.x) {
        const int k0 = (e >> 2) * 16 + 2 * (e & 3);
        const int ks[4] = {k0, k0 + 8, k0 + 1, k0 + 9};
        uint32_t l4 = 0, m4 = 0, t4 = 0;
#pragma unroll
        for (int b = 0; b < 4; b++) {
            int X = 0;
            if (ks[b] < K) {
                float v = x[ks[b]];
                if (k_scale) v *= k_scale[ks[b]];
                X = ug_fixed(v, s);
            }
            sx += X;
            uint32_t dt, dm, dl;
            ug_digits(X, dt, dm, dl);
            l4 |= dl << (8 * b);
            m4 |= dm << (8 * b);
            t4 |= dt << (8 * b);
        }
        const int kt = e >> 2, t = e & 3;
        uint32_t* base = tab + (size_t)(kt >> 1) * 64 + t * 2 + (kt & 1);
        base[(3 * r + 0) * 8] = l4;
        base[(3 * r + 1) * 8] = m4;
        base[(3 * r + 2) * 8] = t4;
        if (r == M - 1)
            for (int g = 3 * M; g < 8; g++) base[g * 8] = 0u;
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) sx += __shfl_xor_sync(0xffffffffu, sx, off);
    if ((threadIdx.x & 31) == 0) wsum[threadIdx.x >> 5] = sx;
    __syncthreads();
    if (threadIdx.x == 0) {
        long long tot = 0;
        for (int w = 0; w < (int)(blockDim.x >> 5); w++) tot += wsum[w];
        sumx[r] = tot;
        rsh[r] = bad ? UG_ROW_NONFINITE : -s;
    }
}

// Y = epilogue(X . deq(W)) for M <= MR rows (MR = 1 or 2), the streaming and
// stream-K structure of dz_qmv1_kernel (qmma.cuh): CTA c takes whole n-tiles,
// its W warps split their chunks into W equal contiguous ranges, each warp
// streams its range through its own QMS_STAGES-deep ring of bulk copies; an
// n-tile shared by several warps is summed in shared memory (exact int64
// parts, so the result does not depend on the split) by the last warp to
// arrive.
template <int BITS, int W, int MR>
__global__ void __launch_bounds__(W * 32, 1) dz_qmv1i_kernel(Qmv1iArgs a) {
    constexpr int KT = FragGeom<BITS>::KT;
    constexpr int QMAX = BITS == 8 ? 127 : 7;
    extern __shared__ __align__(128) unsigned char qmv1i_smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, t = lane & 3;
    const int stage_bytes = a.pk * 512;
    uint8_t* ring = qmv1i_smem + (size_t)warp * QMS_STAGES * stage_bytes;
    uint32_t* tab = reinterpret_cast<uint32_t*>(qmv1i_smem + (size_t)W * QMS_STAGES * stage_bytes);
    long long* slots = reinterpret_cast<long long*>(reinterpret_cast<uint8_t*>(tab) + a.tab_bytes);
    int* cnt = reinterpret_cast<int*>(slots + (size_t)a.max_tiles * a.max_parts * 32);
    uint64_t* bars = reinterpret_cast<uint64_t*>(cnt + ((a.max_tiles + 3) & ~3)) + warp * QMS_STAGES;
    int* rsh = reinterpret_cast<int*>(reinterpret_cast<uint64_t*>(cnt + ((a.max_tiles + 3) & ~3)) + W * QMS_STAGES);
    long long* sumx = reinterpret_cast<long long*>(rsh + 16);
    float* wred = reinterpret_cast<float*>(sumx + 2);
    int* wbad = reinterpret_cast<int*>(wred + 32);
    long long* wsum = reinterpret_cast<long long*>(wbad + 32);

    const int G = gridDim.x;
    const int t0 = (int)((long long)blockIdx.x * a.ntiles / G), t1 = (int)(((long long)blockIdx.x + 1) * a.ntiles / G);
    const int C0 = t0 * a.nkg, L = (t1 - t0) * a.nkg;
    auto wstart = [&](int w) { return C0 + (int)((long long)w * L / W); };
    const int my0 = wstart(warp), my1 = wstart(warp + 1);
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

    // programmatic dependent launch: weight copies (constant for the launch)
    // go out before griddepcontrol.wait; activations are read and every
    // global write made after it
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
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
    if (lane == 0)
        for (int i = 0; i < QMS_STAGES - 1 && ic.pos < my1; i++) issue();
    asm volatile("griddepcontrol.wait;" ::: "memory");

    const int nkt = a.nkg * KT;
    for (int r = 0; r < a.M; r++)
        dz_qmv1i_split_row(a.X + (long long)r * a.ldx, a.k_scale, a.K, nkt, r, a.M, tab, rsh, sumx, wred, wbad,
                           wsum);
    __syncthreads();   // counters zeroed, limb table, shifts and sums written

    auto owner_of = [&](int x) {
        int w = (int)(((long long)(x - C0) * W) / (L > 0 ? L : 1));
        if (w > W - 1) w = W - 1;
        while (w < W - 1 && wstart(w + 1) <= x) w++;
        while (w > 0 && wstart(w) > x) w--;
        return w;
    };
    // the column value of an int64 total: bias correction, one rounding, 2^-s
    auto finish = [&](long long tot, int r) {
        const int e = rsh[r];
        if (e == UG_ROW_NONFINITE) return __int_as_float(0x7fc00000);
        return dz_mul_pow2(__ll2float_rn(tot - (long long)QMAX * sumx[r]), e);
    };

    bool failed = false;
    int failed_at = -1;
    Cursor cc = cursor_at(my0);
    int consumed = 0, cstage = 0;
    uint32_t cphase = 0;
    // two accumulator chains (alternate k-tile pairs)
    int acc[2][4];
#pragma unroll
    for (int c = 0; c < 2; c++)
#pragma unroll
        for (int q = 0; q < 4; q++) acc[c][q] = 0;
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
            // B fragments of this lane: one uint2 per pair of k-tiles
            const uint2* tb = reinterpret_cast<const uint2*>(tab) + (size_t)kg0 * (KT / 2) * 32 + lane;
#pragma unroll 2
            for (int c = 0; c < n; c++, tb += (KT / 2) * 32) {
                const uint4 w = w4[c * 32];
                if (BITS == 4) {
                    dz_imma(acc[0], w.x & 0x0F0F0F0Fu, w.x & 0xF0F0F0F0u, w.y & 0x0F0F0F0Fu, w.y & 0xF0F0F0F0u,
                            tb[0]);
                    dz_imma(acc[1], w.z & 0x0F0F0F0Fu, w.z & 0xF0F0F0F0u, w.w & 0x0F0F0F0Fu, w.w & 0xF0F0F0F0u,
                            tb[32]);
                } else {
                    const uint32_t a0 = __byte_perm(w.x, w.y, 0x5140), a1 = __byte_perm(w.x, w.y, 0x7362);
                    const uint32_t a2 = __byte_perm(w.z, w.w, 0x5140), a3 = __byte_perm(w.z, w.w, 0x7362);
                    if (c & 1) dz_imma(acc[1], a0, a1, a2, a3, tb[0]);
                    else dz_imma(acc[0], a0, a1, a2, a3, tb[0]);
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

        // this warp's share of the n-tile. Lane (g, t) holds B columns 2t and
        // 2t + 1 of output columns g (d0, d1) and g + 8 (d2, d3; 16x for
        // INT4); B column j is limb j % 3 of row j / 3. Gather them, combine
        // the limbs in int64 (exact).
        int d[4];
#pragma unroll
        for (int q = 0; q < 4; q++) {
            d[q] = acc[0][q] + acc[1][q];
            acc[0][q] = acc[1][q] = 0;
        }
        if (BITS == 4) {
            d[2] >>= 4;   // exact: every term was 16x
            d[3] >>= 4;
        }
        int bc[2][6];
#pragma unroll
        for (int q = 0; q < 3; q++)
#pragma unroll
            for (int h = 0; h < 2; h++) {
                const int src = (lane & ~3) | q;
                bc[h][2 * q] = __shfl_sync(0xffffffffu, d[2 * h], src);
                bc[h][2 * q + 1] = __shfl_sync(0xffffffffu, d[2 * h + 1], src);
            }
        long long tot[MR][2];
#pragma unroll
        for (int r = 0; r < MR; r++)
#pragma unroll
            for (int h = 0; h < 2; h++)
                tot[r][h] = (long long)bc[h][3 * r] + 256LL * (long long)bc[h][3 * r + 1] +
                            65536LL * (long long)bc[h][3 * r + 2];
        const int n0 = tile * 16 + g;
        const bool whole = my0 <= tile_start && my1 >= tile_end;
        if (whole) {
            if (t == 0) {
#pragma unroll
                for (int r = 0; r < MR; r++) {
                    if (r >= a.M) continue;
                    const float v0 = failed ? __int_as_float(0x7fc00000) : finish(tot[r][0], r);
                    const float v1 = failed ? __int_as_float(0x7fc00000) : finish(tot[r][1], r);
                    dz_qmv_store_row(a.ep, a.M, a.N, r, n0, v0);
                    dz_qmv_store_row(a.ep, a.M, a.N, r, n0 + 8, v1);
                }
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
        long long* mine = slots + ((size_t)lt * a.max_parts + part) * 32;
        if (t == 0) {
#pragma unroll
            for (int r = 0; r < MR; r++) {
                mine[r * 16 + g] = tot[r][0];
                mine[r * 16 + g + 8] = tot[r][1];
            }
        }
        __syncwarp();
        // the counter's low 16 bits count arrivals, the high bits failed parts
        int last = 0;
        if (lane == 0) {
            __threadfence_block();
            const int old = atomicAdd(&cnt[lt], (failed ? 1 << 16 : 0) + 1);
            const bool is_last = (old & 0xFFFF) == nparts - 1;
            const bool bad = failed || (old >> 16) != 0;
            last = is_last ? (bad ? 2 : 1) : 0;
        }
        last = __shfl_sync(0xffffffffu, last, 0);
        if (last) {
            __threadfence_block();
            const bool any_failed = last == 2;
            if (t == 0) {
#pragma unroll
                for (int r = 0; r < MR; r++) {
                    if (r >= a.M) continue;
                    long long s0 = 0, s1 = 0;
                    for (int pp = 0; pp < nparts; pp++) {
                        const long long* sl = slots + ((size_t)lt * a.max_parts + pp) * 32;
                        s0 += sl[r * 16 + g];
                        s1 += sl[r * 16 + g + 8];
                    }
                    const float v0 = any_failed ? __int_as_float(0x7fc00000) : finish(s0, r);
                    const float v1 = any_failed ? __int_as_float(0x7fc00000) : finish(s1, r);
                    dz_qmv_store_row(a.ep, a.M, a.N, r, n0, v0);
                    dz_qmv_store_row(a.ep, a.M, a.N, r, n0 + 8, v1);
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

// Host side (qmvi.cu): the dynamic shared-memory limit of every
// instantiation, and one launch of the instantiation for (bits, a.M).
cudaError_t dz_qmv1i_set_smem(int bytes);
cudaError_t dz_qmv1i_launch(const Qmv1iArgs& a, int bits, int grid, size_t smem, cudaStream_t st);

}  // namespace dz
