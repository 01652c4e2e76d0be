// The decode matvec (M <= 2 activation rows) on CUDA cores with integer dot
// products: the weights stream from HBM in the MMA-fragment layout of
// qmma.cuh (16-byte loads per lane out of bulk-copied shared-memory stages),
// the codes are unpacked in registers and multiplied against the activation
// limbs with dp4a, and the partial sums of a column meet through warp
// shuffles. No tensor-core instruction is issued per chunk, so the loop is
// bound by the weight stream, not by MMA issue.
//
// Integer formulation (the same as the tensor-core GEMM of umma.cuh):
// - each activation row is scaled by 2^s (exact) so that max |x 2^s| lies in
//   [2^21, 2^22), rounded to an integer X and cut into three balanced
//   base-256 digits X = 65536 * top + 256 * mid + low (signed bytes);
// - codes enter as the reference's biased bytes c = level + qmax
//   (src/core/quantize.c:213-221): sum_k c X = sum_k level X + qmax sum_k X,
//   and qmax sum_k X is subtracted once per column;
// - dp4a.u32.s32 of four codes (unsigned) and four limb bytes (signed) adds
//   exactly into int32 (|sum| <= K * 254 * 128 < 2^31 for K <= 65536); the
//   three limb sums combine in int64, convert to fp32 once, and 2^-s and the
//   column scale are applied after.
//
// Which four k a lane's codes cover: in the fragment layout lane l = 4g + t
// holds, per 16-row k-tile, columns g and g + 8 at k in {2t, 2t+1, 2t+8,
// 2t+9}. INT4: (w & 0x0F0F0F0F) is column g and ((w >> 4) & 0x0F0F0F0F)
// column g + 8, bytes in the k order (2t, 2t+8, 2t+1, 2t+9). INT8: the two
// words of a k-tile give column g with one byte permute (0x5140) and column
// g + 8 with another (0x7362), in the same k order. The limb table in shared
// memory stores, per (k-tile, t, row), the three limb words in that order.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

#include "umma.cuh"

namespace dz {

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

__host__ __device__ constexpr unsigned dz_qmv1i_tab_bytes(int nkg, int KT, int MR) {
    return (unsigned)nkg * KT * 4 * MR * 16;
}

__host__ __device__ constexpr size_t dz_qmv1i_smem_bytes(int pk, int W, unsigned tab_bytes, int max_tiles,
                                                         int max_parts) {
    return (size_t)W * QMS_STAGES * pk * 512 + tab_bytes + (size_t)max_tiles * max_parts * 32 * 8 +
           (size_t)((max_tiles + 3) & ~3) * 4 + (size_t)W * QMS_STAGES * 8 + 16 * 4 + 2 * 8 + 32 * 4 + 32 * 4 +
           32 * 8;
}

__device__ __forceinline__ int dz_dp4a_us(uint32_t codes, uint32_t limbs, int acc) {
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(codes), "r"(limbs), "r"(acc));
    return d;
}

// Limbs of row r into the table: entry (kt, t) holds the limb words of
// k = 16 kt + (2t, 2t+8, 2t+1, 2t+9) (zero past K); sets rsh[r] (-s, or
// UG_ROW_NONFINITE) and sumx[r] = sum_k X.
template <int MR>
__device__ __forceinline__ void dz_qmv1i_split_row(const float* __restrict__ x, const float* __restrict__ k_scale,
                                                   int K, int nkt, int r, uint4* __restrict__ tab,
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
    const int s = amax > 0.0f ? (UG_X_BITS - 1) - ilogbf(amax) : 0;
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
        tab[e * MR + r] = make_uint4(l4, m4, t4, 0u);
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
    uint4* tab = reinterpret_cast<uint4*>(qmv1i_smem + (size_t)W * QMS_STAGES * stage_bytes);
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
        dz_qmv1i_split_row<MR>(a.X + (long long)r * a.ldx, a.k_scale, a.K, nkt, r, tab, rsh, sumx, wred, wbad,
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
    int acc[MR][2][3];
#pragma unroll
    for (int r = 0; r < MR; r++)
#pragma unroll
        for (int c = 0; c < 2; c++)
#pragma unroll
            for (int l = 0; l < 3; l++) acc[r][c][l] = 0;
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
            const uint4* tk = tab + ((size_t)kg0 * KT * 4 + t) * MR;
#pragma unroll 2
            for (int c = 0; c < n; c++, tk += KT * 4 * MR) {
                const uint4 w = w4[c * 32];
                const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
                for (int j = 0; j < KT; j++) {
                    uint32_t c0, c1;
                    if (BITS == 4) {
                        c0 = ww[j] & 0x0F0F0F0Fu;
                        c1 = (ww[j] >> 4) & 0x0F0F0F0Fu;
                    } else {
                        c0 = __byte_perm(ww[2 * j], ww[2 * j + 1], 0x5140);
                        c1 = __byte_perm(ww[2 * j], ww[2 * j + 1], 0x7362);
                    }
#pragma unroll
                    for (int r = 0; r < MR; r++) {
                        const uint4 lb = tk[j * 4 * MR + r];
                        acc[r][0][0] = dz_dp4a_us(c0, lb.x, acc[r][0][0]);
                        acc[r][0][1] = dz_dp4a_us(c0, lb.y, acc[r][0][1]);
                        acc[r][0][2] = dz_dp4a_us(c0, lb.z, acc[r][0][2]);
                        acc[r][1][0] = dz_dp4a_us(c1, lb.x, acc[r][1][0]);
                        acc[r][1][1] = dz_dp4a_us(c1, lb.y, acc[r][1][1]);
                        acc[r][1][2] = dz_dp4a_us(c1, lb.z, acc[r][1][2]);
                    }
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

        // this warp's share of the n-tile: limb sums over the four t lanes,
        // combined in int64 (exact)
        long long tot[MR][2];
#pragma unroll
        for (int r = 0; r < MR; r++)
#pragma unroll
            for (int c = 0; c < 2; c++) {
                int s[3];
#pragma unroll
                for (int l = 0; l < 3; l++) {
                    int v = acc[r][c][l];
                    v += __shfl_xor_sync(0xffffffffu, v, 1);
                    v += __shfl_xor_sync(0xffffffffu, v, 2);
                    s[l] = v;
                    acc[r][c][l] = 0;
                }
                tot[r][c] = (long long)s[0] + 256LL * (long long)s[1] + 65536LL * (long long)s[2];
            }
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

}  // namespace dz
