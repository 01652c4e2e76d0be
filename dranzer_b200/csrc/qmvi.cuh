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

// The B-fragment table: per pair of k-tiles, 32 lanes x two words, pairs
// QI_PAIR_WORDS apart. The 8 words of padding put the four pairs that one
// warp's stores meet (8 k-tiles) on different banks when the table is built.
constexpr int QI_PAIR_WORDS = 72;
__host__ __device__ constexpr unsigned dz_qmv1i_tab_bytes(int nkg, int KT) {
    return (unsigned)nkg * KT / 2 * QI_PAIR_WORDS * 4;
}

// Shared memory: rings, table, tile slots and counters, barriers, row
// shifts and sums, reduction scratch, a copy of the epilogue's parameters,
// then its column scales, biases and M rows of residuals for the CTA's
// columns (max_tiles * 16 each) and the output segments' row offsets
// (3 segments x 2 rows).
__host__ __device__ constexpr size_t dz_qmv1i_smem_bytes(int pk, int W, unsigned tab_bytes, int max_tiles,
                                                         int max_parts, int M) {
    return (size_t)W * QMS_STAGES * pk * 512 + tab_bytes + (size_t)max_tiles * max_parts * 32 * 8 +
           (size_t)((max_tiles + 3) & ~3) * 4 + (size_t)W * QMS_STAGES * 8 + 16 * 4 + 2 * 8 + 32 * 4 + 32 * 4 +
           32 * 8 + sizeof(QmvEpilogue) + (size_t)(2 + M) * max_tiles * 16 * 4 + 6 * 4;
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

// The activation split of the matvec, in two halves around the issue of the
// weight ring's remaining copies.
//
// Entry e of a row covers k = k0, k0 + 8, k0 + 1, k0 + 9 with
// k0 = 16 (e / 4) + 2 (e % 4): k-tile kt = e / 4 and t = e % 4 of the
// B-fragment table. Thread i keeps entries i + j blockDim.x (j < QI_CE) of
// every row in registers: the loads all go out at once, before the ring's
// remaining copies, so that they do not wait in the memory queues behind
// the weight stream, and both passes (row maximum, then digits) read the
// registers. Entries past the cache (K above 4 QI_CE blockDim.x) are read
// again in each pass.
constexpr int QI_CE = 4;

template <int MR>
struct QiSplitRegs {
    float v[MR][QI_CE][4];
};

__device__ __forceinline__ float dz_qmv1i_x(const Qmv1iArgs& a, int r, int k) {
    float v = a.X[(long long)r * a.ldx + k];
    if (a.k_scale) v *= a.k_scale[k];
    return v;
}

// First half: the loads of the cached entries (zero past K and past M).
template <int MR>
__device__ __forceinline__ void dz_qmv1i_split_load(const Qmv1iArgs& a, int nent, QiSplitRegs<MR>& R) {
#pragma unroll
    for (int r = 0; r < MR; r++)
#pragma unroll
        for (int j = 0; j < QI_CE; j++) {
            const int e = threadIdx.x + j * blockDim.x;
            const int k0 = (e >> 2) * 16 + 2 * (e & 3);
#pragma unroll
            for (int b = 0; b < 4; b++) {
                const int k = k0 + 8 * (b & 1) + (b >> 1);
                R.v[r][j][b] = (r < a.M && e < nent && k < a.K) ? dz_qmv1i_x(a, r, k) : 0.0f;
            }
        }
}

// Second half: per row the largest magnitude (block-wide), the shift s with
// max |x 2^s| in [2^21, 2^22), the digits X = 65536 top + 256 mid + low of
// every k into the table (lanes g = 3r + limb, word kt & 1 of pair kt / 2;
// lanes g >= 3M zero), rsh[r] (-s, or UG_ROW_NONFINITE) and
// sumx[r] = sum_k X. Ends with the table, rsh and sumx written (block
// barrier).
template <int MR, int W>
__device__ __forceinline__ void dz_qmv1i_split_finish(const Qmv1iArgs& a, int nent, const QiSplitRegs<MR>& R,
                                                      uint32_t* __restrict__ tab, int* __restrict__ rsh,
                                                      long long* __restrict__ sumx, float* wred, int* wbad,
                                                      long long* wsum) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float m[MR];
    int bad[MR];
#pragma unroll
    for (int r = 0; r < MR; r++) {
        m[r] = 0.0f;
        bad[r] = 0;
#pragma unroll
        for (int j = 0; j < QI_CE; j++)
#pragma unroll
            for (int b = 0; b < 4; b++) {
                const float v = R.v[r][j][b];
                if (!(fabsf(v) <= 3.402823466e38f)) bad[r] = 1;
                else m[r] = fmaxf(m[r], fabsf(v));
            }
    }
    for (int e = threadIdx.x + QI_CE * blockDim.x; e < nent; e += blockDim.x) {
        const int k0 = (e >> 2) * 16 + 2 * (e & 3);
#pragma unroll
        for (int r = 0; r < MR; r++)
#pragma unroll
            for (int b = 0; b < 4; b++) {
                const int k = k0 + 8 * (b & 1) + (b >> 1);
                if (r >= a.M || k >= a.K) continue;
                const float v = dz_qmv1i_x(a, r, k);
                if (!(fabsf(v) <= 3.402823466e38f)) bad[r] = 1;
                else m[r] = fmaxf(m[r], fabsf(v));
            }
    }
#pragma unroll
    for (int r = 0; r < MR; r++) {
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) {
            m[r] = fmaxf(m[r], __shfl_xor_sync(0xffffffffu, m[r], off));
            bad[r] |= __shfl_xor_sync(0xffffffffu, bad[r], off);
        }
        if (lane == 0) {
            wred[r * W + warp] = m[r];
            wbad[r * W + warp] = bad[r];
        }
    }
    __syncthreads();
    int sh[MR];
#pragma unroll
    for (int r = 0; r < MR; r++) {
        float amax = 0.0f;
        for (int w = 0; w < W; w++) {
            amax = fmaxf(amax, wred[r * W + w]);
            bad[r] |= wbad[r * W + w];
        }
        sh[r] = amax > 0.0f ? (UG_X_BITS - 1) - dz_ilogb(amax) : 0;
    }
    long long sx[MR];
#pragma unroll
    for (int r = 0; r < MR; r++) sx[r] = 0;
    // digits of one entry of every row, and the zero lanes. X = rint(x 2^s)
    // needs no clamp (|x 2^s| < 2^22 by the choice of s) and a non-finite x
    // gives 0, as ug_fixed. With Y = X + 0x8080 the balanced base-256 digits
    // of ug_digits are (byte 0 of Y) - 128, (byte 1 of Y) - 128 and Y >> 16,
    // so the limbs of four k are byte permutes of the four Y.
    auto put = [&](int e, const float (&v)[MR][4]) {
        const int kt = e >> 2, t = e & 3;
        uint32_t* base = tab + (size_t)(kt >> 1) * QI_PAIR_WORDS + t * 2 + (kt & 1);
#pragma unroll
        for (int r = 0; r < MR; r++) {
            if (r >= a.M) break;
            uint32_t Y[4];
            int xs = 0;
#pragma unroll
            for (int b = 0; b < 4; b++) {
                const float f = v[r][b];
                const int X = fabsf(f) <= 3.402823466e38f ? __float2int_rn(dz_mul_pow2(f, sh[r])) : 0;
                xs += X;
                Y[b] = (uint32_t)(X + 0x8080);
            }
            sx[r] += xs;
            const uint32_t l4 = __byte_perm(__byte_perm(Y[0], Y[1], 0x0040), __byte_perm(Y[2], Y[3], 0x0040), 0x5410) ^
                                0x80808080u;
            const uint32_t m4 = __byte_perm(__byte_perm(Y[0], Y[1], 0x0051), __byte_perm(Y[2], Y[3], 0x0051), 0x5410) ^
                                0x80808080u;
            const uint32_t t4 = __byte_perm(__byte_perm(Y[0], Y[1], 0x0062), __byte_perm(Y[2], Y[3], 0x0062), 0x5410);
            base[(3 * r + 0) * 8] = l4;
            base[(3 * r + 1) * 8] = m4;
            base[(3 * r + 2) * 8] = t4;
        }
        for (int g = 3 * a.M; g < 8; g++) base[g * 8] = 0u;
    };
#pragma unroll
    for (int j = 0; j < QI_CE; j++) {
        const int e = threadIdx.x + j * blockDim.x;
        if (e >= nent) break;
        float v[MR][4];
#pragma unroll
        for (int r = 0; r < MR; r++)
#pragma unroll
            for (int b = 0; b < 4; b++) v[r][b] = R.v[r][j][b];
        put(e, v);
    }
    for (int e = threadIdx.x + QI_CE * blockDim.x; e < nent; e += blockDim.x) {
        const int k0 = (e >> 2) * 16 + 2 * (e & 3);
        float v[MR][4];
#pragma unroll
        for (int r = 0; r < MR; r++)
#pragma unroll
            for (int b = 0; b < 4; b++) {
                const int k = k0 + 8 * (b & 1) + (b >> 1);
                v[r][b] = (r < a.M && k < a.K) ? dz_qmv1i_x(a, r, k) : 0.0f;
            }
        put(e, v);
    }
#pragma unroll
    for (int r = 0; r < MR; r++) {
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) sx[r] += __shfl_xor_sync(0xffffffffu, sx[r], off);
        if (lane == 0) wsum[r * W + warp] = sx[r];
    }
    __syncthreads();
#pragma unroll
    for (int r = 0; r < MR; r++) {   // thread r, constant indices into bad / sh
        if ((int)threadIdx.x != r || r >= a.M) continue;
        long long tot = 0;
        for (int w = 0; w < W; w++) tot += wsum[r * W + w];
        sumx[r] = tot;
        rsh[r] = bad[r] ? UG_ROW_NONFINITE : -sh[r];
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
    // 32-bit: the host keeps max_tiles * nkg * W below 2^31
    auto wstart = [&](int w) { return C0 + (w * L) / W; };
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
    // one piece per warp goes out before the wait; the activation loads go
    // out right after it, ahead of the ring's other copies (a load queued
    // behind the whole ring would wait for it to drain), and the ring fills
    // while the limb table is built
    if (lane == 0 && ic.pos < my1) issue();
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const int nent = a.nkg * KT * 4;
    QiSplitRegs<MR> xr;
    dz_qmv1i_split_load<MR>(a, nent, xr);
    // the epilogue's per-column inputs of this CTA's columns and the output
    // segments' row offsets, loaded with the activations: the tile
    // epilogues then read only shared memory, and the stores are the last
    // global accesses of a warp
    const int ncols = (t1 - t0) * 16, EC = a.max_tiles * 16;
    QmvEpilogue* s_ep = reinterpret_cast<QmvEpilogue*>(wsum + 32);   // the epilogue's parameters
    float* e_cs = reinterpret_cast<float*>(s_ep + 1);
    float* e_bi = e_cs + EC;
    float* e_res = e_bi + EC;                                   // [MR][EC]
    int* e_roff = reinterpret_cast<int*>(e_res + MR * EC);      // [3 segments][2 rows]
    auto epi_load = [&](int c, float& cs, float& bi, float (&res)[MR]) {
        const int n = t0 * 16 + c;
        const bool ok = c < ncols && n < a.N;
        cs = (ok && a.ep.col_scale) ? a.ep.col_scale[n] : 0.0f;
        bi = (ok && a.ep.bias) ? a.ep.bias[n] : 0.0f;
#pragma unroll
        for (int r = 0; r < MR; r++)
            res[r] = (ok && a.ep.residual && r < a.M) ? a.ep.residual[(long long)r * a.ep.ld_res + n] : 0.0f;
    };
    float ecs, ebi, eres[MR];
    epi_load(threadIdx.x, ecs, ebi, eres);
    int eroff = 0;
    if (threadIdx.x < 6) {
        const int si = threadIdx.x >> 1, r = threadIdx.x & 1;
        const int* ro = si == 0 ? a.ep.seg_row_off[0] : si == 1 ? a.ep.seg_row_off[1] : a.ep.seg_row_off[2];
        if (si < a.ep.nseg && ro && r < a.M) eroff = ro[r];
    }
    if (lane == 0)
        for (int i = 1; i < QMS_STAGES && ic.pos < my1; i++) issue();
    dz_qmv1i_split_finish<MR, W>(a, nent, xr, tab, rsh, sumx, wred, wbad, wsum);
    for (int c = threadIdx.x; c < ncols; c += blockDim.x) {
        if (c >= (int)blockDim.x) epi_load(c, ecs, ebi, eres);
        e_cs[c] = ecs;
        e_bi[c] = ebi;
#pragma unroll
        for (int r = 0; r < MR; r++) e_res[r * EC + c] = eres[r];
    }
    if (threadIdx.x < 6) e_roff[threadIdx.x] = eroff;
    if (threadIdx.x == 0) *s_ep = a.ep;
    __syncthreads();   // counters zeroed, limb table, shifts, sums and epilogue inputs written
    // the fused epilogue of one output value (dz_qmv_store_row's arithmetic)
    // (parameters from the shared copy: the first tile end comes when the
    // memory system is busiest, and a constant-cache miss then waits long)
    auto store = [&](int r, int n, float v) {
        if (r >= a.M || n >= a.N) return;
        const QmvEpilogue& ep = *s_ep;
        const int c = n - t0 * 16;
        float y = ep.col_scale ? v * e_cs[c] : v;
        if (ep.bias) y = y + e_bi[c];
        if (ep.residual) y = y + e_res[r * EC + c];
        if (ep.act) y = dz_act(y, ep.act);
        const int si = (ep.nseg > 1 && n >= ep.seg_start[1]) + (ep.nseg > 2 && n >= ep.seg_start[2]);
        const DzSeg sg = dz_seg_of(ep, n);
        long long off = (long long)r * sg.ld + (n - sg.start);
        if (sg.row_off) off += e_roff[si * 2 + r];
        sg.ptr[off] = y;
    };

    auto owner_of = [&](int x) {
        int w = ((x - C0) * W) / (L > 0 ? L : 1);
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
            const uint2* tb = reinterpret_cast<const uint2*>(tab) + (size_t)kg0 * (KT / 2) * (QI_PAIR_WORDS / 2) + lane;
#pragma unroll 2
            for (int c = 0; c < n; c++, tb += (KT / 2) * (QI_PAIR_WORDS / 2)) {
                const uint4 w = w4[c * 32];
                if (BITS == 4) {
                    dz_imma(acc[0], w.x & 0x0F0F0F0Fu, w.x & 0xF0F0F0F0u, w.y & 0x0F0F0F0Fu, w.y & 0xF0F0F0F0u,
                            tb[0]);
                    dz_imma(acc[1], w.z & 0x0F0F0F0Fu, w.z & 0xF0F0F0F0u, w.w & 0x0F0F0F0Fu, w.w & 0xF0F0F0F0u,
                            tb[QI_PAIR_WORDS / 2]);
                } else {
                    const uint32_t a0 = __byte_perm(w.x, w.y, 0x5140), a1 = __byte_perm(w.x, w.y, 0x7362);
                    const uint32_t a2 = __byte_perm(w.z, w.w, 0x5140), a3 = __byte_perm(w.z, w.w, 0x7362);
                    if (c & 1) dz_imma(acc[1], a0, a1, a2, a3, tb[0]);
                    else dz_imma(acc[0], a0, a1, a2, a3, tb[0]);
                }
            }
        }
        __syncwarp();   // the stage is free: lane 0 refills it with the next piece
        if (!failed && lane == 0 && ic.pos < my1) issue();
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
                    store(r, n0, v0);
                    store(r, n0 + 8, v1);
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
                    store(r, n0, v0);
                    store(r, n0 + 8, v1);
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
