// Batched-prefill causal attention on the tensor cores (attention_head_forward,
// src/core/transformer.c:73-190, causal form): for one (64 queries, head,
// sequence), S = Q K^T / sqrtf(hd) over the prompt's keys j <= t, softmax,
// O = P V.
//
// Both products run as mma.sync m16n8k8 TF32 with fp32 accumulation in the
// three-term split that keeps fp32 accuracy: each fp32 operand x is cut into
// hi = tf32(x) and lo = tf32(x - hi) (round to nearest, 11 significant bits
// each), and a.b is accumulated as hi(a) hi(b) + hi(a) lo(b) + lo(a) hi(b);
// the dropped lo(a) lo(b) term is below 2^-22 of the product. The softmax
// runs online per query row over key tiles of 32 (running max and sum,
// rescaled) with expf, as the CUDA-core kernel does; so the result differs
// from the reference's two-pass fp32 form within fp32 noise.
//
// Block: 4 warps, 16 queries each. K and V tiles of 32 rows are
// double-buffered with cp.async; the scores' fragments come straight from
// shared memory rows (padded stride: conflict-free), and P goes through a
// per-warp shared-memory tile to change from the accumulator layout to the
// A-operand layout.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace dz {

constexpr int PT_QT = 64;            // queries per block
constexpr int PT_KT = 32;            // keys per tile
constexpr int PT_THREADS = 128;      // 4 warps x 16 queries
constexpr int PT_PLD = PT_KT + 4;    // per-warp P tile row stride (floats)

__host__ __device__ constexpr size_t dz_pfattn_smem(int hd) {
    return ((size_t)PT_QT * (hd + 4) + 4 * (size_t)PT_KT * (hd + 4) + 4 * 16 * (size_t)PT_PLD) * sizeof(float);
}

static __device__ __forceinline__ void pt_cp16(void* dst, const void* src, bool valid) {
    const uint32_t d = (uint32_t)__cvta_generic_to_shared(dst);
    const int n = valid ? 16 : 0;   // zero-fill rows past the last key or query
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(d), "l"(src), "r"(n) : "memory");
}
static __device__ __forceinline__ void pt_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
static __device__ __forceinline__ void pt_wait1() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }
static __device__ __forceinline__ void pt_wait0() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

// x -> (hi, lo) tf32 bit patterns
static __device__ __forceinline__ void pt_split(float x, uint32_t& hi, uint32_t& lo) {
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(hi) : "f"(x));
    const float r = __fsub_rn(x, __uint_as_float(hi));
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(lo) : "f"(r));
}

static __device__ __forceinline__ void pt_mma(float* d, const uint32_t* a, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// An A fragment (4 fp32 values, split once into ah / al) times a B fragment
// (2 fp32 values), three-term split
static __device__ __forceinline__ void pt_split4(const float* a, uint32_t* ah, uint32_t* al) {
#pragma unroll
    for (int i = 0; i < 4; i++) pt_split(a[i], ah[i], al[i]);
}
static __device__ __forceinline__ void pt_mma3(float* d, const uint32_t* ah, const uint32_t* al, float b0f,
                                               float b1f) {
    uint32_t bh0, bl0, bh1, bl1;
    pt_split(b0f, bh0, bl0);
    pt_split(b1f, bh1, bl1);
    pt_mma(d, al, bh0, bh1);
    pt_mma(d, ah, bl0, bl1);
    pt_mma(d, ah, bh0, bh1);
}

template <int HDW>   // head_dim / 32: 2 or 4
__global__ void __launch_bounds__(PT_THREADS, 2) dz_pfattn_kernel(
    const float* __restrict__ q, const float* __restrict__ keys, const float* __restrict__ values,
    const int* __restrict__ lens, float* __restrict__ out, int T, int dim, int capacity) {
    constexpr int HD = HDW * 32;
    constexpr int LD = HD + 4;               // Q / K / V tile row stride (floats)
    constexpr int CH = HD / 4;               // 16-byte chunks per row
    constexpr int NT_S = PT_KT / 8;          // score n-tiles per key tile
    constexpr int NT_O = HD / 8;             // output n-tiles
    extern __shared__ __align__(16) float pt_smem[];
    float* qs = pt_smem;                     // [PT_QT][LD]
    float* kb = qs + PT_QT * LD;             // [2][PT_KT][LD]
    float* vb = kb + 2 * PT_KT * LD;         // [2][PT_KT][LD]
    float* pw = vb + 2 * PT_KT * LD;         // [4 warps][16][PT_PLD]
    // heavy (late) query blocks first
    const int q0 = (gridDim.x - 1 - blockIdx.x) * PT_QT, h = blockIdx.y, s = blockIdx.z;
    const int len = lens ? lens[s] : T;
    if (q0 >= len) return;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int g = lane >> 2, t4 = lane & 3;
    const float* K = keys + (long long)s * capacity * dim + h * HD;
    const float* V = values + (long long)s * capacity * dim + h * HD;
    const long long row0 = (long long)s * T;
    const int tq_last = min(q0 + PT_QT, len) - 1;
    auto load_tile = [&](int j0, int buf) {
        for (int i = tid; i < PT_KT * CH; i += PT_THREADS) {
            const int kj = i / CH, c = i - kj * CH;
            const int j = j0 + kj;
            const bool in = j <= tq_last;
            const int jj = in ? j : 0;
            pt_cp16(kb + (buf * PT_KT + kj) * LD + 4 * c, K + (long long)jj * dim + 4 * c, in);
            pt_cp16(vb + (buf * PT_KT + kj) * LD + 4 * c, V + (long long)jj * dim + 4 * c, in);
        }
        pt_commit();
    };
    for (int i = tid; i < PT_QT * CH; i += PT_THREADS) {
        const int qi = i / CH, c = i - qi * CH;
        const int t = q0 + qi;
        pt_cp16(qs + qi * LD + 4 * c, q + (row0 + (t < len ? t : 0)) * dim + h * HD + 4 * c, t < len);
    }
    load_tile(0, 0);   // one group: Q and the first tile

    const float denom = sqrtf((float)HD);
    const int r0 = q0 + warp * 16 + g, r1 = r0 + 8;   // this thread's two query rows
    const float* qw = qs + (warp * 16) * LD;
    float* pwarp = pw + warp * 16 * PT_PLD;
    float o[NT_O][4];
#pragma unroll
    for (int n = 0; n < NT_O; n++) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.0f;
    float m0 = -3.402823466e38f, m1 = -3.402823466e38f, l0 = 0.0f, l1 = 0.0f;
    int buf = 0;
    for (int j0 = 0; j0 <= tq_last; j0 += PT_KT, buf ^= 1) {
        if (j0 + PT_KT <= tq_last) {
            load_tile(j0 + PT_KT, buf ^ 1);
            pt_wait1();
        } else {
            pt_wait0();
        }
        __syncthreads();   // tile `buf` (and Q) landed for every thread
        const float* ks = kb + buf * PT_KT * LD;
        const float* vs = vb + buf * PT_KT * LD;
        // S = Q K^T for this warp's 16 queries x 32 keys
        float sc[NT_S][4];
#pragma unroll
        for (int n = 0; n < NT_S; n++) sc[n][0] = sc[n][1] = sc[n][2] = sc[n][3] = 0.0f;
        if (j0 <= q0 + warp * 16 + 15) {   // a warp whose queries all precede the tile skips it
#pragma unroll 4
            for (int k0 = 0; k0 < HD; k0 += 8) {
                const float a[4] = {qw[g * LD + k0 + t4], qw[(g + 8) * LD + k0 + t4], qw[g * LD + k0 + t4 + 4],
                                    qw[(g + 8) * LD + k0 + t4 + 4]};
                uint32_t ah[4], al[4];
                pt_split4(a, ah, al);
#pragma unroll
                for (int n = 0; n < NT_S; n++) {
                    const float* kr = ks + (n * 8 + g) * LD + k0 + t4;
                    pt_mma3(sc[n], ah, al, kr[0], kr[4]);
                }
            }
        }
        // online softmax over the tile: this thread holds rows r0 (c0, c1) and
        // r1 (c2, c3) at key columns j0 + 8n + 2 t4 + {0, 1}
        float tmax0 = m0, tmax1 = m1;
#pragma unroll
        for (int n = 0; n < NT_S; n++) {
#pragma unroll
            for (int e = 0; e < 2; e++) {
                const int j = j0 + n * 8 + 2 * t4 + e;
                sc[n][e] = sc[n][e] / denom;
                sc[n][2 + e] = sc[n][2 + e] / denom;
                if (j <= r0 && r0 < len) tmax0 = fmaxf(tmax0, sc[n][e]);
                if (j <= r1 && r1 < len) tmax1 = fmaxf(tmax1, sc[n][2 + e]);
            }
        }
#pragma unroll
        for (int off = 1; off <= 2; off <<= 1) {
            tmax0 = fmaxf(tmax0, __shfl_xor_sync(0xffffffffu, tmax0, off));
            tmax1 = fmaxf(tmax1, __shfl_xor_sync(0xffffffffu, tmax1, off));
        }
        const float c0 = expf(m0 - tmax0), c1 = expf(m1 - tmax1);
        m0 = tmax0;
        m1 = tmax1;
        float ps0 = 0.0f, ps1 = 0.0f;
#pragma unroll
        for (int n = 0; n < NT_S; n++) {
            float p[4];
#pragma unroll
            for (int e = 0; e < 2; e++) {
                const int j = j0 + n * 8 + 2 * t4 + e;
                p[e] = (j <= r0 && r0 < len) ? expf(sc[n][e] - m0) : 0.0f;
                p[2 + e] = (j <= r1 && r1 < len) ? expf(sc[n][2 + e] - m1) : 0.0f;
            }
            ps0 += p[0] + p[1];
            ps1 += p[2] + p[3];
            *reinterpret_cast<float2*>(pwarp + g * PT_PLD + n * 8 + 2 * t4) = make_float2(p[0], p[1]);
            *reinterpret_cast<float2*>(pwarp + (g + 8) * PT_PLD + n * 8 + 2 * t4) = make_float2(p[2], p[3]);
        }
#pragma unroll
        for (int off = 1; off <= 2; off <<= 1) {
            ps0 += __shfl_xor_sync(0xffffffffu, ps0, off);
            ps1 += __shfl_xor_sync(0xffffffffu, ps1, off);
        }
        l0 = l0 * c0 + ps0;
        l1 = l1 * c1 + ps1;
#pragma unroll
        for (int n = 0; n < NT_O; n++) {
            o[n][0] *= c0;
            o[n][1] *= c0;
            o[n][2] *= c1;
            o[n][3] *= c1;
        }
        __syncwarp();   // this warp's P tile written
        // O += P V over the tile's 32 keys (nothing to add for a warp whose
        // queries all precede the tile)
#pragma unroll
        for (int k0 = 0; k0 < PT_KT && j0 <= q0 + warp * 16 + 15; k0 += 8) {
            const float a[4] = {pwarp[g * PT_PLD + k0 + t4], pwarp[(g + 8) * PT_PLD + k0 + t4],
                                pwarp[g * PT_PLD + k0 + t4 + 4], pwarp[(g + 8) * PT_PLD + k0 + t4 + 4]};
            uint32_t ah[4], al[4];
            pt_split4(a, ah, al);
#pragma unroll
            for (int n = 0; n < NT_O; n++) {
                const float* vr = vs + (k0 + t4) * LD + n * 8 + g;
                pt_mma3(o[n], ah, al, vr[0], vr[4 * LD]);
            }
        }
        __syncthreads();   // tile `buf` and the P tiles consumed before they are rewritten
    }
    const float inv0 = 1.0f / l0, inv1 = 1.0f / l1;
#pragma unroll
    for (int n = 0; n < NT_O; n++) {
        const int col = h * HD + n * 8 + 2 * t4;
        if (r0 < len)
            *reinterpret_cast<float2*>(out + (row0 + r0) * dim + col) = make_float2(o[n][0] * inv0, o[n][1] * inv0);
        if (r1 < len)
            *reinterpret_cast<float2*>(out + (row0 + r1) * dim + col) = make_float2(o[n][2] * inv1, o[n][3] * inv1);
    }
}

// Host side (pfattn.cu): shared-memory limits once per device; the launch for
// head dimension 64 or 128 (cudaErrorNotSupported otherwise).
cudaError_t dz_pfattn_set_smem();
cudaError_t dz_pfattn_launch(const float* q, const float* keys, const float* values, const int* lens, float* out,
                             int T, int dim, int capacity, int head_dim, int heads, int seqs, cudaStream_t st);

}  // namespace dz
