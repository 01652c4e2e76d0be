// Decode-step attention over the fp32 KV ring, streamed through shared memory
// by the bulk-copy engine (attention_head_forward_token,
// src/core/transformer.c:686-713): for one (head, sequence), score_j =
// (q . k_j) / sqrtf(hd) over the logical context j = 0..ctx-1 at physical
// slot (start + j) % capacity, softmax, o = sum_j p_j v_j.
//
// The step reads every context row of K and V once (the KV ring is the
// step's dominant HBM traffic), so the kernel is built to keep many bytes in
// flight: per block, tiles of 32 keys (the head's 32 K rows and 32 V rows,
// hd * 4 bytes each) land in a ring of shared-memory stages, each tile by two
// 2-D tensor copies (one for K, one for V: a box of hd floats x 32 ring
// rows, completion counted on the stage's mbarrier; a tile that wraps round
// the ring goes as one bulk copy per row instead); 8 consumer warps take 4
// keys each per tile. The softmax runs online per warp (running max and sum, rescaled) and
// the warps' partial results merge at the end, so its rounding differs from
// the reference's two-pass form within fp32 noise. Waits are bounded (about
// one second, %globaltimer); on a timeout the block records status 1, waits
// for its copies in flight and returns.
#pragma once
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

namespace dz {

constexpr int AD_THREADS = 256;
constexpr int AD_WARPS = AD_THREADS / 32;
constexpr int AD_KT = 32;                   // keys per tile
constexpr int AD_KPW = AD_KT / AD_WARPS;    // keys per warp per tile

template <int HDW>   // head_dim / 32: 2 or 4
struct AdCfg {
    static constexpr int HD = HDW * 32;
    static constexpr int ROW = HD * 4;                      // bytes of one K or V row of the head
    static constexpr int STAGE = 2 * AD_KT * ROW;           // K tile then V tile
    static constexpr int STAGES = HDW == 4 ? 3 : 5;         // 96 KB / 80 KB: two blocks per SM
    static constexpr int SMEM = STAGES * STAGE + 64;        // + the stage barriers
};

struct AdArgs {
    const float* q;        // [B][dim]
    const float* keys;     // [B][capacity][dim], this layer
    const float* values;
    const int* start;      // [B] ring state after the step's begin
    const int* ctx;
    float* out;            // [B][dim]
    int dim, capacity;
    int* status;
    int layer_row0;        // this layer's first row in the tensor maps' [rows][dim] view
};

static __device__ __forceinline__ uint32_t ad_smem_addr(const void* p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}
static __device__ __forceinline__ uint64_t ad_now_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
static __device__ __forceinline__ bool ad_mbar_test(uint64_t* bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(ad_smem_addr(bar)), "r"(parity)
        : "memory");
    return done != 0;
}
// false after about one second without the phase completing
static __device__ __forceinline__ bool ad_mbar_wait(uint64_t* bar, uint32_t parity) {
#pragma unroll 1
    for (int i = 0; i < 8; i++)
        if (ad_mbar_test(bar, parity)) return true;
    const uint64_t t0 = ad_now_ns();
    for (unsigned i = 0;; i++) {
        if (ad_mbar_test(bar, parity)) return true;
        if ((i & 255u) == 255u && ad_now_ns() - t0 > 1000000000ull) return false;
    }
}

static __device__ __forceinline__ void ad_tma_2d(void* dst, const CUtensorMap* tm, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            ad_smem_addr(dst)),
        "l"(reinterpret_cast<uint64_t>(tm)), "r"(x), "r"(y), "r"(ad_smem_addr(bar))
        : "memory");
}

// tmK / tmV: every layer's K (V) ring as one [layers * B * capacity][dim]
// fp32 tensor, box {hd, 32}.
template <int HDW>
__global__ void __launch_bounds__(AD_THREADS, 2) dz_attn_decode_kernel(const __grid_constant__ CUtensorMap tmK,
                                                                       const __grid_constant__ CUtensorMap tmV,
                                                                       AdArgs a) {
    using C = AdCfg<HDW>;
    extern __shared__ __align__(128) uint8_t ad_smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(ad_smem + C::STAGES * C::STAGE);
    const int h = blockIdx.x, b = blockIdx.y;
    const int ctx = a.ctx[b], start = a.start[b];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int ntiles = (ctx + AD_KT - 1) / AD_KT;
    const long long row_stride = (long long)a.dim * 4;
    const uint8_t* kbase = reinterpret_cast<const uint8_t*>(a.keys + (long long)b * a.capacity * a.dim + h * C::HD);
    const uint8_t* vbase = reinterpret_cast<const uint8_t*>(a.values + (long long)b * a.capacity * a.dim + h * C::HD);
    if (threadIdx.x == 0) {
        for (int s = 0; s < C::STAGES; s++)
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(ad_smem_addr(&full[s])) : "memory");
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    // warp 0: tile t's rows into stage t % STAGES: two tensor copies, or one
    // K and one V row per lane for a tile that wraps round the ring
    const int row_b = a.layer_row0 + b * a.capacity;
    auto issue = [&](int t) {
        const int s = t % C::STAGES;
        const int j0 = t * AD_KT;
        const int n = min(AD_KT, ctx - j0);
        uint8_t* ks = ad_smem + s * C::STAGE;
        uint8_t* vs = ks + AD_KT * C::ROW;
        int p0 = start + j0;   // start < capacity and j0 < ctx <= capacity
        if (p0 >= a.capacity) p0 -= a.capacity;
        if (p0 + n <= a.capacity) {
            // the box's rows past n (another sequence's rows, or past the
            // tensor: zero-filled) are never used
            if (lane == 0) {
                asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(ad_smem_addr(&full[s])),
                             "r"((uint32_t)(2 * AD_KT * C::ROW))
                             : "memory");
                ad_tma_2d(ks, &tmK, h * C::HD, row_b + p0, &full[s]);
                ad_tma_2d(vs, &tmV, h * C::HD, row_b + p0, &full[s]);
            }
            return;
        }
        if (lane == 0)
            asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(ad_smem_addr(&full[s])),
                         "r"((uint32_t)(2 * n * C::ROW))
                         : "memory");
        __syncwarp();
        if (lane < n) {
            int phys = p0 + lane;
            if (phys >= a.capacity) phys -= a.capacity;
            asm volatile(
                "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                    ad_smem_addr(ks + lane * C::ROW)),
                "l"(kbase + phys * row_stride), "r"((uint32_t)C::ROW), "r"(ad_smem_addr(&full[s]))
                : "memory");
            asm volatile(
                "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                    ad_smem_addr(vs + lane * C::ROW)),
                "l"(vbase + phys * row_stride), "r"((uint32_t)C::ROW), "r"(ad_smem_addr(&full[s]))
                : "memory");
        }
    };
    if (warp == 0)
        for (int t = 0; t < C::STAGES && t < ntiles; t++) issue(t);

    float qv[HDW];
    {
        const float* qp = a.q + (long long)b * a.dim + h * C::HD + lane * HDW;
        if (HDW == 4) {
            const float4 v = *reinterpret_cast<const float4*>(qp);
            qv[0] = v.x; qv[1] = v.y; qv[2] = v.z; qv[3] = v.w;
        } else {
            const float2 v = *reinterpret_cast<const float2*>(qp);
            qv[0] = v.x; qv[1] = v.y;
        }
    }
    const float denom = sqrtf((float)C::HD);
    float m = -3.402823466e38f, l = 0.0f, o[HDW];
#pragma unroll
    for (int c = 0; c < HDW; c++) o[c] = 0.0f;
    int t = 0;
    bool failed = false;
    for (; t < ntiles; t++) {
        const int s = t % C::STAGES;
        const bool got = ad_mbar_wait(&full[s], (uint32_t)((t / C::STAGES) & 1));
        if (got) {
            const float* ks = reinterpret_cast<const float*>(ad_smem + s * C::STAGE);
            const float* vs = ks + AD_KT * C::HD;
            float sc[AD_KPW];
#pragma unroll
            for (int u = 0; u < AD_KPW; u++) {
                const float* kr = ks + (warp * AD_KPW + u) * C::HD + lane * HDW;
                float d = 0.0f;
                if (HDW == 4) {
                    const float4 k4 = *reinterpret_cast<const float4*>(kr);
                    d = fmaf(qv[0], k4.x, d);
                    d = fmaf(qv[1], k4.y, d);
                    d = fmaf(qv[2], k4.z, d);
                    d = fmaf(qv[3], k4.w, d);
                } else {
                    const float2 k2 = *reinterpret_cast<const float2*>(kr);
                    d = fmaf(qv[0], k2.x, d);
                    d = fmaf(qv[1], k2.y, d);
                }
                sc[u] = d;
            }
#pragma unroll
            for (int off = 16; off >= 1; off >>= 1)
#pragma unroll
                for (int u = 0; u < AD_KPW; u++) sc[u] += __shfl_xor_sync(0xffffffffu, sc[u], off);
            const int jw = t * AD_KT + warp * AD_KPW;
            float tmax = m;
#pragma unroll
            for (int u = 0; u < AD_KPW; u++) {
                sc[u] = sc[u] / denom;
                if (jw + u < ctx) tmax = fmaxf(tmax, sc[u]);
            }
            const float corr = expf(m - tmax);
            l *= corr;
#pragma unroll
            for (int c = 0; c < HDW; c++) o[c] *= corr;
            m = tmax;
#pragma unroll
            for (int u = 0; u < AD_KPW; u++) {
                if (jw + u < ctx) {
                    const float p = expf(sc[u] - m);
                    l += p;
                    const float* vr = vs + (warp * AD_KPW + u) * C::HD + lane * HDW;
                    if (HDW == 4) {
                        const float4 v4 = *reinterpret_cast<const float4*>(vr);
                        o[0] = fmaf(p, v4.x, o[0]);
                        o[1] = fmaf(p, v4.y, o[1]);
                        o[2] = fmaf(p, v4.z, o[2]);
                        o[3] = fmaf(p, v4.w, o[3]);
                    } else {
                        const float2 v2 = *reinterpret_cast<const float2*>(vr);
                        o[0] = fmaf(p, v2.x, o[0]);
                        o[1] = fmaf(p, v2.y, o[1]);
                    }
                }
            }
        }
        // every warp is done with stage s (or some thread gave up waiting)
        if (__syncthreads_or(!got)) {
            failed = true;
            break;
        }
        if (warp == 0 && t + C::STAGES < ntiles) issue(t + C::STAGES);
    }
    if (failed) {
        if (threadIdx.x == 0 && a.status) atomicExch(a.status, 1);
        // copies still in flight land before the block's shared memory is released
        for (int u = t; u < ntiles && u < t + C::STAGES; u++)
            (void)ad_mbar_wait(&full[u % C::STAGES], (uint32_t)((u / C::STAGES) & 1));
        return;
    }
    // merge the warps' partial softmax states (stage memory is free now)
    float* sm_m = reinterpret_cast<float*>(ad_smem);
    float* sm_l = sm_m + AD_WARPS;
    float* sm_o = sm_l + AD_WARPS;   // [AD_WARPS][HD]
    if (lane == 0) {
        sm_m[warp] = m;
        sm_l[warp] = l;
    }
#pragma unroll
    for (int c = 0; c < HDW; c++) sm_o[warp * C::HD + lane * HDW + c] = o[c];
    __syncthreads();
    if (warp == 0) {
        float M = sm_m[0];
        for (int w = 1; w < AD_WARPS; w++) M = fmaxf(M, sm_m[w]);
        float L = 0.0f, acc[HDW];
#pragma unroll
        for (int c = 0; c < HDW; c++) acc[c] = 0.0f;
        for (int w = 0; w < AD_WARPS; w++) {
            const float f = sm_l[w] > 0.0f ? expf(sm_m[w] - M) : 0.0f;
            L += sm_l[w] * f;
#pragma unroll
            for (int c = 0; c < HDW; c++) acc[c] = fmaf(sm_o[w * C::HD + lane * HDW + c], f, acc[c]);
        }
        const float inv = 1.0f / L;
        float* op = a.out + (long long)b * a.dim + h * C::HD + lane * HDW;
#pragma unroll
        for (int c = 0; c < HDW; c++) op[c] = acc[c] * inv;
    }
}

// Host side (attn.cu): set the kernels' shared-memory limits once; launch
// for head dimension 64 or 128 (cudaErrorNotSupported otherwise).
cudaError_t dz_attn_decode_set_smem();
cudaError_t dz_attn_decode_launch(const CUtensorMap& tmK, const CUtensorMap& tmV, const AdArgs& a, int head_dim,
                                  int heads, int batch, cudaStream_t st);

}  // namespace dz
