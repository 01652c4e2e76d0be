// LayerNorm fused with the activation split of the tensor-core GEMM that
// reads its output (umma.cuh): the norm writes its fp32 rows (the residual
// path reads them) and also the next product's limb planes and row shift,
// so that product needs no split kernel.
//
// The statistics and the element formula are those of dz_layernorm_kernel
// (decode.cuh; layer_normalize, src/core/tensor_ops.c:88-111), and the limbs
// those of dz_limb_split_kernel (ug_fixed, ug_digits): the fp32 output, the
// limbs and the shift are bit for bit what the two kernels write.
#pragma once
#include "decode.cuh"
#include "umma.cuh"

namespace dz {

constexpr int LN_LIMBS_V4 = 4;                                       // float4s per thread
constexpr int LN_LIMBS_MAX_DIM = LN_THREADS * 4 * LN_LIMBS_V4;       // 4096

// One block of LN_THREADS per row (dim <= LN_LIMBS_MAX_DIM, dim % 4 == 0, rows
// and norm parameters 16-byte aligned): y = norm(x + residual), the element
// pass in float4s; L[limb][row][k] (planes of M x Kp, zero for dim <= k < Kp,
// four k per 32-bit store) and shift[row] = -s, or UG_ROW_NONFINITE for a row
// holding inf or NaN.
__global__ void __launch_bounds__(LN_THREADS) dz_layernorm_limbs_kernel(
    const float* __restrict__ x, const float* __restrict__ residual, const float* __restrict__ gamma,
    const float* __restrict__ beta, float* __restrict__ y, int dim, float eps, int M, int Kp,
    int8_t* __restrict__ L, int* __restrict__ shift) {
    __shared__ float red[LN_THREADS / 32];
    __shared__ float stat;
    __shared__ float wred[LN_THREADS / 32];
    __shared__ int wbad[LN_THREADS / 32];
    const int r = blockIdx.x;
    const float* xr = x + (long long)r * dim;
    const float* rr = residual ? residual + (long long)r * dim : nullptr;
    float* yr = y + (long long)r * dim;
    float mean, sd;
    dz_ln_stats(xr, rr, dim, eps, red, &stat, mean, sd);
    float4 yv[LN_LIMBS_V4];
    float m = 0.0f;
    int bad = 0;
#pragma unroll
    for (int j = 0; j < LN_LIMBS_V4; j++) {
        const int i = (j * LN_THREADS + (int)threadIdx.x) * 4;
        yv[j] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        if (i >= dim) continue;
        float4 xv = *reinterpret_cast<const float4*>(xr + i);
        if (rr) {
            const float4 rv = *reinterpret_cast<const float4*>(rr + i);
            xv.x = xv.x + rv.x;
            xv.y = xv.y + rv.y;
            xv.z = xv.z + rv.z;
            xv.w = xv.w + rv.w;
        }
        const float4 g = *reinterpret_cast<const float4*>(gamma + i);
        const float4 b = *reinterpret_cast<const float4*>(beta + i);
        yv[j].x = dz_ln_value(xv.x, mean, sd, g.x, b.x);
        yv[j].y = dz_ln_value(xv.y, mean, sd, g.y, b.y);
        yv[j].z = dz_ln_value(xv.z, mean, sd, g.z, b.z);
        yv[j].w = dz_ln_value(xv.w, mean, sd, g.w, b.w);
        *reinterpret_cast<float4*>(yr + i) = yv[j];
        const float e[4] = {yv[j].x, yv[j].y, yv[j].z, yv[j].w};
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
    for (int w = 0; w < LN_THREADS / 32; w++) {
        amax = fmaxf(amax, wred[w]);
        bad |= wbad[w];
    }
    const int s = amax > 0.0f ? (UG_X_BITS - 1) - dz_ilogb(amax) : 0;
    const size_t plane = (size_t)M * Kp;
    int8_t* lr = L + (size_t)r * Kp;
#pragma unroll
    for (int j = 0; j < LN_LIMBS_V4; j++) {
        const int i = (j * LN_THREADS + (int)threadIdx.x) * 4;
        if (i >= Kp) continue;
        const float e[4] = {yv[j].x, yv[j].y, yv[j].z, yv[j].w};   // zero past dim
        uint32_t t4 = 0, m4 = 0, l4 = 0;
#pragma unroll
        for (int c = 0; c < 4; c++) {
            uint32_t dt, dm, dl;
            ug_digits(ug_fixed(e[c], s), dt, dm, dl);
            t4 |= dt << (8 * c);
            m4 |= dm << (8 * c);
            l4 |= dl << (8 * c);
        }
        *reinterpret_cast<uint32_t*>(lr + i) = t4;
        *reinterpret_cast<uint32_t*>(lr + plane + i) = m4;
        *reinterpret_cast<uint32_t*>(lr + 2 * plane + i) = l4;
    }
    if (threadIdx.x == 0) shift[r] = bad ? UG_ROW_NONFINITE : -s;
}

}  // namespace dz
