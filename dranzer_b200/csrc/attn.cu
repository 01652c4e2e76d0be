// Translation unit of the streamed decode attention (attn.cuh): its code is
// generated apart from the other kernels so that neither's register
// allocation depends on the other's inlining.
#include "attn.cuh"

namespace dz {

cudaError_t dz_attn_decode_set_smem() {
    cudaError_t e = cudaFuncSetAttribute(dz_attn_decode_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         AdCfg<4>::SMEM);
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(dz_attn_decode_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 AdCfg<2>::SMEM);
    return e;
}

cudaError_t dz_attn_decode_launch(const CUtensorMap& tmK, const CUtensorMap& tmV, const AdArgs& a, int head_dim,
                                  int heads, int batch, cudaStream_t st) {
    const dim3 grid((unsigned)heads, (unsigned)batch);
    if (head_dim == 128)
        dz_attn_decode_kernel<4><<<grid, AD_THREADS, AdCfg<4>::SMEM, st>>>(tmK, tmV, a);
    else if (head_dim == 64)
        dz_attn_decode_kernel<2><<<grid, AD_THREADS, AdCfg<2>::SMEM, st>>>(tmK, tmV, a);
    else
        return cudaErrorNotSupported;
    return cudaGetLastError();
}

}  // namespace dz
