// Translation unit of the tensor-core prefill attention (pfattn.cuh), apart
// from the other kernels so that its register allocation does not depend on
// theirs.
#include "pfattn.cuh"

namespace dz {

cudaError_t dz_pfattn_set_smem() {
    cudaError_t e = cudaFuncSetAttribute(dz_pfattn_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)dz_pfattn_smem(128));
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(dz_pfattn_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)dz_pfattn_smem(64));
    return e;
}

cudaError_t dz_pfattn_launch(const float* q, const float* keys, const float* values, const int* lens, float* out,
                             int T, int dim, int capacity, int head_dim, int heads, int seqs, cudaStream_t st) {
    const dim3 grid((unsigned)((T + PT_QT - 1) / PT_QT), (unsigned)heads, (unsigned)seqs);
    if (head_dim == 128)
        dz_pfattn_kernel<4><<<grid, PT_THREADS, dz_pfattn_smem(128), st>>>(q, keys, values, lens, out, T, dim,
                                                                          capacity);
    else if (head_dim == 64)
        dz_pfattn_kernel<2><<<grid, PT_THREADS, dz_pfattn_smem(64), st>>>(q, keys, values, lens, out, T, dim,
                                                                         capacity);
    else
        return cudaErrorNotSupported;
    return cudaGetLastError();
}

}  // namespace dz
