// The integer-MMA decode matvec (qmvi.cuh) in a translation unit of its own:
// its instantiations stay out of dz_cuda.cu, whose other kernels (the fused
// generation kernel above all) are compiled exactly as without it.
#define DZ_KERNEL_LINKAGE static   // the helper headers' own kernels stay private to dz_cuda.cu
#include "qmvi.cuh"

namespace dz {

cudaError_t dz_qmv1i_set_smem(int bytes) {
    const void* k[4] = {(const void*)dz_qmv1i_kernel<4, QMV1I_WARPS, 1>, (const void*)dz_qmv1i_kernel<4, QMV1I_WARPS, 2>,
                        (const void*)dz_qmv1i_kernel<8, QMV1I_WARPS, 1>, (const void*)dz_qmv1i_kernel<8, QMV1I_WARPS, 2>};
    for (const void* f : k) {
        const cudaError_t e = cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

cudaError_t dz_qmv1i_launch(const Qmv1iArgs& a, int bits, int grid, size_t smem, cudaStream_t st) {
    void (*k)(Qmv1iArgs) = bits == 8 ? (a.M == 2 ? dz_qmv1i_kernel<8, QMV1I_WARPS, 2> : dz_qmv1i_kernel<8, QMV1I_WARPS, 1>)
                                     : (a.M == 2 ? dz_qmv1i_kernel<4, QMV1I_WARPS, 2> : dz_qmv1i_kernel<4, QMV1I_WARPS, 1>);
    // programmatic dependent launch: the kernel streams weights before it
    // waits for the previous kernel in the stream
    cudaLaunchConfig_t cfg;
    memset(&cfg, 0, sizeof(cfg));
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3(QMV1I_WARPS * 32);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaLaunchKernelEx(&cfg, k, a) != cudaSuccess) {
        (void)cudaGetLastError();
        k<<<grid, QMV1I_WARPS * 32, smem, st>>>(a);
    }
    return cudaGetLastError();
}

}  // namespace dz
