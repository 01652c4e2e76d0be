// The fused one-CTA-per-sequence generation kernel (seqgen.cuh) in a
// translation unit of its own, so that its code does not depend on what the
// other kernels of dz_cuda.cu compile to (shared inline helpers and library
// calls are inlined per unit).
#define DZ_KERNEL_LINKAGE static   // the helper headers' own kernels stay private to dz_cuda.cu
#include "seqgen.cuh"

namespace dz {

cudaError_t dz_seqgen_set_smem(int bits, int bytes) {
    return bits == 8 ? cudaFuncSetAttribute(dz_seqgen_kernel<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes)
                     : cudaFuncSetAttribute(dz_seqgen_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
}

cudaError_t dz_seqgen_launch(const SeqParams& p, int bits, int blocks, size_t smem, cudaStream_t st) {
    if (bits == 8) dz_seqgen_kernel<8><<<blocks, SEQ_THREADS, smem, st>>>(p);
    else dz_seqgen_kernel<4><<<blocks, SEQ_THREADS, smem, st>>>(p);
    return cudaGetLastError();
}

}  // namespace dz
