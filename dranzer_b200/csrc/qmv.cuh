// Epilogue shared by the quantized matvec kernels (qmma.cuh): per-column scale,
// bias, residual, ReLU, and routing of output columns to up to three
// destinations (the fused QKV product writes q, and K / V straight into each
// sequence's ring slot, src/core/transformer.c:722-728).
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace dz {

constexpr int QMV_THREADS = 256;
constexpr int QMV_WARPS = QMV_THREADS / 32;

struct QmvEpilogue {
    const int* row_shift;     // [M] exponent to undo the activation scaling, or nullptr
    const float* col_scale;   // [Np] per-column scale, or nullptr (scale 1)
    const float* bias;        // [N] or nullptr
    const float* residual;    // [M][ld_res] or nullptr, added after bias
    long long ld_res;
    int act;                  // activation applied last: DZ_ACT_NONE / RELU / GELU
    // Output column segments: columns [seg_start[i], seg_start[i+1]) go to
    // seg_ptr[i] + row*seg_ld[i] + (seg_row_off ? seg_row_off[row] : 0) + (n - seg_start[i]).
    int nseg;
    int seg_start[4];
    float* seg_ptr[3];
    long long seg_ld[3];
    const int* seg_row_off[3];
};

// FFN activations (src/core/tensor_ops.c:17-20 gelu, src/core/transformer.c:
// 485 relu), in the reference's operation order without contraction.
enum { DZ_ACT_NONE = 0, DZ_ACT_RELU = 1, DZ_ACT_GELU = 2 };
__device__ __forceinline__ float dz_act(float y, int act) {
    if (act == DZ_ACT_RELU) return y > 0.0f ? y : 0.0f;
    if (act == DZ_ACT_GELU)
        return __fmul_rn(__fmul_rn(0.5f, y), __fadd_rn(1.0f, erff(__fmul_rn(y, 0.70710678118654752440f))));
    return y;
}

// The output segment holding column n. Only constant indices into the
// epilogue's arrays: a kernel parameter indexed with a run-time value has to
// be addressable, and every access through it then becomes a generic load.
struct DzSeg {
    float* ptr;
    long long ld;
    const int* row_off;
    int start, end;
};
__device__ __forceinline__ DzSeg dz_seg_of(const QmvEpilogue& e, int n) {
    DzSeg s{e.seg_ptr[0], e.seg_ld[0], e.seg_row_off[0], e.seg_start[0], e.nseg > 1 ? e.seg_start[1] : 0x7fffffff};
    if (e.nseg > 1 && n >= e.seg_start[1])
        s = DzSeg{e.seg_ptr[1], e.seg_ld[1], e.seg_row_off[1], e.seg_start[1], e.nseg > 2 ? e.seg_start[2] : 0x7fffffff};
    if (e.nseg > 2 && n >= e.seg_start[2])
        s = DzSeg{e.seg_ptr[2], e.seg_ld[2], e.seg_row_off[2], e.seg_start[2], 0x7fffffff};
    return s;
}

__device__ __forceinline__ void dz_qmv_store_row(const QmvEpilogue& e, int M, int N, int m, int n, float acc) {
    if (m >= M || n >= N) return;
    if (e.row_shift) {   // acc * 2^row_shift[m], exact for normal results
        const int x = e.row_shift[m];
        if (x >= -126 && x <= 127) {
            acc *= __int_as_float((x + 127) << 23);
        } else {
            const int h = x / 2;
            acc = (acc * __int_as_float((h + 127) << 23)) * __int_as_float((x - h + 127) << 23);
        }
    }
    float y = e.col_scale ? acc * e.col_scale[n] : acc;
    if (e.bias) y = y + e.bias[n];
    if (e.residual) y = y + e.residual[(long long)m * e.ld_res + n];
    if (e.act) y = dz_act(y, e.act);
    const DzSeg sg = dz_seg_of(e, n);
    long long off = (long long)m * sg.ld + (n - sg.start);
    if (sg.row_off) off += sg.row_off[m];
    sg.ptr[off] = y;
}

}  // namespace dz
