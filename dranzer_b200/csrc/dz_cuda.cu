// dranzer-b200 CUDA shim: handles, device layout, launch plans and the C ABI
// of include/dz_cuda.h. Kernels live in qmv.cuh, decode.cuh and select.cuh.
#include "dz_cuda.h"
#include "dz_host.h"

#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <algorithm>
#include <map>
#include <mutex>
#include <new>
#include <string>
#include <tuple>
#include <vector>

#include "decode.cuh"
#include "qmv.cuh"
#include "qmma.cuh"
#include "select.cuh"
#include "prefill.cuh"
#include "seqgen.cuh"
#include "umma.cuh"
#include "qmvi.cuh"
#include "arch.cuh"
#include "attn.cuh"
#include "pfattn.cuh"
#include "normlimbs.cuh"

using namespace dz;

// ------------------------------------------------------------------ errors

static thread_local int g_status = DZ_OK;
static thread_local char g_message[512] = "";

static int fail(int status, const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_message, sizeof(g_message), fmt, ap);
    va_end(ap);
    g_status = status;
    return status;
}

#define DZ_CUDA(call)                                                                      \
    do {                                                                                   \
        cudaError_t e_ = (call);                                                           \
        if (e_ != cudaSuccess)                                                             \
            return fail(e_ == cudaErrorMemoryAllocation ? DZ_E_NOMEM : DZ_E_DEVICE,        \
                        "%s: %s (%s:%d)", #call, cudaGetErrorString(e_), __FILE__, __LINE__); \
    } while (0)

extern "C" int dz_cuda_last_error(char* buf, size_t n) {
    if (buf && n) {
        strncpy(buf, g_message, n - 1);
        buf[n - 1] = 0;
    }
    return g_status;
}

// Switches to a handle's device for the duration of a call.
struct DeviceGuard {
    int prev = -1;
    bool ok = true;
    explicit DeviceGuard(int dev) {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        if (prev != dev) ok = cudaSetDevice(dev) == cudaSuccess;
    }
    ~DeviceGuard() {
        int cur;
        if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
    }
};

extern "C" int dz_cuda_available(void) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) {
        cudaGetLastError();
        return 0;
    }
    for (int d = 0; d < n; d++) {
        cudaDeviceProp p;
        if (cudaGetDeviceProperties(&p, d) == cudaSuccess && p.major == 10) return 1;
    }
    return 0;
}

// -------------------------------------------------------- device matrices

// A quantized matrix on the device, codes in the MMA-fragment layout of qmma.cuh.
struct DevQMat {
    int K = 0, N = 0, Np = 0, bits = 0, gran = 0;
    int ntiles = 0, nkg = 0;     // n-tiles of 16 columns, k-groups of 64 (INT4) / 32 (INT8) rows
    uint8_t* codes = nullptr;
    float* col_scale = nullptr;  // [Np] (COLUMN / TENSOR expanded), zero in padding
    float* k_scale = nullptr;    // [K] ROW granularity
    size_t code_bytes = 0, scale_bytes = 0;
    // the levels again, one signed byte each, in K-major 16 KB blocks
    // [n / 128][k / 128][n % 128][k % 128], with their TMA map, for the
    // tensor-core kernels
    int8_t* kn = nullptr;
    CUtensorMap tm_kn;
};

static void free_qmat(DevQMat& m) {
    cudaFree(m.codes);
    cudaFree(m.col_scale);
    cudaFree(m.k_scale);
    cudaFree(m.kn);
    m = DevQMat();
}

// cuTensorMapEncodeTiled from the driver (no link-time dependency on libcuda).
using TensorMapEncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                       const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                       CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
static TensorMapEncodeFn tensor_map_encoder() {
    static TensorMapEncodeFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<TensorMapEncodeFn>(p);
    });
    return fn;
}

// A 128 x 128-byte tiled uint8 TMA map with the 128-byte swizzle over a
// tensor of `rank` dims (dims[0] innermost, strides in bytes for dims 1..).
static bool encode_u8_map(CUtensorMap* tm, void* base, int rank, const cuuint64_t* dims, const cuuint64_t* strides,
                          const cuuint32_t* box) {
    TensorMapEncodeFn enc = tensor_map_encoder();
    if (!enc) return false;
    const cuuint32_t es[5] = {1, 1, 1, 1, 1};
    return enc(tm, CU_TENSOR_MAP_DATA_TYPE_UINT8, (cuuint32_t)rank, base, dims, strides, box, es,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

static int round_up(int x, int m) { return (x + m - 1) / m * m; }

static int check_blob(const dz_tensor_blob_t* w) {
    size_t ns = 0, nb = 0;
    if (!w || !w->scales || !w->packed || w->rows == 0 || w->cols == 0 ||
        (w->bits != 4 && w->bits != 8) || w->rows > (1u << 30) || w->cols > (1u << 30) ||
        dz_quantized_scale_count(w->rows, w->cols, w->granularity, &ns) != 0 ||
        dz_quantized_packed_size(w->rows * w->cols, w->bits, &nb) != 0 || w->scale_count != ns ||
        w->packed_size != nb)
        return fail(DZ_E_INVALID, "quantized blob: bad shape, bit width or buffer sizes");
    return DZ_OK;
}

// Builds the fragment layout of the column concatenation of `srcs` (same K,
// bits and granularity). Device allocations are recorded in *out as they are
// made, so the caller's free_qmat(*out) releases them on any failure.
static int make_qmat_into(const std::vector<const dz_tensor_blob_t*>& srcs, cudaStream_t st, DevQMat& m,
                          std::vector<uint8_t*>& staging) {
    const dz_tensor_blob_t* s0 = srcs[0];
    if (srcs.size() > 3) return fail(DZ_E_INVALID, "at most three concatenated matrices");
    for (auto* s : srcs) {
        int rc = check_blob(s);
        if (rc) return rc;
        if (s->rows != s0->rows || s->bits != s0->bits || s->granularity != s0->granularity)
            return fail(DZ_E_INVALID, "concatenated matrices disagree in K, bits or granularity");
    }
    if (srcs.size() > 1 && s0->granularity == DZ_GRAN_ROW)
        return fail(DZ_E_INVALID, "ROW-granularity matrices cannot share one device matrix");
    m.K = (int)s0->rows;
    m.bits = s0->bits;
    m.gran = s0->granularity;
    FragSources fs;
    memset(&fs, 0, sizeof(fs));
    fs.nsrc = (int)srcs.size();
    int N = 0;
    for (size_t i = 0; i < srcs.size(); i++) {
        fs.off[i] = N;
        N += (int)srcs[i]->cols;
    }
    fs.off[srcs.size()] = N;
    m.N = N;
    m.Np = round_up(N, 16);
    m.ntiles = m.Np / 16;
    const int KG = m.bits == 8 ? 32 : 64;
    m.nkg = round_up(m.K, KG) / KG;
    m.code_bytes = (size_t)m.ntiles * m.nkg * 512;
    DZ_CUDA(cudaMalloc(&m.codes, m.code_bytes));
    DZ_CUDA(cudaMalloc(&m.col_scale, (size_t)m.Np * sizeof(float)));
    DZ_CUDA(cudaMemsetAsync(m.col_scale, 0, (size_t)m.Np * sizeof(float), st));
    m.scale_bytes = (size_t)N * 4;
    if (m.gran == DZ_GRAN_ROW) {
        DZ_CUDA(cudaMalloc(&m.k_scale, (size_t)m.K * sizeof(float)));
        DZ_CUDA(cudaMemcpyAsync(m.k_scale, s0->scales, (size_t)m.K * 4, cudaMemcpyHostToDevice, st));
        std::vector<float> ones(m.Np, 0.0f);
        for (int i = 0; i < N; i++) ones[i] = 1.0f;
        DZ_CUDA(cudaMemcpyAsync(m.col_scale, ones.data(), (size_t)m.Np * 4, cudaMemcpyHostToDevice, st));
        DZ_CUDA(cudaStreamSynchronize(st));
        m.scale_bytes = (size_t)m.K * 4;
    }
    for (size_t i = 0; i < srcs.size(); i++) {
        uint8_t* d = nullptr;
        DZ_CUDA(cudaMalloc(&d, srcs[i]->packed_size));
        staging.push_back(d);
        DZ_CUDA(cudaMemcpyAsync(d, srcs[i]->packed, srcs[i]->packed_size, cudaMemcpyHostToDevice, st));
        fs.ref[i] = d;
        if (m.gran == DZ_GRAN_COLUMN) {
            DZ_CUDA(cudaMemcpyAsync(m.col_scale + fs.off[i], srcs[i]->scales, srcs[i]->cols * 4,
                                    cudaMemcpyHostToDevice, st));
        } else if (m.gran == DZ_GRAN_TENSOR) {
            std::vector<float> rep(srcs[i]->cols, srcs[i]->scales[0]);
            DZ_CUDA(cudaMemcpyAsync(m.col_scale + fs.off[i], rep.data(), srcs[i]->cols * 4, cudaMemcpyHostToDevice,
                                    st));
            DZ_CUDA(cudaStreamSynchronize(st));
        }
    }
    const long long nwords = (long long)m.ntiles * m.nkg * 128;
    dz_frag_repack_kernel<<<(unsigned)((nwords + 255) / 256), 256, 0, st>>>(fs, reinterpret_cast<uint32_t*>(m.codes),
                                                                           m.K, m.bits, m.nkg, nwords);
    DZ_CUDA(cudaGetLastError());
    if (tensor_map_encoder() && m.K <= UG_MAX_K) {
        // K-major level blocks for the tensor-core kernels
        const int nt = (N + UG_BN - 1) / UG_BN, nkb = (m.K + UG_BK - 1) / UG_BK;
        const size_t blk = (size_t)UG_BN * UG_BK, bytes = (size_t)nt * nkb * blk;
        DZ_CUDA(cudaMalloc(&m.kn, bytes));
        DZ_CUDA(cudaMemsetAsync(m.kn, 0, bytes, st));
        for (size_t i = 0; i < srcs.size(); i++) {
            const long long total = (long long)m.K * (long long)srcs[i]->cols;
            dz_code_blocks_kernel<<<(unsigned)((total + 255) / 256), 256, 0, st>>>(
                fs.ref[i], m.bits, (long long)srcs[i]->cols, total, m.kn, nkb, fs.off[i]);
            DZ_CUDA(cudaGetLastError());
        }
        const cuuint64_t dims[4] = {(cuuint64_t)UG_BK, (cuuint64_t)UG_BN, (cuuint64_t)nkb, (cuuint64_t)nt};
        const cuuint64_t strides[3] = {(cuuint64_t)UG_BK, (cuuint64_t)blk, (cuuint64_t)blk * nkb};
        const cuuint32_t box[4] = {UG_BK, UG_BN, 1, 1};
        if (!encode_u8_map(&m.tm_kn, m.kn, 4, dims, strides, box)) {
            cudaFree(m.kn);
            m.kn = nullptr;
        }
    }
    DZ_CUDA(cudaStreamSynchronize(st));
    return DZ_OK;
}

static int make_qmat(const std::vector<const dz_tensor_blob_t*>& srcs, cudaStream_t st, DevQMat* out) {
    std::vector<uint8_t*> staging;
    int rc = make_qmat_into(srcs, st, *out, staging);
    for (uint8_t* p : staging) cudaFree(p);
    return rc;
}

// ---------------------------------------------------------------- profiler

// Optional per-launch CUDA events (dz_cuda_profile_generate): each launch
// site brackets its kernel with two events on the launching stream and
// records the kernel class and its algorithmic bytes / flops.
struct ProfRec {
    int kind;
    double bytes, flops;
    cudaEvent_t a, b;
};
static thread_local std::vector<ProfRec>* g_prof = nullptr;

struct ProfScope {
    ProfRec rec{};
    cudaStream_t st;
    bool on;
    ProfScope(int kind, double bytes, double flops, cudaStream_t s) : st(s), on(g_prof != nullptr) {
        if (!on) return;
        rec.kind = kind;
        rec.bytes = bytes;
        rec.flops = flops;
        cudaEventCreate(&rec.a);
        cudaEventCreate(&rec.b);
        cudaEventRecord(rec.a, st);
    }
    ~ProfScope() {
        if (!on) return;
        cudaEventRecord(rec.b, st);
        g_prof->push_back(rec);
    }
};

// ------------------------------------------------------------- qmv plans

template <int BITS, int NB, int NT>
static void launch_qmm_t(const QmmArgs& a, unsigned grid, cudaStream_t st) {
    dz_qmm_kernel<BITS, NB, NT><<<grid, QMV_THREADS, 0, st>>>(a);
}

template <int BITS>
static void launch_qmm_bits(const QmmArgs& a, int NB, unsigned grid, cudaStream_t st) {
    switch (NB) {
        case 1: launch_qmm_t<BITS, 1, 4>(a, grid, st); break;
        case 2: launch_qmm_t<BITS, 2, 2>(a, grid, st); break;
        case 4: launch_qmm_t<BITS, 4, 2>(a, grid, st); break;
        default: launch_qmm_t<BITS, 8, 1>(a, grid, st); break;
    }
}

static int g_num_sms = 148;

static size_t r256(size_t n) { return (n + 255) & ~(size_t)255; }

// Bytes of split-activation scratch one matvec of this matrix needs for M
// rows: the B-fragment-ordered splits (16 bytes per k row per row pair), then
// the M row exponents.
static size_t qmv_xf_bytes(const DevQMat& W, int M) {
    const int KG = W.bits == 8 ? 32 : 64;
    return (size_t)W.nkg * KG * (size_t)((M + 1) / 2) * 16;
}
// Bytes of scratch the tensor-core GEMM needs for M rows: three limb planes
// of M x (K rounded up to 128) bytes and the row exponents.
// Split-K parts of the tensor-core GEMM: a grid of fewer tiles than half the
// SMs with a long k (32 or more k blocks) gets its k blocks cut into parts
// (at least eight k blocks each, at most eight parts) so that about one CTA
// per SM runs; below that k a part's main loop is too short to pay for
// storing and adding the int64 partial tiles. Off while g_no_split_k is set
// (callers with a fixed scratch budget).
static thread_local bool g_no_split_k = false;
static int ugemm_kparts(const DevQMat& W, int M) {
    if (g_no_split_k) return 1;
    const int tiles = ((W.N + UG_BN - 1) / UG_BN) * ((M + UG_BM - 1) / UG_BM);
    const int nkb = round_up(W.K, UG_BK) / UG_BK;
    if (2 * tiles > g_num_sms || nkb < 32) return 1;
    return std::max(1, std::min({g_num_sms / tiles, nkb / 8, 8}));
}
static size_t ugemm_scratch_bytes(const DevQMat& W, int M) {
    const size_t kp = (size_t)round_up(W.K, UG_BK);
    size_t b = r256(3 * (size_t)M * kp) + r256((size_t)M * 4);
    const int parts = ugemm_kparts(W, M);
    if (parts > 1)
        b += (size_t)((W.N + UG_BN - 1) / UG_BN) * ((M + UG_BM - 1) / UG_BM) * parts * UG_BM * UG_BN * 8;
    return b;
}
// Every scratch buffer starts with the GEMV's per-tile counters, shared by
// all matrices that use the buffer (each launch leaves the counters it used
// at zero; the scratch is zeroed when allocated); the kernels' own scratch
// follows.
constexpr int UGEMV_MAX_TILES = 4096;
constexpr size_t SCRATCH_COUNTERS = (size_t)UGEMV_MAX_TILES * 4;
// CTAs of the GEMV: one per SM, fewer when the matrix has fewer than
// UV_MIN_STAGES_PER_CTA stages for each.
static int ugemv_grid(const DevQMat& W) {
    const long long total = (long long)((W.N + UG_BN - 1) / UG_BN) * ((W.K + UG_BK - 1) / UG_BK);
    return (int)std::max(1LL, std::min((long long)g_num_sms, total / UV_MIN_STAGES_PER_CTA));
}
// Scratch of the tensor-core GEMV for M <= 16 rows: limbs, exponents and two
// int64 partial slots per CTA.
static size_t ugemv_scratch_bytes(const DevQMat& W, int M) {
    const size_t kp = (size_t)round_up(W.K, UG_BK);
    return r256(3 * (size_t)M * kp) + r256((size_t)M * 4) + r256((size_t)ugemv_grid(W) * 2 * UV_SLOT_ELEMS * 8);
}
static size_t qmv_scratch_bytes(const DevQMat& W, int M) {
    const size_t xf = r256(qmv_xf_bytes(W, M)) + r256((size_t)M * 4);
    if (!W.kn) return SCRATCH_COUNTERS + xf;
    return SCRATCH_COUNTERS +
           std::max({xf, ugemm_scratch_bytes(W, M), M <= UV_N ? ugemv_scratch_bytes(W, M) : (size_t)0});
}

template <int BITS, int NB, int NT, int W, bool XIN>
static void launch_qms_t(const QmsArgs& a, unsigned grid, size_t smem, cudaStream_t st) {
    dz_qms_kernel<BITS, NB, NT, W, XIN><<<grid, W * 32, smem, st>>>(a);
}

// Streaming-kernel shape per row count: NB row pairs per MMA group, NT n-tiles
// per warp, W warps per CTA.
static void qms_shape(int M, int* NB, int* NT, int* W) {
    *NB = M <= 2 ? 1 : M <= 4 ? 2 : M <= 8 ? 4 : 8;
    *NT = *NB == 1 ? 1 : *NB == 2 ? 2 : *NB == 4 ? 4 : 2;
    *W = *NB <= 2 ? 16 : 8;
}

template <int BITS, bool XIN>
static void launch_qms_bits(const QmsArgs& a, int NB, unsigned grid, size_t smem, cudaStream_t st) {
    switch (NB) {
        case 1: launch_qms_t<BITS, 1, 1, 16, XIN>(a, grid, smem, st); break;
        case 2: launch_qms_t<BITS, 2, 2, 16, XIN>(a, grid, smem, st); break;
        case 4: launch_qms_t<BITS, 4, 4, 8, XIN>(a, grid, smem, st); break;
        default: launch_qms_t<BITS, 8, 2, 8, XIN>(a, grid, smem, st); break;
    }
}

// Warps per CTA of the stream-K matvec (M <= 2).
constexpr int QMV1_WARPS = 16;

// The streaming kernels take more than the default 48 KB of shared memory;
// the attribute is set once per device, outside any stream capture.
static std::mutex g_qms_mutex;
static bool g_qms_ready[256];
static int g_smem_optin = 232448;

static int qms_prepare(int device) {
    if (device < 0 || device >= 256) return fail(DZ_E_DEVICE, "device %d out of range", device);
    std::lock_guard<std::mutex> lock(g_qms_mutex);
    if (g_qms_ready[device]) return DZ_OK;
    int optin = 0;
    DZ_CUDA(cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, device));
    g_smem_optin = optin;
#define DZ_QMS_ATTR(B, NB, NT, W, X) \
    DZ_CUDA(cudaFuncSetAttribute(dz_qms_kernel<B, NB, NT, W, X>, cudaFuncAttributeMaxDynamicSharedMemorySize, optin))
#define DZ_QMS_ATTR2(B, X) \
    DZ_QMS_ATTR(B, 1, 1, 16, X); DZ_QMS_ATTR(B, 2, 2, 16, X); DZ_QMS_ATTR(B, 4, 4, 8, X); DZ_QMS_ATTR(B, 8, 2, 8, X)
    DZ_QMS_ATTR2(4, false); DZ_QMS_ATTR2(4, true); DZ_QMS_ATTR2(8, false); DZ_QMS_ATTR2(8, true);
#undef DZ_QMS_ATTR2
#undef DZ_QMS_ATTR
#define DZ_QMV1_ATTR(B, X) \
    DZ_CUDA(cudaFuncSetAttribute(dz_qmv1_kernel<B, QMV1_WARPS, X>, cudaFuncAttributeMaxDynamicSharedMemorySize, optin))
    DZ_QMV1_ATTR(4, false); DZ_QMV1_ATTR(4, true); DZ_QMV1_ATTR(8, false); DZ_QMV1_ATTR(8, true);
#undef DZ_QMV1_ATTR
    DZ_CUDA(dz_qmv1i_set_smem(optin));
    DZ_CUDA(dz_attn_decode_set_smem());
    DZ_CUDA(dz_pfattn_set_smem());
    DZ_CUDA(cudaFuncSetAttribute(dz_ugemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)UG_SMEM_BYTES));
    DZ_CUDA(cudaFuncSetAttribute(dz_ugemv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)UV_SMEM_BYTES));
    // the split runs right before the GEMV (and may share SMs with it): the
    // same shared-memory carve-out spares a reconfiguration between them
    DZ_CUDA(cudaFuncSetAttribute(dz_limb_split_chunk_kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                                 (int)cudaSharedmemCarveoutMaxShared));
    g_qms_ready[device] = true;
    return DZ_OK;
}

// Rows up to which the streaming kernel serves a product.
constexpr int QMS_MAX_M = 16;
// B fragments up to this size are copied into each CTA's shared memory.
constexpr unsigned QMS_XF_SMEM_MAX = 96u << 10;

// k-parts for the streaming kernel: the split of n-groups x k-groups over the
// warps of g_num_sms persistent CTAs with the fewest k-groups on the busiest
// warp (ties: fewer k-parts, fewer reductions).
static int qms_kparts(int n_groups, int nkg, int W, int* nrounds_out, unsigned* grid_out) {
    long long best_cost = -1;
    int best = 1;
    for (int kp = 1; kp <= W; kp *= 2) {
        const long long per_round = W / kp;
        const long long rounds = (n_groups + per_round - 1) / per_round;
        const long long grid = std::min<long long>(rounds, g_num_sms);
        const long long waves = (rounds + grid - 1) / grid;
        const long long per = (nkg + kp - 1) / kp;
        const long long cost = waves * per + waves;   // + one reduction per round
        if (best_cost < 0 || cost < best_cost) {
            best_cost = cost;
            best = kp;
        }
    }
    const long long per_round = W / best;
    const long long rounds = (n_groups + per_round - 1) / per_round;
    *nrounds_out = (int)rounds;
    *grid_out = (unsigned)std::min<long long>(rounds, g_num_sms);
    return best;
}

// Which M <= 2 matvec kernel runs: the integer dot-product kernel
// (dz_qmv1i_kernel, the default) or the fp16 tensor-core one
// (dz_qmv1_kernel). DZ_MATVEC_KERNEL=mma in the environment selects the
// latter, for comparison; both compute the same product.
static bool matvec_int_kernel() {
    static const bool v = [] {
        const char* e = getenv("DZ_MATVEC_KERNEL");
        return !(e && strcmp(e, "mma") == 0);
    }();
    return v;
}

// Which decode attention runs for head dimensions 64 and 128: the streamed
// kernel (attn.cuh, the default) or the register-blocked one
// (dz_attention_decode2_kernel). DZ_ATTN_KERNEL=regs in the environment
// selects the latter, for comparison; both compute the same attention.
static bool attn_streamed_kernel() {
    static const bool v = [] {
        const char* e = getenv("DZ_ATTN_KERNEL");
        return !(e && strcmp(e, "regs") == 0);
    }();
    return v;
}

// Which causal prefill attention runs for head dimensions 64 and 128: the
// tensor-core kernel (pfattn.cuh, the default) or the CUDA-core one
// (dz_attention_prefill_kernel). DZ_PREFILL_ATTN=simt in the environment
// selects the latter, for comparison; both compute the same attention.
static bool prefill_attn_tensor_cores() {
    static const bool v = [] {
        const char* e = getenv("DZ_PREFILL_ATTN");
        return !(e && strcmp(e, "simt") == 0);
    }();
    return v;
}

// Launch geometry of the integer dot-product matvec (qmvi.cuh): grid, tiles
// per CTA, parts per tile, chunks per piece and shared memory. False when it
// is not selected, K is above its exact range, or its limb table and one
// stage per warp do not fit shared memory.
struct Qmv1iPlan {
    int G, max_tiles, max_parts, pk;
    unsigned tab_bytes;
    size_t smem;
};
static bool qmv1i_plan(const DevQMat& W, int M, Qmv1iPlan* p) {
    constexpr int WP = QMV1I_WARPS;
    if (W.K > QI_MAX_K || M < 1 || M > 2 || !matvec_int_kernel()) return false;
    const int KT = W.bits == 8 ? 2 : 4;
    p->tab_bytes = dz_qmv1i_tab_bytes(W.nkg, KT);
    p->G = std::min(g_num_sms, W.ntiles);
    p->max_tiles = (W.ntiles + p->G - 1) / p->G;
    // a tile meets at most (nkg - 2) / shortest range + 2 non-empty warp ranges
    const long long per_min = (long long)(W.ntiles / p->G) * W.nkg / WP;
    p->max_parts =
        per_min >= 1 ? (int)std::min<long long>(WP, std::max<long long>(1, (W.nkg - 2) / per_min + 2)) : WP;
    if ((long long)p->max_tiles * W.nkg * WP >= (1LL << 31)) return false;   // the kernel's 32-bit range arithmetic
    const size_t fixed = dz_qmv1i_smem_bytes(0, WP, p->tab_bytes, p->max_tiles, p->max_parts, M);
    if (fixed + (size_t)WP * QMS_STAGES * 512 > (size_t)g_smem_optin) return false;
    p->pk = (int)std::min<size_t>(16, ((size_t)g_smem_optin - fixed) / ((size_t)WP * QMS_STAGES * 512));
    p->smem = dz_qmv1i_smem_bytes(p->pk, WP, p->tab_bytes, p->max_tiles, p->max_parts, M);
    return true;
}

static bool qmv1i_launch(const DevQMat& W, const float* X, long long ldx, int M, const QmvEpilogue& ep,
                         cudaStream_t st, int* status, double qmv_bytes) {
    Qmv1iPlan pl;
    if (!qmv1i_plan(W, M, &pl)) return false;
    Qmv1iArgs a;
    memset(&a, 0, sizeof(a));
    a.codes = W.codes;
    a.N = W.N;
    a.nkg = W.nkg;
    a.ntiles = W.ntiles;
    a.X = X;
    a.ldx = ldx;
    a.k_scale = W.k_scale;
    a.K = W.K;
    a.M = M;
    a.status = status;
    a.ep = ep;
    a.ep.row_shift = nullptr;
    a.tab_bytes = pl.tab_bytes;
    a.max_tiles = pl.max_tiles;
    a.max_parts = pl.max_parts;
    a.pk = pl.pk;
    ProfScope prof(DZ_KERNEL_QMV, qmv_bytes, 2.0 * M * W.K * W.N, st);
    (void)dz_qmv1i_launch(a, W.bits, pl.G, pl.smem, st);
    return true;
}

// The stream-K matvec for M <= 2 (dz_qmv1_kernel). False when its shared
// memory does not fit (very wide matrices); the caller then uses the
// round-based streaming kernel.
static bool qmv1_launch(const DevQMat& W, const float* X, long long ldx, int M, const QmvEpilogue& ep,
                        cudaStream_t st, const uint32_t* XF, const int* shift, unsigned xf_bytes, int* status,
                        double qmv_bytes) {
    constexpr int WP = QMV1_WARPS;
    Qmv1Args a;
    memset(&a, 0, sizeof(a));
    a.codes = W.codes;
    a.N = W.N;
    a.nkg = W.nkg;
    a.ntiles = W.ntiles;
    a.X = X;
    a.ldx = ldx;
    a.k_scale = W.k_scale;
    a.K = W.K;
    a.XF = XF;
    a.row_shift = shift;
    a.M = M;
    a.xf_bytes = xf_bytes;
    a.status = status;
    a.ep = ep;
    a.ep.row_shift = nullptr;
    const int G = std::min(g_num_sms, W.ntiles);
    a.max_tiles = (W.ntiles + G - 1) / G;
    // a tile meets at most (nkg - 2) / shortest range + 2 non-empty warp ranges
    const long long per_min = (long long)(W.ntiles / G) * W.nkg / WP;
    a.max_parts = per_min >= 1 ? (int)std::min<long long>(WP, std::max<long long>(1, (W.nkg - 2) / per_min + 2)) : WP;
    const size_t fixed = dz_qmv1_smem_bytes(0, WP, xf_bytes, a.max_tiles, a.max_parts);
    if (fixed + (size_t)WP * QMS_STAGES * 512 > (size_t)g_smem_optin) return false;
    a.pk = (int)std::min<size_t>(16, ((size_t)g_smem_optin - fixed) / ((size_t)WP * QMS_STAGES * 512));
    const size_t smem = dz_qmv1_smem_bytes(a.pk, WP, xf_bytes, a.max_tiles, a.max_parts);
    ProfScope prof(DZ_KERNEL_QMV, qmv_bytes, 2.0 * M * W.K * W.N, st);
    // programmatic dependent launch: weight streaming may start while the
    // previous kernel in the stream drains (the kernel waits for it before
    // touching activations or outputs)
    cudaLaunchConfig_t cfg;
    memset(&cfg, 0, sizeof(cfg));
    cfg.gridDim = dim3((unsigned)G);
    cfg.blockDim = dim3(WP * 32);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    void (*k)(Qmv1Args) = W.bits == 8 ? (xf_bytes ? dz_qmv1_kernel<8, WP, true> : dz_qmv1_kernel<8, WP, false>)
                                      : (xf_bytes ? dz_qmv1_kernel<4, WP, true> : dz_qmv1_kernel<4, WP, false>);
    if (cudaLaunchKernelEx(&cfg, k, a) != cudaSuccess) {
        (void)cudaGetLastError();
        k<<<G, WP * 32, smem, st>>>(a);
    }
    return true;
}

// Y = epilogue(X . deq(W)) for M rows on the tensor cores. Up to
// QMS_MAX_M rows whose B fragments fit QMS_XF_SMEM_MAX: one streaming kernel
// that splits the activations itself. Otherwise the activation split into
// `scratch` (qmv_scratch_bytes), then the streaming (M <= QMS_MAX_M) or the
// register-blocked MMA kernel. A bulk-copy wait that gives up sets *status
// (when given) and leaves NaN in the tile. Returns the launches (1 or 2).

// The tensor-core GEMV takes M <= 16 rows where it measured faster than the
// CUDA-core matvec kernels (B200, K x N from 2048 x 2048 to 4096 x 32000):
// from 8 rows on every matrix of at least 2^20 codes, from 3 rows on matrices
// of at least 2^25 codes. Below that the matvec kernels' lower fixed cost wins.
constexpr size_t UGEMV_MIN_WEIGHTS = (size_t)1 << 20;
constexpr size_t UGEMV_LARGE_WEIGHTS = (size_t)1 << 25;
static bool use_ugemv(const DevQMat& W, int M) {
    const size_t kn = (size_t)W.K * W.N;
    if (!W.kn || kn < UGEMV_MIN_WEIGHTS || M > UV_N || (W.N + UG_BN - 1) / UG_BN > UGEMV_MAX_TILES) return false;
    return M >= 8 || (M >= 3 && kn >= UGEMV_LARGE_WEIGHTS);
}

// Rows and matrix size from which products go to the tensor-core GEMM.
constexpr int UGEMM_MIN_M = QMS_MAX_M + 1;
constexpr size_t UGEMM_MIN_WEIGHTS = (size_t)1 << 20;

// The tensor-core GEMM (umma.cuh): limb split, then one CTA per 128 x 128
// output tile. Returns the launches (2), or 0 when its TMA map cannot be made.
static int launch_ugemm(const DevQMat& W, const float* X, long long ldx, int M, const QmvEpilogue& ep_in,
                        cudaStream_t st, void* scratch, int* counters, int* status, bool limbs_ready = false) {
    const int Kp = round_up(W.K, UG_BK);
    int8_t* L = static_cast<int8_t*>(scratch);
    int* shift = reinterpret_cast<int*>(static_cast<uint8_t*>(scratch) + r256(3 * (size_t)M * Kp));
    const int parts = ugemm_kparts(W, M);
    long long* partial = parts > 1 ? reinterpret_cast<long long*>(static_cast<uint8_t*>(scratch) +
                                                                   r256(3 * (size_t)M * Kp) + r256((size_t)M * 4))
                                   : nullptr;
    CUtensorMap tmA;
    const cuuint64_t dims[3] = {(cuuint64_t)Kp, (cuuint64_t)M, (cuuint64_t)UG_LIMBS};
    const cuuint64_t strides[2] = {(cuuint64_t)Kp, (cuuint64_t)Kp * M};
    const cuuint32_t box[3] = {UG_BK, UG_BM, 1};
    if (!encode_u8_map(&tmA, L, 3, dims, strides, box)) return 0;
    // the split and the GEMM are programmatic dependents of the kernels
    // before them (each waits, griddepcontrol.wait, before it reads what they
    // wrote or writes what they read), so launch latency and the GEMM's
    // prologue and first weight loads overlap the kernel ahead
    cudaLaunchAttribute pdl[1];
    pdl[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    pdl[0].val.programmaticStreamSerializationAllowed = 1;
    if (!limbs_ready) {   // (else the norm before wrote the limbs and shifts: dz_layernorm_limbs_kernel)
        ProfScope prof(DZ_KERNEL_SPLIT, 4.0 * M * W.K + 3.0 * M * Kp, 0, st);
        // a warp per row from one wave of rows on (fewer block barriers per byte)
        const bool warp_rows = M >= 2 * g_num_sms;
        cudaLaunchConfig_t sc;
        memset(&sc, 0, sizeof(sc));
        sc.gridDim = dim3(warp_rows ? (unsigned)((M + UG_SPLIT_WARP_ROWS - 1) / UG_SPLIT_WARP_ROWS) : (unsigned)M);
        sc.blockDim = dim3(256);
        sc.stream = st;
        sc.attrs = pdl;
        sc.numAttrs = 1;
        if (cudaLaunchKernelEx(&sc, warp_rows ? dz_limb_split_warp_kernel : dz_limb_split_kernel, X, ldx, W.k_scale,
                               M, W.K, Kp, L, shift) != cudaSuccess) {
            (void)cudaGetLastError();
            if (warp_rows)
                dz_limb_split_warp_kernel<<<sc.gridDim, 256, 0, st>>>(X, ldx, W.k_scale, M, W.K, Kp, L, shift);
            else
                dz_limb_split_kernel<<<sc.gridDim, 256, 0, st>>>(X, ldx, W.k_scale, M, W.K, Kp, L, shift);
        }
    }
    UgArgs a;
    memset(&a, 0, sizeof(a));
    a.M = M;
    a.N = W.N;
    a.K = W.K;
    a.nkb = Kp / UG_BK;
    a.shift = shift;
    a.status = status;
    a.ep = ep_in;
    a.ep.row_shift = nullptr;
    a.kparts = parts;
    a.partial = partial;
    a.counters = counters;
    const dim3 grid((unsigned)((W.N + UG_BN - 1) / UG_BN), (unsigned)((M + UG_BM - 1) / UG_BM), (unsigned)parts);
    ProfScope prof(DZ_KERNEL_QMV,
                   (double)W.K * W.N + (double)W.scale_bytes + 4.0 * M * W.K + 4.0 * M * W.N,
                   2.0 * M * W.K * W.N, st);
    cudaLaunchConfig_t cfg;
    memset(&cfg, 0, sizeof(cfg));
    cfg.gridDim = grid;
    cfg.blockDim = dim3(UG_THREADS);
    cfg.dynamicSmemBytes = UG_SMEM_BYTES;
    cfg.stream = st;
    cfg.attrs = pdl;
    cfg.numAttrs = 1;
    if (cudaLaunchKernelEx(&cfg, dz_ugemm_kernel, tmA, W.tm_kn, a) != cudaSuccess) {
        (void)cudaGetLastError();
        dz_ugemm_kernel<<<grid, UG_THREADS, UG_SMEM_BYTES, st>>>(tmA, W.tm_kn, a);
    }
    return limbs_ready ? 1 : 2;
}

// The tensor-core GEMV for M <= 16 (umma.cuh): chunked limb split, then the
// stream-K kernel on ugemv_grid CTAs. Returns the launches (2), or 0 when its
// TMA map cannot be made.
static int launch_ugemv(const DevQMat& W, const float* X, long long ldx, int M, const QmvEpilogue& ep_in,
                        cudaStream_t st, void* scratch, int* counter, int* status) {
    const int Kp = round_up(W.K, UG_BK);
    const int nch = (Kp + UG_SPLIT_CHUNK - 1) / UG_SPLIT_CHUNK;
    const int ntiles = (W.N + UG_BN - 1) / UG_BN;
    uint8_t* p = static_cast<uint8_t*>(scratch);
    int8_t* L = reinterpret_cast<int8_t*>(p);
    p += r256(3 * (size_t)M * Kp);
    int* shift = reinterpret_cast<int*>(p);
    p += r256((size_t)M * 4);
    long long* partial = reinterpret_cast<long long*>(p);
    CUtensorMap tmL;
    const cuuint64_t dims[3] = {(cuuint64_t)Kp, (cuuint64_t)M, (cuuint64_t)UG_LIMBS};
    const cuuint64_t strides[2] = {(cuuint64_t)Kp, (cuuint64_t)Kp * M};
    const cuuint32_t box[3] = {UG_BK, UV_N, 1};
    if (!encode_u8_map(&tmL, L, 3, dims, strides, box)) return 0;
    {
        ProfScope prof(DZ_KERNEL_SPLIT, 4.0 * M * W.K * nch + 3.0 * M * Kp, 0, st);
        // programmatic dependent of the previous kernel: its blocks wait
        // (griddepcontrol.wait) before reading X or writing the limbs
        cudaLaunchConfig_t sc;
        memset(&sc, 0, sizeof(sc));
        sc.gridDim = dim3((unsigned)nch, (unsigned)M);
        sc.blockDim = dim3(256);
        sc.stream = st;
        cudaLaunchAttribute sa[1];
        sa[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        sa[0].val.programmaticStreamSerializationAllowed = 1;
        sc.attrs = sa;
        sc.numAttrs = 1;
        if (cudaLaunchKernelEx(&sc, dz_limb_split_chunk_kernel, X, ldx, W.k_scale, M, W.K, Kp, L, shift) !=
            cudaSuccess) {
            (void)cudaGetLastError();
            dz_limb_split_chunk_kernel<<<sc.gridDim, 256, 0, st>>>(X, ldx, W.k_scale, M, W.K, Kp, L, shift);
        }
    }
    UvArgs a;
    memset(&a, 0, sizeof(a));
    a.M = M;
    a.N = W.N;
    a.K = W.K;
    a.nkb = Kp / UG_BK;
    a.ntiles = ntiles;
    a.total = (long long)ntiles * a.nkb;
    a.shift = shift;
    a.partial = partial;
    a.counter = counter;
    a.status = status;
    a.ep = ep_in;
    a.ep.row_shift = nullptr;
    ProfScope prof(DZ_KERNEL_QMV, (double)W.K * W.N + (double)W.scale_bytes + 4.0 * M * W.K + 4.0 * M * W.N,
                   2.0 * M * W.K * W.N, st);
    // programmatic dependent of the split: weight streaming starts before the
    // split grid completes (the kernel waits for it before reading limbs)
    cudaLaunchConfig_t cfg;
    memset(&cfg, 0, sizeof(cfg));
    cfg.gridDim = dim3((unsigned)ugemv_grid(W));
    cfg.blockDim = dim3(UG_THREADS);
    cfg.dynamicSmemBytes = UV_SMEM_BYTES;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaLaunchKernelEx(&cfg, dz_ugemv_kernel, W.tm_kn, tmL, a) != cudaSuccess) {
        (void)cudaGetLastError();
        dz_ugemv_kernel<<<cfg.gridDim, UG_THREADS, UV_SMEM_BYTES, st>>>(W.tm_kn, tmL, a);
    }
    return 2;
}

// limbs_ready: the norm before wrote this product's limbs and shifts into
// the scratch (launch_norm_limbs), used when the product runs on the GEMM.
static int launch_qmv(const DevQMat& W, const float* X, long long ldx, int M, const QmvEpilogue& ep_in,
                      cudaStream_t st, void* scratch, int* status, bool limbs_ready = false) {
    int* counters = static_cast<int*>(scratch);
    scratch = static_cast<uint8_t*>(scratch) + SCRATCH_COUNTERS;
    if (M <= UV_N && use_ugemv(W, M)) {
        const int n = launch_ugemv(W, X, ldx, M, ep_in, st, scratch, counters, status);
        if (n) return n;
    }
    // small matrices stay on the register-blocked kernel: the GEMM's fixed
    // cost per tile (pipeline fill, tensor-memory drain) would dominate
    if (M >= UGEMM_MIN_M && W.kn && (size_t)W.K * W.N >= UGEMM_MIN_WEIGHTS) {
        const int n = launch_ugemm(W, X, ldx, M, ep_in, st, scratch, counters, status, limbs_ready);
        if (n) return n;
    }
    const int KG = W.bits == 8 ? 32 : 64;
    const int KT = KG / 16;
    const int Kp = W.nkg * KG;
    const int nbt = (M + 1) / 2;
    uint32_t* XF = static_cast<uint32_t*>(scratch);
    int* shift = reinterpret_cast<int*>(static_cast<uint8_t*>(scratch) + r256(qmv_xf_bytes(W, M)));
    const size_t xf = qmv_xf_bytes(W, M);
    bool xin = M <= QMS_MAX_M && xf <= QMS_XF_SMEM_MAX;
    if (xin) {   // the in-kernel split holds QMS_XIN_PAIRS element pairs per thread
        int NB, NT, WP;
        qms_shape(M, &NB, &NT, &WP);
        xin = (long long)Kp / 2 <= (long long)QMS_XIN_PAIRS * WP * 32;
    }
    if (M <= 2 &&
        qmv1i_launch(W, X, ldx, M, ep_in, st, status,
                     (double)W.K * W.N * W.bits / 8 + (double)W.scale_bytes + 4.0 * M * W.K + 4.0 * M * W.N))
        return 1;
    int launches = 1;
    if (!xin) {
        ProfScope prof(DZ_KERNEL_SPLIT, 4.0 * M * W.K + 16.0 * nbt * Kp, 0, st);
        const dim3 grid((unsigned)((Kp / 2 + DZ_SPLIT_PAIRS - 1) / DZ_SPLIT_PAIRS), (unsigned)M);
        if (KT == 2) dz_split_rows_kernel<2><<<grid, 256, 0, st>>>(X, ldx, W.k_scale, M, W.K, W.nkg, nbt, XF, shift);
        else dz_split_rows_kernel<4><<<grid, 256, 0, st>>>(X, ldx, W.k_scale, M, W.K, W.nkg, nbt, XF, shift);
        launches++;
    }
    QmvEpilogue ep = ep_in;
    ep.row_shift = shift;
    const double qmv_bytes = (double)W.K * W.N * W.bits / 8 + (double)W.scale_bytes + 4.0 * M * W.K + 4.0 * M * W.N;
    if (M <= 2 && qmv1_launch(W, X, ldx, M, ep_in, st, XF, shift, xin ? (unsigned)xf : 0u, status, qmv_bytes))
        return launches;
    if (M <= QMS_MAX_M) {
        int NB, NT, WP;
        qms_shape(M, &NB, &NT, &WP);
        QmsArgs a;
        memset(&a, 0, sizeof(a));
        a.codes = W.codes;
        a.N = W.N;
        a.nkg = W.nkg;
        a.ntiles = W.ntiles;
        a.X = X;
        a.ldx = ldx;
        a.k_scale = W.k_scale;
        a.K = W.K;
        a.XF = XF;
        a.row_shift = shift;
        a.nbt = nbt;
        a.M = M;
        a.status = status;
        a.ep = ep_in;
        a.ep.row_shift = nullptr;
        a.n_groups = (W.ntiles + NT - 1) / NT;
        unsigned grid = 1;
        a.kparts = qms_kparts(a.n_groups, W.nkg, WP, &a.nrounds, &grid);
        a.per = (W.nkg + a.kparts - 1) / a.kparts;
        a.xf_bytes = xin ? (unsigned)xf : 0u;
        const size_t fixed = dz_qms_smem_bytes(0, NT, NB, WP, a.xf_bytes);
        const int pk_budget = (int)(((size_t)g_smem_optin - fixed) / ((size_t)WP * QMS_STAGES * NT * 512));
        a.pk = std::max(1, std::min(16 / NT, pk_budget));
        a.pk = std::min(a.pk, std::max(1, a.per));
        const size_t smem = dz_qms_smem_bytes(a.pk, NT, NB, WP, a.xf_bytes);
        ProfScope prof(DZ_KERNEL_QMV, qmv_bytes, 2.0 * M * W.K * W.N, st);
        if (W.bits == 8) {
            if (xin) launch_qms_bits<8, true>(a, NB, grid, smem, st);
            else launch_qms_bits<8, false>(a, NB, grid, smem, st);
        } else {
            if (xin) launch_qms_bits<4, true>(a, NB, grid, smem, st);
            else launch_qms_bits<4, false>(a, NB, grid, smem, st);
        }
        return launches;
    }
    QmmArgs a;
    a.codes = W.codes;
    a.K = W.K;
    a.N = W.N;
    a.nkg = W.nkg;
    a.ntiles = W.ntiles;
    a.XF = XF;
    a.nbt = nbt;
    a.M = M;
    a.ep = ep;
    const int NB = M <= 2 ? 1 : M <= 4 ? 2 : M <= 8 ? 4 : 8;
    const int NT = NB == 1 ? 4 : NB == 8 ? 1 : 2;
    a.m_passes = (M + 2 * NB - 1) / (2 * NB);
    a.n_groups = (W.ntiles + NT - 1) / NT;
    const long long units = (long long)a.n_groups * a.m_passes;
    const long long target = (long long)g_num_sms * 32;
    int kp = 1;
    while (kp < QMV_WARPS && units * kp * 2 <= target && W.nkg / (kp * 2) >= 2) kp *= 2;
    a.kparts = kp;
    a.kg_per_part = (W.nkg + kp - 1) / kp;
    const int units_per_cta = QMV_WARPS / kp;
    const unsigned grid = (unsigned)((units + units_per_cta - 1) / units_per_cta);
    ProfScope prof(DZ_KERNEL_QMV, qmv_bytes, 2.0 * M * W.K * W.N, st);
    if (W.bits == 8) launch_qmm_bits<8>(a, NB, grid, st);
    else launch_qmm_bits<4>(a, NB, grid, st);
    return launches;
}

// The launches launch_qmv makes for this matrix at M rows (mirrors its choices).
static int qmv_launches(const DevQMat& W, int M) {
    if (M >= UGEMM_MIN_M && W.kn && (size_t)W.K * W.N >= UGEMM_MIN_WEIGHTS) return 2;
    if (M <= UV_N && use_ugemv(W, M)) return 2;
    Qmv1iPlan pl;
    if (qmv1i_plan(W, M, &pl)) return 1;
    const int KG = W.bits == 8 ? 32 : 64;
    const int Kp = W.nkg * KG;
    bool xin = M <= QMS_MAX_M && qmv_xf_bytes(W, M) <= QMS_XF_SMEM_MAX;
    if (xin) {
        int NB, NT, WP;
        qms_shape(M, &NB, &NT, &WP);
        xin = (long long)Kp / 2 <= (long long)QMS_XIN_PAIRS * WP * 32;
    }
    return xin ? 1 : 2;
}

static QmvEpilogue plain_epilogue(const DevQMat& W, float* Y, long long ldy) {
    QmvEpilogue e;
    memset(&e, 0, sizeof(e));
    e.col_scale = W.col_scale;
    e.nseg = 1;
    e.seg_start[0] = 0;
    e.seg_start[1] = W.N;
    e.seg_ptr[0] = Y;
    e.seg_ld[0] = ldy;
    return e;
}

// ------------------------------------------------------------- qmatrix API

struct dz_cuda_qmatrix {
    int device;
    DevQMat m;
    cudaStream_t stream;
    void* scratch = nullptr;            // split activations, grown to the largest M used
    size_t scratch_bytes = 0;
    int* status = nullptr;              // device word: a weight-copy wait gave up
};

static int qmatrix_scratch(dz_cuda_qmatrix_t* q, int M) {
    const size_t need = qmv_scratch_bytes(q->m, M);
    if (need <= q->scratch_bytes) return DZ_OK;
    cudaFree(q->scratch);
    q->scratch = nullptr;
    q->scratch_bytes = 0;
    DZ_CUDA(cudaMalloc(&q->scratch, need));
    DZ_CUDA(cudaMemset(q->scratch, 0, need));   // the GEMV's per-tile counters start at zero
    q->scratch_bytes = need;
    return DZ_OK;
}

extern "C" int dz_cuda_qmatrix_create(int device, const dz_tensor_blob_t* w, dz_cuda_qmatrix_t** out) {
    if (!out) return fail(DZ_E_INVALID, "null output handle");
    *out = nullptr;
    DeviceGuard g(device);
    if (!g.ok) return fail(DZ_E_DEVICE, "cannot select device %d", device);
    cudaDeviceGetAttribute(&g_num_sms, cudaDevAttrMultiProcessorCount, device);
    auto* q = new (std::nothrow) dz_cuda_qmatrix;
    if (!q) return fail(DZ_E_NOMEM, "host allocation");
    q->device = device;
    if (cudaStreamCreateWithFlags(&q->stream, cudaStreamNonBlocking) != cudaSuccess) {
        delete q;
        return fail(DZ_E_DEVICE, "stream creation failed");
    }
    int rc = qms_prepare(device);
    if (!rc) rc = make_qmat({w}, q->stream, &q->m);
    if (!rc && cudaMalloc(&q->status, 4) != cudaSuccess) rc = fail(DZ_E_NOMEM, "device allocation");
    if (!rc && cudaMemsetAsync(q->status, 0, 4, q->stream) != cudaSuccess) rc = fail(DZ_E_DEVICE, "memset");
    if (rc) {
        free_qmat(q->m);
        cudaFree(q->status);
        cudaStreamDestroy(q->stream);
        delete q;
        return rc;
    }
    *out = q;
    return DZ_OK;
}

extern "C" void dz_cuda_qmatrix_free(dz_cuda_qmatrix_t* q) {
    if (!q) return;
    DeviceGuard g(q->device);
    free_qmat(q->m);
    cudaFree(q->scratch);
    cudaFree(q->status);
    cudaStreamDestroy(q->stream);
    delete q;
}

extern "C" size_t dz_cuda_qmatrix_bytes(const dz_cuda_qmatrix_t* q) {
    if (!q) return 0;
    return (size_t)q->m.K * q->m.N * q->m.bits / 8 + q->m.scale_bytes;
}

extern "C" int dz_cuda_qmatrix_unpack(const dz_cuda_qmatrix_t* q, float* dst) {
    if (!q || !dst) return fail(DZ_E_INVALID, "null argument");
    DeviceGuard g(q->device);
    const long long total = (long long)q->m.K * q->m.N;
    float* d = nullptr;
    DZ_CUDA(cudaMalloc(&d, total * 4));
    const float* scales = q->m.gran == DZ_GRAN_ROW ? q->m.k_scale : q->m.col_scale;
    int gran = q->m.gran == DZ_GRAN_TENSOR ? DZ_GRAN_COLUMN : q->m.gran;  // expanded per column
    dz_frag_dequant_kernel<<<(unsigned)((total + 255) / 256), 256, 0, q->stream>>>(q->m.codes, scales, gran, d,
                                                                                q->m.K, q->m.N, q->m.bits, q->m.nkg);
    cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess) e = cudaMemcpyAsync(dst, d, total * 4, cudaMemcpyDeviceToHost, q->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(q->stream);
    cudaFree(d);
    if (e != cudaSuccess) return fail(DZ_E_DEVICE, "unpack: %s", cudaGetErrorString(e));
    return DZ_OK;
}

extern "C" int dz_cuda_qmatrix_codes(const dz_cuda_qmatrix_t* q, uint8_t* packed) {
    if (!q || !packed) return fail(DZ_E_INVALID, "null argument");
    DeviceGuard g(q->device);
    size_t nb = 0;
    dz_quantized_packed_size((size_t)q->m.K * q->m.N, q->m.bits, &nb);
    uint8_t* d = nullptr;
    DZ_CUDA(cudaMalloc(&d, nb));
    dz_frag_unrepack_kernel<<<(unsigned)((nb + 255) / 256), 256, 0, q->stream>>>(q->m.codes, d, q->m.K, q->m.N,
                                                                             q->m.bits, q->m.nkg, (long long)nb);
    cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess) e = cudaMemcpyAsync(packed, d, nb, cudaMemcpyDeviceToHost, q->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(q->stream);
    cudaFree(d);
    if (e != cudaSuccess) return fail(DZ_E_DEVICE, "codes: %s", cudaGetErrorString(e));
    return DZ_OK;
}

extern "C" int dz_cuda_matmul_quantized_async(const float* A, const dz_cuda_qmatrix_t* q, float* C, size_t m,
                                              size_t k, void* stream) {
    if (!q || !A || !C || m == 0 || k != (size_t)q->m.K || m > (1u << 24))
        return fail(DZ_E_INVALID, "matmul_quantized: bad arguments (k must equal the matrix rows)");
    DeviceGuard g(q->device);
    // the scratch grows outside any stream work; a caller capturing this into a
    // graph makes one uncaptured call with its largest m first
    int rc = qmatrix_scratch(const_cast<dz_cuda_qmatrix_t*>(q), (int)m);
    if (rc) return rc;
    QmvEpilogue ep = plain_epilogue(q->m, C, q->m.N);
    launch_qmv(q->m, A, (long long)k, (int)m, ep, (cudaStream_t)stream, q->scratch, q->status);
    DZ_CUDA(cudaGetLastError());
    return DZ_OK;
}

extern "C" int dz_cuda_matmul_quantized(const float* A, const dz_cuda_qmatrix_t* q, float* C, size_t m,
                                        size_t k) {
    if (!q || !A || !C || m == 0 || k != (size_t)q->m.K)
        return fail(DZ_E_INVALID, "matmul_quantized: bad arguments (k must equal the matrix rows)");
    DeviceGuard g(q->device);
    float *dA = nullptr, *dC = nullptr;
    const size_t n = (size_t)q->m.N;
    DZ_CUDA(cudaMalloc(&dA, m * k * 4));
    if (cudaMalloc(&dC, m * n * 4) != cudaSuccess) {
        cudaFree(dA);
        return fail(DZ_E_NOMEM, "device allocation");
    }
    cudaError_t e = cudaMemcpyAsync(dA, A, m * k * 4, cudaMemcpyHostToDevice, q->stream);
    int rc = DZ_OK;
    if (e == cudaSuccess) rc = dz_cuda_matmul_quantized_async(dA, q, dC, m, k, q->stream);
    int timed_out = 0;
    if (e == cudaSuccess && rc == DZ_OK) e = cudaMemcpyAsync(C, dC, m * n * 4, cudaMemcpyDeviceToHost, q->stream);
    if (e == cudaSuccess && rc == DZ_OK)
        e = cudaMemcpyAsync(&timed_out, q->status, 4, cudaMemcpyDeviceToHost, q->stream);
    if (e == cudaSuccess && rc == DZ_OK) e = cudaStreamSynchronize(q->stream);
    cudaFree(dA);
    cudaFree(dC);
    if (rc) return rc;
    if (e != cudaSuccess) return fail(DZ_E_DEVICE, "matmul_quantized: %s", cudaGetErrorString(e));
    if (timed_out) {
        cudaMemsetAsync(q->status, 0, 4, q->stream);
        return fail(DZ_E_TIMEOUT, "matmul_quantized: a weight copy did not arrive within 1 s");
    }
    return DZ_OK;
}

// ------------------------------------------------------------------ model

struct DevLayer {
    bool fused_qkv = false;
    // with SwiGLU, w1 is [W_ff1 | W_ff_gate] (2F columns), or W_ff1 alone and
    // wg the gate for ROW-granularity scales; b1 is then [b_ff1 | b_ff_gate]
    DevQMat qkv, q, k, v, wo, w1, wg, w2;
    float *g1 = nullptr, *be1 = nullptr, *b1 = nullptr, *b2 = nullptr, *g2 = nullptr, *be2 = nullptr;
};

// Architecture bits (src/include/core/model_types.h:26-36).
enum : uint32_t { ARCH_TIED = 1, ARCH_ROPE = 2, ARCH_RMSNORM = 4, ARCH_GELU = 8, ARCH_SWIGLU = 16 };

struct dz_cuda_model {
    int device = 0;
    dz_model_desc_t desc{};
    std::atomic<int> refs{1};
    float* emb = nullptr;
    float* out_bias = nullptr;
    float* pe = nullptr;
    long long pe_rows = 0;
    std::vector<DevLayer> layers;
    DevQMat head;                 // empty with tied embeddings (the head is emb^T, fp32)
    uint32_t flags = 0;
    bool tied = false, rope = false, rms = false, swiglu = false;
    int act = DZ_ACT_RELU;        // FFN activation (without SwiGLU)
    float* rope_tab = nullptr;    // [pe_rows][hd / 2][cos, sin]
    size_t step_bytes = 0;
    std::vector<void*> f32_allocs;
    // fused one-CTA-per-sequence generation (seqgen.cuh), when the model fits it
    bool seq_ok = false;
    int seq_bits = 0, seq_buf_bytes = 0;
    SeqLayer* seq_layers = nullptr;   // device array [L]
    SeqMat seq_head{};
    std::vector<void*> seq_blobs;
    // tensor parallelism over heads / FFN columns (1 rank: the whole model)
    int tp_rank = 0, tp_world = 1;
    int Hl = 0, dl = 0, Fl = 0;   // local heads, attention width Hl*hd, FFN width F/world
    ncclComm_t comm = nullptr;
};

// NCCL, loaded at run time (the copy the process already holds, else the
// system's libnccl.so.2), so the library has no link-time dependency on it.
struct NcclApi {
    ncclResult_t (*get_unique_id)(ncclUniqueId*);
    ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int);
    ncclResult_t (*all_reduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t, cudaStream_t);
    ncclResult_t (*comm_destroy)(ncclComm_t);
    const char* (*error_string)(ncclResult_t);
};
static const NcclApi* nccl_api() {
    static NcclApi api;
    static bool ok = false;
    static std::once_flag once;
    std::call_once(once, [] {
        void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
        if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) return;
        api.get_unique_id = reinterpret_cast<decltype(api.get_unique_id)>(dlsym(h, "ncclGetUniqueId"));
        api.comm_init_rank = reinterpret_cast<decltype(api.comm_init_rank)>(dlsym(h, "ncclCommInitRank"));
        api.all_reduce = reinterpret_cast<decltype(api.all_reduce)>(dlsym(h, "ncclAllReduce"));
        api.comm_destroy = reinterpret_cast<decltype(api.comm_destroy)>(dlsym(h, "ncclCommDestroy"));
        api.error_string = reinterpret_cast<decltype(api.error_string)>(dlsym(h, "ncclGetErrorString"));
        ok = api.get_unique_id && api.comm_init_rank && api.all_reduce && api.comm_destroy && api.error_string;
    });
    return ok ? &api : nullptr;
}

static void model_release(dz_cuda_model_t* m) {
    if (!m || --m->refs > 0) return;
    DeviceGuard g(m->device);
    if (m->comm && nccl_api()) nccl_api()->comm_destroy(m->comm);
    for (auto& L : m->layers) {
        free_qmat(L.qkv); free_qmat(L.q); free_qmat(L.k); free_qmat(L.v);
        free_qmat(L.wo); free_qmat(L.w1); free_qmat(L.wg); free_qmat(L.w2);
    }
    free_qmat(m->head);
    for (void* p : m->f32_allocs) cudaFree(p);
    cudaFree(m->seq_layers);
    for (void* b : m->seq_blobs) cudaFree(b);
    delete m;
}

static int upload_f32(dz_cuda_model_t* m, const dz_tensor_blob_t& t, size_t expect, float** out,
                      cudaStream_t st) {
    if (t.bits != 0 || !t.f32 || t.rows * t.cols != expect)
        return fail(DZ_E_UNSUPPORTED, "tensor expected as float32 (default quantization policy)");
    float* d = nullptr;
    DZ_CUDA(cudaMalloc(&d, expect * 4));
    m->f32_allocs.push_back(d);
    DZ_CUDA(cudaMemcpyAsync(d, t.f32, expect * 4, cudaMemcpyHostToDevice, st));
    *out = d;
    return DZ_OK;
}

constexpr int SEQ_SMEM_LIMIT = 232448;   // 227 KB of shared memory per block on sm_100
constexpr int SEQ_BUF_LIMIT = 96 * 1024;

// One fused-kernel blob: [codes | column scales (Np) | bias | gamma, beta], each
// section 16-byte aligned, assembled on the device from the model's arrays.
static bool seq_blob(dz_cuda_model_t* m, const DevQMat& q, const float* bias, int nbias, const float* gamma,
                     const float* beta, int D, SeqMat* out) {
    auto r16 = [](size_t n) { return (n + 15) & ~(size_t)15; };
    size_t off = r16(q.code_bytes);
    const size_t scale_off = off;
    off += r16((size_t)q.Np * 4);
    const size_t bias_off = bias ? off : 0;
    if (bias) off += r16((size_t)nbias * 4);
    const size_t gamma_off = gamma ? off : 0;
    if (gamma) off += r16((size_t)D * 4) * 2;
    uint8_t* blob = nullptr;
    if (cudaMalloc(&blob, off) != cudaSuccess) return false;
    m->seq_blobs.push_back(blob);
    bool ok = cudaMemcpy(blob, q.codes, q.code_bytes, cudaMemcpyDeviceToDevice) == cudaSuccess &&
              cudaMemcpy(blob + scale_off, q.col_scale, (size_t)q.Np * 4, cudaMemcpyDeviceToDevice) == cudaSuccess;
    if (ok && bias) ok = cudaMemcpy(blob + bias_off, bias, (size_t)nbias * 4, cudaMemcpyDeviceToDevice) == cudaSuccess;
    if (ok && gamma) {
        ok = cudaMemcpy(blob + gamma_off, gamma, (size_t)D * 4, cudaMemcpyDeviceToDevice) == cudaSuccess &&
             cudaMemcpy(blob + gamma_off + (size_t)D * 4, beta, (size_t)D * 4, cudaMemcpyDeviceToDevice) ==
                 cudaSuccess;
    }
    if (!ok) return false;
    out->blob = blob;
    out->K = q.K;
    out->N = q.N;
    out->nkg = q.nkg;
    out->ntiles = q.ntiles;
    out->bytes = (unsigned)off;
    out->scale_off = (unsigned)scale_off;
    out->bias_off = (unsigned)bias_off;
    out->gamma_off = (unsigned)gamma_off;
    return true;
}


// Shared-memory bytes of dz_seqgen_kernel (its carve-up in seqgen.cuh), with
// or without the per-layer K/V staging area.
static size_t seq_smem_bytes(const dz_cuda_model_t* m, int cap, bool kv_smem) {
    const size_t D = m->desc.embedding_dim, F = 4 * D, V = m->desc.vocab_size, H = m->desc.num_heads;
    size_t P = 1;
    while (P < V) P <<= 1;
    const size_t pv = V > (size_t)SEQ_THREADS ? V : (size_t)SEQ_THREADS;
    auto r4 = [](size_t n) { return (n + 3) & ~(size_t)3; };
    const size_t table = (sizeof(SeqLayer) * m->layers.size() + 15) & ~(size_t)15;
    const size_t xs_stride = (F + 63) / 64 * 64;
    return 2 * (size_t)m->seq_buf_bytes + 64 + table + 8 * (P > (size_t)SEQ_THREADS ? P : (size_t)SEQ_THREADS) +
           4 * (5 * r4(D) + r4(F) + 2 * r4(V) + r4(H * (size_t)cap) + 64 + 2 * r4(pv)) +
           (kv_smem ? 8 * r4((size_t)cap * D) : 0) + 2 * 4 * r4(3 * xs_stride / 2);
}

static bool seq_kv_smem(const dz_cuda_model_t* m, int cap) {
    return seq_smem_bytes(m, cap, true) <= (size_t)SEQ_SMEM_LIMIT;
}

static size_t seq_smem_for(const dz_cuda_model_t* m, int cap) {
    return seq_smem_bytes(m, cap, seq_kv_smem(m, cap));
}

// Decides whether the fused path can run this model and builds its blobs and
// layer table.
static void prepare_seqgen(dz_cuda_model_t* m) {
    m->seq_ok = false;
    if (m->flags) return;   // the fused kernel runs the default architecture
    if (m->layers.empty() || m->desc.embedding_dim % 4 != 0) return;  // 16-byte aligned activations
    // the fused attention keeps a head's output in four registers per lane
    if (m->desc.num_heads == 0 || m->desc.embedding_dim / m->desc.num_heads > 128) return;
    const int bits = m->head.bits;
    if (bits != 4 && bits != 8 || m->head.k_scale) return;
    for (auto& L : m->layers) {
        if (!L.fused_qkv || L.qkv.k_scale || L.wo.k_scale || L.w1.k_scale || L.w2.k_scale) return;
        for (const DevQMat* q : {&L.qkv, &L.wo, &L.w1, &L.w2})
            if (q->bits != bits) return;
    }
    const int D = (int)m->desc.embedding_dim, F = 4 * D, V = (int)m->desc.vocab_size;
    std::vector<SeqLayer> host(m->layers.size());
    size_t buf = 0;
    bool ok = true;
    for (size_t l = 0; l < m->layers.size() && ok; l++) {
        const DevLayer& L = m->layers[l];
        ok = seq_blob(m, L.qkv, nullptr, 0, nullptr, nullptr, D, &host[l].qkv) &&
             seq_blob(m, L.wo, nullptr, 0, L.g1, L.be1, D, &host[l].wo) &&
             seq_blob(m, L.w1, L.b1, F, nullptr, nullptr, D, &host[l].w1) &&
             seq_blob(m, L.w2, L.b2, D, L.g2, L.be2, D, &host[l].w2);
        for (const SeqMat* q : {&host[l].qkv, &host[l].wo, &host[l].w1, &host[l].w2})
            buf = q->bytes > buf ? q->bytes : buf;
    }
    ok = ok && seq_blob(m, m->head, m->out_bias, V, nullptr, nullptr, D, &m->seq_head);
    if (ok) buf = m->seq_head.bytes > buf ? m->seq_head.bytes : buf;
    if (ok && buf <= (size_t)SEQ_BUF_LIMIT && cudaMalloc(&m->seq_layers, host.size() * sizeof(SeqLayer)) == cudaSuccess) {
        ok = cudaMemcpy(m->seq_layers, host.data(), host.size() * sizeof(SeqLayer), cudaMemcpyHostToDevice) ==
             cudaSuccess;
    } else {
        ok = false;
    }
    if (!ok) {
        cudaGetLastError();
        for (void* b : m->seq_blobs) cudaFree(b);
        m->seq_blobs.clear();
        cudaFree(m->seq_layers);
        m->seq_layers = nullptr;
        return;
    }
    m->seq_bits = bits;
    m->seq_buf_bytes = (int)buf;
    m->seq_ok = true;
}

// A quantized projection blob owned by the host while a shard is built.
struct SliceBlob {
    dz_tensor_blob_t blob;
    std::vector<float> scales;
    std::vector<uint8_t> packed;
};

// Rows (axis 0) or columns (axis 1) [start, start + count) of a projection blob.
static int slice_blob(const dz_tensor_blob_t& t, int axis, size_t start, size_t count, SliceBlob* out) {
    const size_t r2 = axis == 0 ? count : t.rows, c2 = axis == 0 ? t.cols : count;
    size_t ns = 0, nb = 0;
    dz_quantized_scale_count(r2, c2, t.granularity, &ns);
    dz_quantized_packed_size(r2 * c2, t.bits, &nb);
    out->scales.resize(ns);
    out->packed.resize(nb);
    if (dz_quantized_slice(t.scales, t.scale_count, t.packed, t.packed_size, t.rows, t.cols, t.bits,
                           t.granularity, axis, start, count, out->scales.data(), out->packed.data()) != DZ_OK)
        return fail(DZ_E_INVALID, "tensor-parallel slice of a %zux%zu projection", t.rows, t.cols);
    out->blob = t;
    out->blob.rows = r2;
    out->blob.cols = c2;
    out->blob.scales = out->scales.data();
    out->blob.scale_count = ns;
    out->blob.packed = out->packed.data();
    out->blob.packed_size = nb;
    return DZ_OK;
}

static int build_model(const dz_model_desc_t* desc, const dz_tensor_blob_t* tensors, size_t n, int device,
                       int tp_rank, int tp_world, ncclComm_t comm, dz_cuda_model_t** out);

extern "C" int dz_cuda_model_create(const dz_model_desc_t* desc, const dz_tensor_blob_t* tensors, size_t n,
                                    int device, dz_cuda_model_t** out) {
    return build_model(desc, tensors, n, device, 0, 1, nullptr, out);
}

extern "C" int dz_cuda_tp_unique_id(uint8_t* id) {
    if (!id) return fail(DZ_E_INVALID, "null id buffer");
    const NcclApi* api = nccl_api();
    if (!api) return fail(DZ_E_UNSUPPORTED, "NCCL (libnccl.so.2) not found");
    ncclUniqueId u;
    ncclResult_t r = api->get_unique_id(&u);
    if (r != ncclSuccess) return fail(DZ_E_DEVICE, "ncclGetUniqueId: %s", api->error_string(r));
    static_assert(sizeof(ncclUniqueId) == DZ_TP_ID_BYTES, "NCCL unique id size");
    memcpy(id, &u, sizeof(u));
    return DZ_OK;
}

extern "C" int dz_cuda_model_create_tp(const dz_model_desc_t* desc, const dz_tensor_blob_t* tensors, size_t n,
                                       int device, int tp_rank, int tp_world, const uint8_t* id,
                                       dz_cuda_model_t** out) {
    if (!out) return fail(DZ_E_INVALID, "null output handle");
    *out = nullptr;
    if (!desc || tp_world < 1 || tp_rank < 0 || tp_rank >= tp_world || (tp_world > 1 && !id))
        return fail(DZ_E_INVALID, "tensor-parallel rank %d of %d", tp_rank, tp_world);
    if (desc->num_heads % (size_t)tp_world || (4 * desc->embedding_dim) % (size_t)tp_world)
        return fail(DZ_E_INVALID, "heads and FFN width must divide by the %d ranks", tp_world);
    if (tp_world == 1) return build_model(desc, tensors, n, device, 0, 1, nullptr, out);
    const NcclApi* api = nccl_api();
    if (!api) return fail(DZ_E_UNSUPPORTED, "NCCL (libnccl.so.2) not found");
    ncclComm_t comm = nullptr;
    {
        DeviceGuard g(device);
        if (!g.ok) return fail(DZ_E_DEVICE, "cannot select device %d", device);
        ncclUniqueId u;
        memcpy(&u, id, sizeof(u));
        ncclResult_t r = api->comm_init_rank(&comm, tp_world, u, tp_rank);
        if (r != ncclSuccess) return fail(DZ_E_DEVICE, "ncclCommInitRank: %s", api->error_string(r));
    }
    int rc = build_model(desc, tensors, n, device, tp_rank, tp_world, comm, out);
    if (rc) {
        DeviceGuard g(device);
        api->comm_destroy(comm);
    }
    return rc;
}

static int build_model(const dz_model_desc_t* desc, const dz_tensor_blob_t* tensors, size_t n, int device,
                       int tp_rank, int tp_world, ncclComm_t comm, dz_cuda_model_t** out) {
    if (!out) return fail(DZ_E_INVALID, "null output handle");
    *out = nullptr;
    if (!desc || !tensors) return fail(DZ_E_INVALID, "null argument");
    const uint32_t flags = desc->architecture_flags;
    const size_t D = desc->embedding_dim, V = desc->vocab_size, H = desc->num_heads, F = 4 * D;
    if (D == 0 || H == 0 || D % H || V == 0 || desc->num_layers == 0 || desc->max_seq_len == 0)
        return fail(DZ_E_INVALID, "bad model shape");
    if (flags && tp_world > 1)
        return fail(DZ_E_UNSUPPORTED, "tensor parallelism runs the default architecture only (flags 0x%x)", flags);
    if ((flags & ARCH_ROPE) && ((D / H) % 2))
        return fail(DZ_E_INVALID, "RoPE needs an even head dimension");
    if (n != dz_model_tensor_layout(desc, nullptr, 0))
        return fail(DZ_E_INVALID, "tensor count %zu does not match the model", n);
    std::vector<dz_tensor_blob_t> lay(n);
    dz_model_tensor_layout(desc, lay.data(), n);
    for (size_t i = 0; i < n; i++) {
        if (tensors[i].kind != lay[i].kind || tensors[i].rows != lay[i].rows || tensors[i].cols != lay[i].cols)
            return fail(DZ_E_INVALID, "tensor %zu kind/shape mismatch", i);
        if (lay[i].kind == DZ_KIND_PROJECTION && tensors[i].bits == 0)
            return fail(DZ_E_UNSUPPORTED, "float32 projection %zu: use the CPU path", i);
    }
    DeviceGuard g(device);
    if (!g.ok) return fail(DZ_E_DEVICE, "cannot select device %d", device);
    cudaDeviceGetAttribute(&g_num_sms, cudaDevAttrMultiProcessorCount, device);
    if (int rc0 = qms_prepare(device)) return rc0;
    auto* m = new (std::nothrow) dz_cuda_model;
    if (!m) return fail(DZ_E_NOMEM, "host allocation");
    m->device = device;
    m->desc = *desc;
    m->tp_rank = tp_rank;
    m->tp_world = tp_world;
    m->Hl = (int)(H / tp_world);
    m->dl = (int)(D / tp_world);
    m->Fl = (int)(F / tp_world);
    m->flags = flags;
    m->tied = (flags & ARCH_TIED) != 0;
    m->rope = (flags & ARCH_ROPE) != 0;
    m->rms = (flags & ARCH_RMSNORM) != 0;
    m->swiglu = (flags & ARCH_SWIGLU) != 0;
    m->act = (flags & ARCH_GELU) ? DZ_ACT_GELU : DZ_ACT_RELU;
    cudaStream_t st;
    if (cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking) != cudaSuccess) {
        delete m;
        return fail(DZ_E_DEVICE, "stream creation failed");
    }
    int rc = DZ_OK;
    size_t step = 0;
    do {
        // tensors in model_param_tensors order for the architecture bits
        // (src/core/model_params.c:39-103)
        const dz_tensor_blob_t* t = tensors;
        size_t ti = 0;
        if ((rc = upload_f32(m, t[ti++], V * D, &m->emb, st))) break;
        if (!m->tied && (rc = make_qmat({&t[ti++]}, st, &m->head))) break;
        if ((rc = upload_f32(m, t[ti++], V, &m->out_bias, st))) break;
        step += (m->tied ? V * D * 4 : m->head.code_bytes + m->head.scale_bytes) + V * 4 + D * 4;
        m->layers.resize(desc->num_layers);
        for (size_t l = 0; l < desc->num_layers && !rc; l++) {
            DevLayer& L = m->layers[l];
            const dz_tensor_blob_t *tq = &t[ti], *tk = &t[ti + 1], *tv = &t[ti + 2], *two = &t[ti + 3];
            ti += 4;
            const dz_tensor_blob_t* tg1 = &t[ti++];
            const dz_tensor_blob_t* tbe1 = m->rms ? nullptr : &t[ti++];
            const dz_tensor_blob_t *tw1 = &t[ti++], *tb1 = &t[ti++];
            const dz_tensor_blob_t* twg = m->swiglu ? &t[ti++] : nullptr;
            const dz_tensor_blob_t* tbg = m->swiglu ? &t[ti++] : nullptr;
            const dz_tensor_blob_t *tw2 = &t[ti++], *tb2 = &t[ti++], *tg2 = &t[ti++];
            const dz_tensor_blob_t* tbe2 = m->rms ? nullptr : &t[ti++];
            SliceBlob sq, sk, sv, swo, sw1, sw2;
            if (tp_world > 1) {
                // this rank's heads (columns of Q, K, V; rows of W_o) and FFN columns (W1) / rows (W2)
                const size_t d0 = (size_t)tp_rank * m->dl, f0 = (size_t)tp_rank * m->Fl;
                if ((rc = slice_blob(*tq, 1, d0, m->dl, &sq)) || (rc = slice_blob(*tk, 1, d0, m->dl, &sk)) ||
                    (rc = slice_blob(*tv, 1, d0, m->dl, &sv)) || (rc = slice_blob(*two, 0, d0, m->dl, &swo)) ||
                    (rc = slice_blob(*tw1, 1, f0, m->Fl, &sw1)) || (rc = slice_blob(*tw2, 0, f0, m->Fl, &sw2)))
                    break;
                tq = &sq.blob; tk = &sk.blob; tv = &sv.blob;
                two = &swo.blob; tw1 = &sw1.blob; tw2 = &sw2.blob;
            }
            L.fused_qkv = tq->granularity != DZ_GRAN_ROW;
            if (L.fused_qkv) {
                if ((rc = make_qmat({tq, tk, tv}, st, &L.qkv))) break;
                step += L.qkv.code_bytes + L.qkv.scale_bytes;
            } else {
                if ((rc = make_qmat({tq}, st, &L.q)) || (rc = make_qmat({tk}, st, &L.k)) ||
                    (rc = make_qmat({tv}, st, &L.v)))
                    break;
                step += 3 * (L.q.code_bytes + L.q.scale_bytes);
            }
            if ((rc = make_qmat({two}, st, &L.wo))) break;
            if ((rc = upload_f32(m, *tg1, D, &L.g1, st)) || (tbe1 && (rc = upload_f32(m, *tbe1, D, &L.be1, st))))
                break;
            if (m->swiglu) {
                // one 2F-column product [x W_ff1 + b_ff1 | x W_ff_gate + b_ff_gate]
                // (two for ROW-granularity scales, which two matrices cannot share)
                if (tw1->granularity == DZ_GRAN_ROW) {
                    if ((rc = make_qmat({tw1}, st, &L.w1)) || (rc = make_qmat({twg}, st, &L.wg))) break;
                } else if ((rc = make_qmat({tw1, twg}, st, &L.w1))) {
                    break;
                }
                if (tb1->bits != 0 || tbg->bits != 0 || !tb1->f32 || !tbg->f32 || tb1->rows * tb1->cols != F ||
                    tbg->rows * tbg->cols != F) {
                    rc = fail(DZ_E_UNSUPPORTED, "FFN biases expected as float32");
                    break;
                }
                float* d = nullptr;
                if (cudaMalloc(&d, 2 * F * 4) != cudaSuccess) { rc = fail(DZ_E_NOMEM, "bias"); break; }
                m->f32_allocs.push_back(d);
                cudaMemcpyAsync(d, tb1->f32, F * 4, cudaMemcpyHostToDevice, st);
                cudaMemcpyAsync(d + F, tbg->f32, F * 4, cudaMemcpyHostToDevice, st);
                L.b1 = d;
            } else {
                if ((rc = make_qmat({tw1}, st, &L.w1))) break;
                if ((rc = upload_f32(m, *tb1, F, &L.b1, st))) break;
                if (tp_world > 1) L.b1 += (size_t)tp_rank * m->Fl;   // this rank's FFN columns
            }
            if ((rc = make_qmat({tw2}, st, &L.w2))) break;
            if ((rc = upload_f32(m, *tb2, D, &L.b2, st)) || (rc = upload_f32(m, *tg2, D, &L.g2, st)) ||
                (tbe2 && (rc = upload_f32(m, *tbe2, D, &L.be2, st))))
                break;
            step += L.wo.code_bytes + L.wo.scale_bytes + L.w1.code_bytes + L.w1.scale_bytes + L.wg.code_bytes +
                    L.wg.scale_bytes + L.w2.code_bytes +
                    L.w2.scale_bytes + ((m->rms ? 4 : 6) * D + (m->swiglu ? 2 : 1) * F) * 4;
        }
        if (rc) break;
        // sinusoid table for positions [0, max_seq_len + 4096), computed on the
        // host exactly as compute_positional_encoding does
        m->pe_rows = (long long)desc->max_seq_len + 4096;
        std::vector<float> pe((size_t)m->pe_rows * D);
        dz_positional_encoding(pe.data(), (size_t)m->pe_rows, D);
        float* dpe = nullptr;
        if (cudaMalloc(&dpe, pe.size() * 4) != cudaSuccess) { rc = fail(DZ_E_NOMEM, "pe table"); break; }
        m->f32_allocs.push_back(dpe);
        m->pe = dpe;
        if (cudaMemcpyAsync(dpe, pe.data(), pe.size() * 4, cudaMemcpyHostToDevice, st) != cudaSuccess ||
            cudaStreamSynchronize(st) != cudaSuccess) {
            rc = fail(DZ_E_DEVICE, "pe upload");
            break;
        }
        if (m->rope) {
            // cos / sin of position * 10000^(-2p / head_dim) for the same
            // positions, in double as rope_rotate computes them
            // (src/core/transformer.c:33-38), rounded to float
            const size_t hd = D / H, half = hd / 2;
            std::vector<float> rt((size_t)m->pe_rows * half * 2);
            for (size_t pos = 0; pos < (size_t)m->pe_rows; pos++)
                for (size_t pp = 0; pp < half; pp++) {
                    const double angle = (double)pos * pow(10000.0, -(double)(2 * pp) / (double)hd);
                    rt[(pos * half + pp) * 2] = (float)cos(angle);
                    rt[(pos * half + pp) * 2 + 1] = (float)sin(angle);
                }
            float* drt = nullptr;
            if (cudaMalloc(&drt, rt.size() * 4) != cudaSuccess) { rc = fail(DZ_E_NOMEM, "rope table"); break; }
            m->f32_allocs.push_back(drt);
            m->rope_tab = drt;
            if (cudaMemcpyAsync(drt, rt.data(), rt.size() * 4, cudaMemcpyHostToDevice, st) != cudaSuccess ||
                cudaStreamSynchronize(st) != cudaSuccess) {
                rc = fail(DZ_E_DEVICE, "rope table upload");
                break;
            }
        }
    } while (0);
    cudaStreamSynchronize(st);
    cudaStreamDestroy(st);
    if (rc) {
        model_release(m);
        return rc;
    }
    m->step_bytes = step;
    m->comm = comm;
    if (tp_world == 1) prepare_seqgen(m);
    *out = m;
    return DZ_OK;
}

extern "C" void dz_cuda_model_free(dz_cuda_model_t* m) { model_release(m); }

extern "C" size_t dz_cuda_model_step_bytes(const dz_cuda_model_t* m) { return m ? m->step_bytes : 0; }

// ------------------------------------------------------------------ cache

// The generation loop's controls as one generation uses them (host copy of
// dz_generation_controls_t, stop sequences flattened).
struct GenControls {
    bool on = false;
    float penalty = 1.0f;
    uint32_t eos_id = 0xffffffffu, mask_from = 0xffffffffu;
    int min_new = 0;
    std::vector<uint32_t> stop_tok;
    std::vector<int> stop_off;   // n_stops + 1 offsets
    bool operator<(const GenControls& o) const {
        return std::tie(on, penalty, eos_id, mask_from, min_new, stop_tok, stop_off) <
               std::tie(o.on, o.penalty, o.eos_id, o.mask_from, o.min_new, o.stop_tok, o.stop_off);
    }
};

struct GenKey {
    size_t plen, n_new;
    int strategy;
    float temperature, top_p;
    uint32_t top_k;
    std::vector<uint32_t> masked;
    GenControls ctl;
    const void* prompts;
    const void* seeds;
    const void* out;
    bool operator<(const GenKey& o) const {
        return std::tie(plen, n_new, strategy, temperature, top_p, top_k, masked, ctl, prompts, seeds, out) <
               std::tie(o.plen, o.n_new, o.strategy, o.temperature, o.top_p, o.top_k, o.masked, o.ctl, o.prompts,
                        o.seeds, o.out);
    }
};

struct dz_cuda_cache {
    dz_cuda_model_t* model = nullptr;
    int B = 0, cap = 0;
    cudaStream_t stream = nullptr;
    bool own_stream = false;
    float *keys = nullptr, *values = nullptr;  // [L][B][cap][D]
    // the K / V rings as [L * B * cap][D] fp32 tensors, box {head dim, 32}
    // (the streamed decode attention); kv_maps false: not available
    CUtensorMap tm_keys, tm_values;
    bool kv_maps = false;
    int *start = nullptr, *length = nullptr, *slot = nullptr, *ctx = nullptr, *row_off = nullptr;
    long long* total = nullptr;
    float *hidden = nullptr, *q = nullptr, *concat = nullptr, *attn_raw = nullptr, *attn_norm = nullptr;
    float *ff = nullptr, *ff_raw = nullptr, *logits = nullptr;
    uint32_t* tok = nullptr;
    uint64_t* rng = nullptr;
    uint32_t* masked = nullptr;   // device copy of the masked ids (grown)
    // token history for the repetition penalty: a bit per id fed through the
    // model since reset, per sequence; invalid after a fused-path generation
    uint32_t* seen = nullptr;
    int seen_words = 0;
    bool seen_valid = true;
    uint32_t* gen_state = nullptr;   // [B][DZ_GEN_WORDS] (dz_cuda_generate_ex)
    uint32_t* stop_tok = nullptr;    // device copy of the stop sequences (grown)
    int* stop_off = nullptr;
    size_t stop_tok_cap = 0, stop_off_cap = 0;
    uint32_t* host_gen = nullptr;    // pinned copy of gen_state
    size_t masked_cap = 0;
    // device buffers of the host-facing generate()
    uint32_t* gen_prompts = nullptr;
    size_t gen_prompts_cap = 0;
    uint32_t* gen_out = nullptr;
    size_t gen_out_cap = 0;
    uint64_t* gen_seeds = nullptr;
    uint64_t* host_rng = nullptr;  // pinned staging
    uint32_t* host_ids = nullptr;
    cudaGraphExec_t step_graph = nullptr;
    std::map<GenKey, cudaGraphExec_t> gen_graphs;
    double prof_ctx_bytes_per_layer = 0, prof_ctx_flops_per_layer = 0;  // set per profiled step
    int path = DZ_PATH_AUTO;
    void* xs_scratch = nullptr;          // split activations of the layered path's matvecs
    int* status = nullptr;        // device word the fused kernel reports a timeout in
    unsigned long long* phase_ns = nullptr;  // [SEQ_PHASES] fused-kernel phase clock (profiling)
    int* host_status = nullptr;   // pinned
    std::vector<void*> allocs;
    // batched prefill (prefill.cuh): row buffers for up to pf_rows rows, grown on demand
    int prefill = DZ_PREFILL_AUTO;
    size_t pf_rows = 0;
    float *pf_hidden = nullptr, *pf_q = nullptr, *pf_concat = nullptr, *pf_attn_raw = nullptr;
    float *pf_attn_norm = nullptr, *pf_ff = nullptr, *pf_ff_raw = nullptr;
    int* pf_rowoff = nullptr;
    void* pf_scratch = nullptr;
    uint32_t* pf_ids = nullptr;   // dz_cuda_prefill's device copies
    int* pf_lens = nullptr;
    size_t pf_ids_cap = 0;
    uint8_t* mk_buf = nullptr;    // dz_cuda_forward_masked's padding + attention masks
    size_t mk_cap = 0;
};

static void free_prefill(dz_cuda_cache_t* c) {
    for (void* p : {(void*)c->pf_hidden, (void*)c->pf_q, (void*)c->pf_concat, (void*)c->pf_attn_raw,
                    (void*)c->pf_attn_norm, (void*)c->pf_ff, (void*)c->pf_ff_raw, (void*)c->pf_rowoff,
                    c->pf_scratch, (void*)c->pf_ids, (void*)c->pf_lens, (void*)c->mk_buf})
        cudaFree(p);
    c->mk_buf = nullptr;
    c->mk_cap = 0;
    c->pf_hidden = c->pf_q = c->pf_concat = c->pf_attn_raw = c->pf_attn_norm = c->pf_ff = c->pf_ff_raw = nullptr;
    c->pf_rowoff = nullptr;
    c->pf_scratch = nullptr;
    c->pf_ids = nullptr;
    c->pf_lens = nullptr;
    c->pf_rows = 0;
    c->pf_ids_cap = 0;
}

static int cache_alloc(dz_cuda_cache_t* c, void** p, size_t bytes) {
    DZ_CUDA(cudaMalloc(p, bytes));
    c->allocs.push_back(*p);
    return DZ_OK;
}

static void clear_graphs(dz_cuda_cache_t* c) {
    if (c->step_graph) cudaGraphExecDestroy(c->step_graph);
    c->step_graph = nullptr;
    for (auto& kv : c->gen_graphs) cudaGraphExecDestroy(kv.second);
    c->gen_graphs.clear();
}

extern "C" void dz_cuda_cache_free(dz_cuda_cache_t* c) {
    if (!c) return;
    {
        DeviceGuard g(c->model->device);
        if (c->stream) cudaStreamSynchronize(c->stream);
        clear_graphs(c);
        for (void* p : c->allocs) cudaFree(p);
        cudaFree(c->gen_prompts);
        cudaFree(c->gen_out);
        cudaFree(c->masked);
        cudaFree(c->stop_tok);
        cudaFree(c->stop_off);
        cudaFreeHost(c->host_gen);
        cudaFreeHost(c->host_rng);
        cudaFreeHost(c->host_ids);
        cudaFreeHost(c->host_status);
        free_prefill(c);
        if (c->own_stream && c->stream) cudaStreamDestroy(c->stream);
    }
    model_release(c->model);
    delete c;
}

extern "C" int dz_cuda_cache_create(dz_cuda_model_t* m, size_t batch, size_t capacity, dz_cuda_cache_t** out) {
    if (!out) return fail(DZ_E_INVALID, "null output handle");
    *out = nullptr;
    if (!m || batch == 0 || batch > 65535 || capacity == 0 || capacity > m->desc.max_seq_len)
        return fail(DZ_E_INVALID, "cache: batch must be 1..65535 and capacity 1..max_seq_len");
    DeviceGuard g(m->device);
    auto* c = new (std::nothrow) dz_cuda_cache;
    if (!c) return fail(DZ_E_NOMEM, "host allocation");
    m->refs++;
    c->model = m;
    c->B = (int)batch;
    c->cap = (int)capacity;
    const size_t D = m->desc.embedding_dim, V = m->desc.vocab_size, Lr = m->desc.num_layers;
    const size_t B = batch;
    int rc = DZ_OK;
    if (cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking) != cudaSuccess) {
        rc = fail(DZ_E_DEVICE, "stream creation failed");
    } else {
        c->own_stream = true;
    }
    const size_t dl = m->dl, Fl = m->Fl;   // this rank's attention and FFN widths
    if (!rc) rc = cache_alloc(c, (void**)&c->keys, Lr * B * capacity * dl * 4);
    if (!rc) rc = cache_alloc(c, (void**)&c->values, Lr * B * capacity * dl * 4);
    if (!rc) {
        const size_t hd = D / m->desc.num_heads, rows = Lr * B * capacity;
        TensorMapEncodeFn enc = tensor_map_encoder();
        c->kv_maps = false;
        if (enc && (hd == 64 || hd == 128) && rows < (size_t)INT32_MAX) {
            const cuuint64_t dims[2] = {(cuuint64_t)dl, (cuuint64_t)rows};
            const cuuint64_t strides[1] = {(cuuint64_t)dl * 4};
            const cuuint32_t box[2] = {(cuuint32_t)hd, (cuuint32_t)AD_KT};
            const cuuint32_t es[2] = {1, 1};
            c->kv_maps = true;
            for (auto pr : {std::make_pair(&c->tm_keys, c->keys), std::make_pair(&c->tm_values, c->values)})
                c->kv_maps = c->kv_maps &&
                             enc(pr.first, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, pr.second, dims, strides, box, es,
                                 CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                                 CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
        }
    }
    if (!rc) rc = cache_alloc(c, (void**)&c->start, B * 4);
    if (!rc) rc = cache_alloc(c, (void**)&c->length, B * 4);
    if (!rc) rc = cache_alloc(c, (void**)&c->slot, B * 4);
    if (!rc) rc = cache_alloc(c, (void**)&c->ctx, B * 4);
    if (!rc) rc = cache_alloc(c, (void**)&c->row_off, B * 4);
    if (!rc) rc = cache_alloc(c, (void**)&c->total, B * 8);
    if (!rc) rc = cache_alloc(c, (void**)&c->hidden, B * D * 4);
    if (!rc) rc = cache_alloc(c, (void**)&c->q, B * dl * 4);
    if (!rc) rc = cache_alloc(c, (void**)&c->concat, B * dl * 4);
    if (!rc) rc = cache_alloc(c, (void**)&c->attn_raw, B * D * 4);
    if (!rc) rc = cache_alloc(c, (void**)&c->attn_norm, B * D * 4);
    if (!rc) rc = cache_alloc(c, (void**)&c->ff, B * Fl * (m->swiglu ? 2 : 1) * 4);
    if (!rc) rc = cache_alloc(c, (void**)&c->ff_raw, B * D * 4);
    if (!rc) rc = cache_alloc(c, (void**)&c->logits, B * V * 4);
    if (!rc) rc = cache_alloc(c, (void**)&c->tok, B * 4);
    if (!rc) rc = cache_alloc(c, (void**)&c->rng, B * 8);
    if (!rc) rc = cache_alloc(c, (void**)&c->gen_seeds, B * 8);
    c->seen_words = (int)((V + 31) / 32);
    if (!rc) rc = cache_alloc(c, (void**)&c->seen, B * (size_t)c->seen_words * 4);
    if (!rc) rc = cache_alloc(c, (void**)&c->gen_state, B * DZ_GEN_WORDS * 4);
    if (!rc && cudaMallocHost(&c->host_gen, B * DZ_GEN_WORDS * 4) != cudaSuccess)
        rc = fail(DZ_E_NOMEM, "pinned host");
    if (!rc) {
        size_t xs = 0;
        for (const auto& L : m->layers)
            for (const DevQMat* q : {&L.qkv, &L.q, &L.k, &L.v, &L.wo, &L.w1, &L.wg, &L.w2})
                if (q->codes) xs = std::max(xs, qmv_scratch_bytes(*q, (int)B));
        if (m->head.codes) xs = std::max(xs, qmv_scratch_bytes(m->head, (int)B));
        rc = cache_alloc(c, (void**)&c->xs_scratch, xs);
        if (!rc && cudaMemset(c->xs_scratch, 0, xs) != cudaSuccess) rc = fail(DZ_E_DEVICE, "scratch memset");
    }
    if (!rc) rc = cache_alloc(c, (void**)&c->status, 4);
    if (!rc) rc = cache_alloc(c, (void**)&c->phase_ns, SEQ_PHASES * 8);
    if (!rc && cudaMallocHost(&c->host_status, 4) != cudaSuccess) rc = fail(DZ_E_NOMEM, "pinned host");
    if (!rc && cudaMallocHost(&c->host_rng, B * 8) != cudaSuccess) rc = fail(DZ_E_NOMEM, "pinned host");
    if (!rc && cudaMallocHost(&c->host_ids, B * 4) != cudaSuccess) rc = fail(DZ_E_NOMEM, "pinned host");
    if (!rc) {
        // the largest selection footprint (sorted vocabulary or top-k buffer)
        const size_t smem = dz_select_smem_bytes((int)V, 2, SEL_TOPK_CAP);
        if (smem > 48 * 1024 &&
            cudaFuncSetAttribute(dz_select_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
                cudaSuccess)
            rc = fail(DZ_E_DEVICE, "select kernel shared memory");
    }
    if (!rc && m->seq_ok) {
        const size_t ss = seq_smem_for(m, c->cap);
        if (ss <= (size_t)SEQ_SMEM_LIMIT) {
            // the attribute is an upper bound shared by every cache: raise it to the limit
            cudaError_t e = dz_seqgen_set_smem(m->seq_bits, SEQ_SMEM_LIMIT);
            if (e != cudaSuccess) rc = fail(DZ_E_DEVICE, "fused kernel shared memory: %s", cudaGetErrorString(e));
        }
    }
    if (!rc) {
        cudaMemsetAsync(c->status, 0, 4, c->stream);
        cudaMemsetAsync(c->start, 0, B * 4, c->stream);
        cudaMemsetAsync(c->length, 0, B * 4, c->stream);
        cudaMemsetAsync(c->total, 0, B * 8, c->stream);
        cudaMemsetAsync(c->seen, 0, B * (size_t)c->seen_words * 4, c->stream);
        if (cudaStreamSynchronize(c->stream) != cudaSuccess) rc = fail(DZ_E_DEVICE, "cache init");
    }
    if (rc) {
        dz_cuda_cache_free(c);
        return rc;
    }
    *out = c;
    return DZ_OK;
}

extern "C" int dz_cuda_cache_set_stream(dz_cuda_cache_t* c, void* stream) {
    if (!c) return fail(DZ_E_INVALID, "null cache");
    DeviceGuard g(c->model->device);
    cudaStreamSynchronize(c->stream);
    if (c->own_stream) cudaStreamDestroy(c->stream);
    c->stream = (cudaStream_t)stream;
    c->own_stream = false;
    return DZ_OK;
}

extern "C" void* dz_cuda_cache_stream(const dz_cuda_cache_t* c) { return c ? (void*)c->stream : nullptr; }

__global__ void dz_reset_kernel(int* start, int* length, long long* total, const uint8_t* mask, int B) {
    const int b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b < B && (!mask || mask[b])) {
        start[b] = 0;
        length[b] = 0;
        total[b] = 0;
    }
}

extern "C" int dz_cuda_cache_reset(dz_cuda_cache_t* c, const uint8_t* seq_mask) {
    if (!c) return fail(DZ_E_INVALID, "null cache");
    DeviceGuard g(c->model->device);
    uint8_t* dmask = nullptr;
    if (seq_mask) {
        DZ_CUDA(cudaMalloc(&dmask, c->B));
        DZ_CUDA(cudaMemcpyAsync(dmask, seq_mask, c->B, cudaMemcpyHostToDevice, c->stream));
    }
    dz_reset_kernel<<<(c->B + 255) / 256, 256, 0, c->stream>>>(c->start, c->length, c->total, dmask, c->B);
    dz_seen_clear_kernel<<<dim3((unsigned)((c->seen_words + 255) / 256), (unsigned)c->B), 256, 0, c->stream>>>(
        c->seen, c->seen_words, dmask);
    if (!seq_mask) c->seen_valid = true;
    cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
    cudaFree(dmask);
    if (e != cudaSuccess) return fail(DZ_E_DEVICE, "reset: %s", cudaGetErrorString(e));
    return DZ_OK;
}

// One decode step for all sequences; returns the number of kernel launches.
// Sum of every rank's partial [rows x D] product, in place (tensor parallelism).
static void tp_allreduce(dz_cuda_model_t* m, float* buf, size_t count, cudaStream_t st) {
    if (m->tp_world <= 1) return;
    // bytes: what each rank sends over NVLink in a ring all-reduce, 2 (w - 1) / w of the buffer
    ProfScope prof(DZ_KERNEL_ALLREDUCE, 8.0 * count * (m->tp_world - 1) / m->tp_world, 0, st);
    nccl_api()->all_reduce(buf, buf, count, ncclFloat32, ncclSum, m->comm, st);
}

// Launches of one layer pass over R rows and of the output head.
static int layer_launches(const dz_cuda_model_t* m, const DevLayer& L, int R) {
    int n = L.fused_qkv ? qmv_launches(L.qkv, R) : qmv_launches(L.q, R) + qmv_launches(L.k, R) + qmv_launches(L.v, R);
    n += qmv_launches(L.wo, R) + qmv_launches(L.w1, R) + qmv_launches(L.w2, R);
    if (L.wg.codes) n += qmv_launches(L.wg, R);
    return n + 3 + (m->rope ? 1 : 0) + (m->swiglu ? 1 : 0);   // attention, two norms, RoPE, SwiGLU
}
static int head_launches(const dz_cuda_model_t* m, int B) { return m->tied ? 1 : qmv_launches(m->head, B); }

// The attention-out and FFN-out norms: LayerNorm (src/core/tensor_ops.c:
// 148-171) or RMSNorm (:173-179), eps 1e-6, `res` added to x first.
static void launch_norm(const dz_cuda_model_t* m, const float* x, const float* res, const float* g, const float* be,
                        float* y, int rows, int D, cudaStream_t st) {
    if (m->rms)
        dz_rmsnorm_kernel<<<rows, RMS_THREADS, 0, st>>>(x, res, g, y, D, 1e-6f);
    else
        dz_layernorm_kernel<<<rows, LN_THREADS, 0, st>>>(x, res, g, be, y, D, 1e-6f);
}

// Whether DZ_NORM_LIMBS=0 in the environment turns the norm + split fusion
// off (for comparison: both give the same bits).
static bool norm_limbs_enabled() {
    static const bool v = [] {
        const char* e = getenv("DZ_NORM_LIMBS");
        return !(e && strcmp(e, "0") == 0);
    }();
    return v;
}

// The norm can write the limbs of the product W that reads its `rows` x D
// output when it is a LayerNorm of width <= LN_LIMBS_MAX_DIM, W has no row
// scales (the split would fold them in) and W runs on the tensor-core GEMM.
static bool norm_limbs_ok(const dz_cuda_model_t* m, const DevQMat& W, int rows, int D) {
    return norm_limbs_enabled() && !m->rms && W.codes && !W.k_scale && W.K == D && D <= LN_LIMBS_MAX_DIM &&
           D % 4 == 0 && rows >= UGEMM_MIN_M && W.kn && (size_t)W.K * W.N >= UGEMM_MIN_WEIGHTS;
}
// The fused norm's float4 element pass: every row and parameter 16-byte aligned.
static bool norm_limbs_aligned(const float* x, const float* res, const float* g, const float* be, const float* y) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(res) |
                        reinterpret_cast<uintptr_t>(g) | reinterpret_cast<uintptr_t>(be) | reinterpret_cast<uintptr_t>(y);
    return (a & 15u) == 0;
}

// The norm (launch_norm) fused with the split of W's product: the limbs and
// shifts go where launch_qmv's GEMM reads them in `scratch`. The caller checked
// norm_limbs_ok.
static void launch_norm_limbs(const float* x, const float* res, const float* g, const float* be, float* y, int rows,
                              int D, const DevQMat& W, void* scratch, cudaStream_t st) {
    const int Kp = round_up(W.K, UG_BK);
    uint8_t* base = static_cast<uint8_t*>(scratch) + SCRATCH_COUNTERS;   // launch_qmv -> launch_ugemm layout
    int8_t* L = reinterpret_cast<int8_t*>(base);
    int* shift = reinterpret_cast<int*>(base + r256(3 * (size_t)rows * Kp));
    dz_layernorm_limbs_kernel<<<rows, LN_THREADS, 0, st>>>(x, res, g, be, y, D, 1e-6f, rows, Kp, L, shift);
}

// FFN up-projection of R rows of x into ff (row stride ldf): bias and ReLU /
// GELU in the product's epilogue, or both SwiGLU halves then the gate
// (src/core/transformer.c:819-832). Returns the launches.
static int launch_ffn_up(const dz_cuda_model_t* m, const DevLayer& L, const float* x, int D, int R, float* ff,
                         long long ldf, int F, cudaStream_t st, void* scratch, int* status, bool limbs_ready = false) {
    QmvEpilogue e1 = plain_epilogue(L.w1, ff, ldf);
    e1.bias = L.b1;
    e1.act = m->swiglu ? DZ_ACT_NONE : m->act;
    int n = launch_qmv(L.w1, x, D, R, e1, st, scratch, status, limbs_ready);
    if (L.wg.codes) {
        QmvEpilogue eg = plain_epilogue(L.wg, ff + F, ldf);
        eg.bias = L.b1 + F;
        n += launch_qmv(L.wg, x, D, R, eg, st, scratch, status, limbs_ready);
    }
    if (m->swiglu) {
        dz_swiglu_kernel<<<dim3((unsigned)((F + 255) / 256), (unsigned)std::min(R, 65535)), 256, 0, st>>>(ff, R, F,
                                                                                                        ldf);
        n++;
    }
    return n;
}

// Output head over B hidden rows into c->logits: the quantized W_out, or the
// token embeddings transposed when tied (src/core/lm_head.c:21-46).
static int launch_head(dz_cuda_cache_t* c, cudaStream_t st, bool limbs_ready = false) {
    dz_cuda_model_t* m = c->model;
    const int D = (int)m->desc.embedding_dim, V = (int)m->desc.vocab_size, B = c->B;
    if (m->tied) {
        dz_tied_head_kernel<<<(V + TIED_ROWS - 1) / TIED_ROWS, TIED_ROWS * 32, 0, st>>>(c->hidden, B, m->emb,
                                                                                       m->out_bias, c->logits, V, D);
        return 1;
    }
    QmvEpilogue eh = plain_epilogue(m->head, c->logits, V);
    eh.bias = m->out_bias;
    return launch_qmv(m->head, c->hidden, D, B, eh, st, c->xs_scratch, c->status, limbs_ready);
}

static int enqueue_step(dz_cuda_cache_t* c, const uint32_t* tokens, long long tok_stride) {
    dz_cuda_model_t* m = c->model;
    const int D = (int)m->desc.embedding_dim, V = (int)m->desc.vocab_size;
    const int H = m->Hl, dl = m->dl, F = m->Fl;   // this rank's heads, attention width, FFN width
    const int hd = D / (int)m->desc.num_heads, B = c->B, cap = c->cap;
    cudaStream_t st = c->stream;
    int launches = 0;
    RingState rs{c->start, c->length, c->total, c->slot, c->ctx, c->row_off, c->seen, c->seen_words};
    {
        ProfScope prof(DZ_KERNEL_STEP_BEGIN, (double)B * D * 12, 0, st);
        dz_step_begin_kernel<<<B, 128, 0, st>>>(rs, tokens, tok_stride, m->emb, m->rope ? nullptr : m->pe,
                                                m->pe_rows, c->hidden, D, dl, V, cap);
    }
    launches++;
    const size_t att_smem = (size_t)(cap + hd + ATT_THREADS) * 4;
    bool hidden_limbs = false;   // the previous norm wrote the limbs of the product reading c->hidden
    for (size_t l = 0; l < m->layers.size(); l++) {
        DevLayer& L = m->layers[l];
        float* Kl = c->keys + l * (size_t)B * cap * dl;
        float* Vl = c->values + l * (size_t)B * cap * dl;
        if (L.fused_qkv) {
            QmvEpilogue ep = plain_epilogue(L.qkv, c->q, dl);
            ep.nseg = 3;
            ep.seg_start[0] = 0; ep.seg_start[1] = dl; ep.seg_start[2] = 2 * dl; ep.seg_start[3] = 3 * dl;
            ep.seg_ptr[1] = Kl; ep.seg_ld[1] = (long long)cap * dl; ep.seg_row_off[1] = c->row_off;
            ep.seg_ptr[2] = Vl; ep.seg_ld[2] = (long long)cap * dl; ep.seg_row_off[2] = c->row_off;
            launches += launch_qmv(L.qkv, c->hidden, D, B, ep, st, c->xs_scratch, c->status, hidden_limbs);
        } else {
            QmvEpilogue eq = plain_epilogue(L.q, c->q, dl);
            launches += launch_qmv(L.q, c->hidden, D, B, eq, st, c->xs_scratch, c->status);
            QmvEpilogue ek = plain_epilogue(L.k, Kl, (long long)cap * dl);
            ek.seg_row_off[0] = c->row_off;
            launches += launch_qmv(L.k, c->hidden, D, B, ek, st, c->xs_scratch, c->status);
            QmvEpilogue ev = plain_epilogue(L.v, Vl, (long long)cap * dl);
            ev.seg_row_off[0] = c->row_off;
            launches += launch_qmv(L.v, c->hidden, D, B, ev, st, c->xs_scratch, c->status);
        }
        if (m->rope) {
            dz_rope_decode_kernel<<<B, 128, 0, st>>>(c->q, Kl, (long long)cap * dl, c->row_off, c->total, dl, hd,
                                                     m->rope_tab, m->pe_rows);
            launches++;
        }
        {
            // bytes: the K and V rows of every sequence's context (ctx <= cap; the
            // exact per-step context is device state, so the capacity bound is used
            // only when the profiler cannot read it) + q + output
            ProfScope prof(DZ_KERNEL_ATTENTION, c->prof_ctx_bytes_per_layer + 8.0 * B * dl,
                           c->prof_ctx_flops_per_layer, st);
            AdArgs aa{c->q, Kl, Vl, c->start, c->ctx, c->concat, dl, cap, c->status, (int)(l * B * cap)};
            if ((hd == 128 || hd == 64) && c->kv_maps && attn_streamed_kernel())
                dz_attn_decode_launch(c->tm_keys, c->tm_values, aa, hd, H, B, st);
            else if (hd == 128)
                dz_attention_decode2_kernel<4><<<dim3(H, B), ATT2_THREADS, 0, st>>>(c->q, Kl, Vl, c->start, c->ctx,
                                                                                   c->concat, dl, cap);
            else if (hd == 64)
                dz_attention_decode2_kernel<2><<<dim3(H, B), ATT2_THREADS, 0, st>>>(c->q, Kl, Vl, c->start, c->ctx,
                                                                                   c->concat, dl, cap);
            else
                dz_attention_decode_kernel<<<dim3(H, B), ATT_THREADS, att_smem, st>>>(c->q, Kl, Vl, c->start,
                                                                                     c->ctx, c->concat, dl, hd, cap);
        }
        launches++;
        QmvEpilogue eo = plain_epilogue(L.wo, c->attn_raw, D);
        launches += launch_qmv(L.wo, c->concat, dl, B, eo, st, c->xs_scratch, c->status);
        tp_allreduce(m, c->attn_raw, (size_t)B * D, st);
        const bool ffn_limbs = norm_limbs_ok(m, L.w1, B, D) && (!L.wg.codes || norm_limbs_ok(m, L.wg, B, D)) &&
                               norm_limbs_aligned(c->attn_raw, c->hidden, L.g1, L.be1, c->attn_norm);
        {
            ProfScope prof(DZ_KERNEL_LAYERNORM, 12.0 * B * D + 8.0 * D + (ffn_limbs ? 3.0 * B * D : 0.0), 0, st);
            if (ffn_limbs)
                launch_norm_limbs(c->attn_raw, c->hidden, L.g1, L.be1, c->attn_norm, B, D, L.w1, c->xs_scratch, st);
            else
                launch_norm(m, c->attn_raw, c->hidden, L.g1, L.be1, c->attn_norm, B, D, st);
        }
        launches++;
        const long long ldf = m->swiglu ? 2LL * F : F;
        launches += launch_ffn_up(m, L, c->attn_norm, D, B, c->ff, ldf, F, st, c->xs_scratch, c->status, ffn_limbs);
        QmvEpilogue e2 = plain_epilogue(L.w2, c->ff_raw, D);
        if (m->tp_rank == 0) {   // bias and residual once, before the sum over ranks
            e2.bias = L.b2;
            e2.residual = c->attn_norm;
            e2.ld_res = D;
        }
        launches += launch_qmv(L.w2, c->ff, ldf, B, e2, st, c->xs_scratch, c->status);
        tp_allreduce(m, c->ff_raw, (size_t)B * D, st);
        // the product reading c->hidden next: the next layer's fused QKV, or the head
        const DevQMat* next = l + 1 < m->layers.size() ? (m->layers[l + 1].fused_qkv ? &m->layers[l + 1].qkv : nullptr)
                                                       : (m->tied ? nullptr : &m->head);
        hidden_limbs = next && norm_limbs_ok(m, *next, B, D) &&
                       norm_limbs_aligned(c->ff_raw, nullptr, L.g2, L.be2, c->hidden);
        {
            ProfScope prof(DZ_KERNEL_LAYERNORM, 8.0 * B * D + 8.0 * D + (hidden_limbs ? 3.0 * B * D : 0.0), 0, st);
            if (hidden_limbs)
                launch_norm_limbs(c->ff_raw, nullptr, L.g2, L.be2, c->hidden, B, D, *next, c->xs_scratch, st);
            else
                launch_norm(m, c->ff_raw, nullptr, L.g2, L.be2, c->hidden, B, D, st);
        }
        launches++;
    }
    launches += launch_head(c, st, hidden_limbs);
    return launches;
}

static int ensure_masked(dz_cuda_cache_t* c, const dz_sampling_t* s) {
    if (!s || s->n_masked == 0) return DZ_OK;
    if (!s->masked_ids) return fail(DZ_E_INVALID, "masked_ids is NULL with n_masked > 0");
    if (s->n_masked > c->masked_cap) {
        clear_graphs(c);
        cudaFree(c->masked);
        c->masked = nullptr;
        c->masked_cap = 0;
        DZ_CUDA(cudaMalloc(&c->masked, s->n_masked * 4));
        c->masked_cap = s->n_masked;
    }
    return DZ_OK;
}

static int check_sampling(const dz_cuda_cache_t* c, const dz_sampling_t* s) {
    if (!s) return DZ_OK;
    const int V = (int)c->model->desc.vocab_size;
    if (s->strategy < 0 || s->strategy > 2) return fail(DZ_E_INVALID, "unknown sampling strategy %d", s->strategy);
    if (s->strategy == 2 && s->temperature > 0.0f && V > SEL_SORT_CAP)
        return fail(DZ_E_UNSUPPORTED, "top-p over a vocabulary above %d ids", SEL_SORT_CAP);
    if (s->strategy == 1 && s->temperature > 0.0f && V > SEL_SORT_CAP && s->top_k > (uint32_t)SEL_TOPK_CAP)
        return fail(DZ_E_UNSUPPORTED, "top-k above %d over a vocabulary above %d ids", SEL_TOPK_CAP, SEL_SORT_CAP);
    return DZ_OK;
}

// The device form of a generation's controls: penalty over the token
// history, the unassigned range, and (with `state`) EOS, the minimum length
// and stop sequences from the cache's device copies.
static SelectControls select_controls(const dz_cuda_cache_t* c, const GenControls* g, bool with_state) {
    SelectControls k;
    memset(&k, 0, sizeof(k));
    k.mask_from = 0xffffffffu;
    k.eos_id = 0xffffffffu;
    if (!g || !g->on) return k;
    k.seen = g->penalty > 1.0f ? c->seen : nullptr;
    k.seen_words = c->seen_words;
    k.penalty = g->penalty;
    k.mask_from = g->mask_from;
    if (with_state) {
        k.state = c->gen_state;
        k.eos_id = g->eos_id;
        k.min_new = g->min_new;
        k.stop_tok = c->stop_tok;
        k.stop_off = c->stop_off;
        k.n_stops = (int)g->stop_off.size() - 1;
    }
    return k;
}

static int enqueue_select(dz_cuda_cache_t* c, const dz_sampling_t* s, uint64_t* rng, uint32_t* out,
                          long long out_stride, uint32_t* out2, const SelectControls* ctl = nullptr) {
    SelectArgs a;
    if (ctl) {
        a.ctl = *ctl;
    } else {
        memset(&a.ctl, 0, sizeof(a.ctl));
        a.ctl.mask_from = 0xffffffffu;
        a.ctl.eos_id = 0xffffffffu;
    }
    a.logits = c->logits;
    a.V = (int)c->model->desc.vocab_size;
    a.ld = a.V;
    a.strategy = s ? s->strategy : 0;
    a.temperature = s ? s->temperature : 0.0f;
    a.top_k = s ? (int)s->top_k : 0;
    a.top_p = s ? s->top_p : 0.0f;
    a.masked = (s && s->n_masked) ? c->masked : nullptr;
    a.n_masked = s ? (int)s->n_masked : 0;
    a.rng = rng;
    a.out = out;
    a.out_stride = out_stride;
    a.out2 = out2;
    const size_t smem = dz_select_smem_bytes(a.V, (a.rng && a.strategy) ? a.strategy : 0, a.top_k);
    ProfScope prof(DZ_KERNEL_SELECT, 4.0 * c->B * a.V, 0, c->stream);
    dz_select_kernel<<<c->B, SEL_THREADS, smem, c->stream>>>(a);
    return 1;
}

extern "C" int dz_cuda_forward_tokens(dz_cuda_cache_t* c, const uint32_t* token_ids, float* logits_out) {
    if (!c || !token_ids) return fail(DZ_E_INVALID, "null argument");
    DeviceGuard g(c->model->device);
    const size_t B = c->B, V = c->model->desc.vocab_size;
    memcpy(c->host_ids, token_ids, B * 4);
    DZ_CUDA(cudaMemcpyAsync(c->tok, c->host_ids, B * 4, cudaMemcpyHostToDevice, c->stream));
    if (!c->step_graph) {
        cudaGraph_t graph;
        DZ_CUDA(cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeThreadLocal));
        enqueue_step(c, c->tok, 1);
        cudaError_t e = cudaStreamEndCapture(c->stream, &graph);
        if (e != cudaSuccess) return fail(DZ_E_DEVICE, "capture: %s", cudaGetErrorString(e));
        e = cudaGraphInstantiate(&c->step_graph, graph, 0);
        cudaGraphDestroy(graph);
        if (e != cudaSuccess) {
            c->step_graph = nullptr;
            return fail(DZ_E_DEVICE, "instantiate: %s", cudaGetErrorString(e));
        }
    }
    DZ_CUDA(cudaGraphLaunch(c->step_graph, c->stream));
    if (logits_out) DZ_CUDA(cudaMemcpyAsync(logits_out, c->logits, B * V * 4, cudaMemcpyDeviceToHost, c->stream));
    DZ_CUDA(cudaStreamSynchronize(c->stream));
    return DZ_OK;
}

extern "C" int dz_cuda_select(dz_cuda_cache_t* c, const dz_sampling_t* s, uint64_t* rng_states, uint32_t* out_ids) {
    if (!c || !out_ids) return fail(DZ_E_INVALID, "null argument");
    int rc = check_sampling(c, s);
    if (rc) return rc;
    DeviceGuard g(c->model->device);
    if ((rc = ensure_masked(c, s))) return rc;
    const size_t B = c->B;
    if (s && s->n_masked)
        DZ_CUDA(cudaMemcpyAsync(c->masked, s->masked_ids, s->n_masked * 4, cudaMemcpyHostToDevice, c->stream));
    if (rng_states) {
        memcpy(c->host_rng, rng_states, B * 8);
        DZ_CUDA(cudaMemcpyAsync(c->rng, c->host_rng, B * 8, cudaMemcpyHostToDevice, c->stream));
    }
    enqueue_select(c, s, rng_states ? c->rng : nullptr, c->tok, 1, nullptr);
    DZ_CUDA(cudaGetLastError());
    DZ_CUDA(cudaMemcpyAsync(c->host_ids, c->tok, B * 4, cudaMemcpyDeviceToHost, c->stream));
    if (rng_states) DZ_CUDA(cudaMemcpyAsync(c->host_rng, c->rng, B * 8, cudaMemcpyDeviceToHost, c->stream));
    DZ_CUDA(cudaStreamSynchronize(c->stream));
    memcpy(out_ids, c->host_ids, B * 4);
    if (rng_states) memcpy(rng_states, c->host_rng, B * 8);
    return DZ_OK;
}

static int prepare_controls(dz_cuda_cache_t* c, const dz_generation_controls_t* in, GenControls* out);

extern "C" int dz_cuda_select_ex(dz_cuda_cache_t* c, const dz_sampling_t* s, const dz_generation_controls_t* controls,
                                 uint64_t* rng_states, uint32_t* out_ids) {
    if (!c || !out_ids) return fail(DZ_E_INVALID, "null argument");
    int rc = check_sampling(c, s);
    if (rc) return rc;
    DeviceGuard g(c->model->device);
    GenControls ctl;
    if ((rc = prepare_controls(c, controls, &ctl))) return rc;
    if (ctl.on && ctl.penalty > 1.0f && !c->seen_valid)
        return fail(DZ_E_UNSUPPORTED,
                    "repetition penalty: the last generation ran on the fused path, which keeps no token history; "
                    "reset the cache or generate on the layered path");
    if ((rc = ensure_masked(c, s))) return rc;
    const size_t B = c->B;
    if (s && s->n_masked)
        DZ_CUDA(cudaMemcpyAsync(c->masked, s->masked_ids, s->n_masked * 4, cudaMemcpyHostToDevice, c->stream));
    if (rng_states) {
        memcpy(c->host_rng, rng_states, B * 8);
        DZ_CUDA(cudaMemcpyAsync(c->rng, c->host_rng, B * 8, cudaMemcpyHostToDevice, c->stream));
    }
    // penalty and unassigned range only: EOS, the minimum length and stop
    // sequences stay with the caller's loop, as in the reference
    const SelectControls sc = select_controls(c, &ctl, false);
    enqueue_select(c, s, rng_states ? c->rng : nullptr, c->tok, 1, nullptr, &sc);
    DZ_CUDA(cudaGetLastError());
    DZ_CUDA(cudaMemcpyAsync(c->host_ids, c->tok, B * 4, cudaMemcpyDeviceToHost, c->stream));
    if (rng_states) DZ_CUDA(cudaMemcpyAsync(c->host_rng, c->rng, B * 8, cudaMemcpyDeviceToHost, c->stream));
    DZ_CUDA(cudaStreamSynchronize(c->stream));
    memcpy(out_ids, c->host_ids, B * 4);
    if (rng_states) memcpy(rng_states, c->host_rng, B * 8);
    return DZ_OK;
}

// Whether the fused one-CTA-per-sequence kernel runs this generation.
static bool use_seqgen(const dz_cuda_cache_t* c, const dz_sampling_t* s) {
    const dz_cuda_model_t* m = c->model;
    if (c->path == DZ_PATH_LAYERED || !m->seq_ok) return false;
    if (seq_smem_for(m, c->cap) > (size_t)SEQ_SMEM_LIMIT) return false;
    const bool sampled = s && s->strategy != 0 && s->temperature > 0.0f;
    if (sampled && m->desc.vocab_size > (size_t)SEL_SORT_CAP) return false;
    return true;
}

static int launch_seqgen(dz_cuda_cache_t* c, const uint32_t* prompts, size_t plen, size_t n_new,
                         const dz_sampling_t* s, const uint64_t* seeds, uint32_t* out) {
    const dz_cuda_model_t* m = c->model;
    SeqParams p;
    memset(&p, 0, sizeof(p));
    p.layers = m->seq_layers;
    p.L = (int)m->layers.size();
    p.D = (int)m->desc.embedding_dim;
    p.H = (int)m->desc.num_heads;
    p.V = (int)m->desc.vocab_size;
    p.cap = c->cap;
    p.bits = m->seq_bits;
    p.head = m->seq_head;
    p.emb = m->emb;
    p.pe = m->pe;
    p.pe_rows = m->pe_rows;
    p.out_bias = m->out_bias;
    p.keys = c->keys;
    p.values = c->values;
    p.start = c->start;
    p.length = c->length;
    p.total = c->total;
    p.prompts = prompts;
    p.plen = (int)plen;
    p.out = out;
    p.n_new = (int)n_new;
    p.seeds = seeds;
    p.strategy = s ? s->strategy : 0;
    p.temperature = s ? s->temperature : 0.0f;
    p.top_k = s ? (int)s->top_k : 0;
    p.top_p = s ? s->top_p : 0.0f;
    p.masked = (s && s->n_masked) ? c->masked : nullptr;
    p.n_masked = s ? (int)s->n_masked : 0;
    p.status = c->status;
    p.buf_bytes = m->seq_buf_bytes;
    p.B = c->B;
    p.phase_ns = g_prof ? c->phase_ns : nullptr;
    p.kv_smem = seq_kv_smem(m, c->cap) ? 1 : 0;
    const size_t smem = seq_smem_for(m, c->cap);
    ProfScope prof(DZ_KERNEL_SEQGEN, (double)m->step_bytes * c->B * ((double)plen + (double)n_new - 1.0), 0,
                   c->stream);
    // the dynamic shared-memory attribute was raised at cache creation (outside any capture)
    (void)dz_seqgen_launch(p, m->seq_bits, c->B, smem, c->stream);
    return 1;
}

// ------------------------------------------------------------ batched prefill

// Rows (sequences x prompt positions) one prefill pass holds at most; longer
// batches run in groups of sequences.
constexpr size_t PF_MAX_ROWS = 32768;

static bool prefill_eligible(const dz_cuda_cache_t* c) {
    const dz_cuda_model_t* m = c->model;
    const int D = (int)m->desc.embedding_dim, H = (int)m->desc.num_heads;
    if (H <= 0 || D % H) return false;
    const int hd = D / H;
    return hd == 32 || hd == 64 || hd == 128;
}

// Batched prefill under DZ_PREFILL_AUTO: models wide enough that their
// projections run on the tensor-core GEMM at many rows.
static bool use_batched_prefill(const dz_cuda_cache_t* c, size_t plen) {
    if (plen < 2 || !prefill_eligible(c) || c->prefill == DZ_PREFILL_TOKENS) return false;
    return c->prefill == DZ_PREFILL_BATCHED || c->model->desc.embedding_dim >= 512;
}

static size_t prefill_group(const dz_cuda_cache_t* c, size_t T) {
    size_t S = PF_MAX_ROWS / T;
    if (S < 1) S = 1;
    return S < (size_t)c->B ? S : (size_t)c->B;
}

// Row buffers for groups of prefill_group(T) sequences of T positions
// (allocated outside any stream capture; the attention kernel's shared
// memory attribute is set here too).
static int ensure_prefill(dz_cuda_cache_t* c, size_t T) {
    const size_t rows = prefill_group(c, T) * T;
    if (rows <= c->pf_rows) return DZ_OK;
    clear_graphs(c);   // graphs captured earlier point at the old buffers
    free_prefill(c);
    dz_cuda_model_t* m = c->model;
    const size_t D = m->desc.embedding_dim, F = 4 * D;
    auto al = [&](void** p, size_t bytes) { return cudaMalloc(p, bytes) == cudaSuccess; };
    size_t scratch = 0;
    for (const DevLayer& L : m->layers)
        for (const DevQMat* q : {&L.qkv, &L.q, &L.k, &L.v, &L.wo, &L.w1, &L.wg, &L.w2})
            if (q->codes) scratch = std::max(scratch, qmv_scratch_bytes(*q, (int)rows));
    bool ok = al((void**)&c->pf_hidden, rows * D * 4) && al((void**)&c->pf_q, rows * D * 4) &&
              al((void**)&c->pf_concat, rows * D * 4) && al((void**)&c->pf_attn_raw, rows * D * 4) &&
              al((void**)&c->pf_attn_norm, rows * D * 4) && al((void**)&c->pf_ff, rows * F * (m->swiglu ? 2 : 1) * 4) &&
              al((void**)&c->pf_ff_raw, rows * D * 4) && al((void**)&c->pf_rowoff, rows * 4) &&
              al(&c->pf_scratch, scratch);
    if (!ok) {
        free_prefill(c);
        return fail(DZ_E_NOMEM, "prefill buffers for %zu rows", rows);
    }
    c->pf_rows = rows;
    DZ_CUDA(cudaMemset(c->pf_scratch, 0, scratch));
    DZ_CUDA(cudaFuncSetAttribute(dz_attention_prefill_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)dz_prefill_att_smem(128)));
    DZ_CUDA(cudaFuncSetAttribute(dz_attention_prefill_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)dz_prefill_att_smem(64)));
    DZ_CUDA(cudaFuncSetAttribute(dz_attention_prefill_kernel<4, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)dz_prefill_att_smem(128)));
    DZ_CUDA(cudaFuncSetAttribute(dz_attention_prefill_kernel<2, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)dz_prefill_att_smem(64)));
    return DZ_OK;
}

// Launches enqueue_prefill makes for T positions.
static size_t prefill_launches(const dz_cuda_cache_t* c, size_t T) {
    const dz_cuda_model_t* m = c->model;
    const size_t S = prefill_group(c, T), groups = ((size_t)c->B + S - 1) / S;
    size_t n = 2 + (size_t)head_launches(m, c->B);   // row offsets, ring state, head
    for (size_t g = 0; g < groups; g++) {
        const int R = (int)(std::min((size_t)c->B, (g + 1) * S) - g * S) * (int)T;
        n += 2;   // embedding, gather
        for (const auto& L : m->layers) n += layer_launches(m, L, R);
    }
    return n;
}

// The masked full-prefix forward (model_forward_masked, src/core/
// transformer.c:527-576) on the prefill kernels: device copies of the padding
// mask [B][T] and attention mask [B][T][T] (either null) and each sequence's
// last real position + 1 [B].
struct PrefillMask {
    const uint8_t* pad = nullptr;
    const uint8_t* att = nullptr;
    const int* last = nullptr;
};

// Prefill of T positions of every sequence (ids_dev [B][ld], lens_dev [B]
// positions per sequence or null for all T) into empty rings: all positions
// of a group of sequences per layer pass, then the head on each sequence's
// last position into c->logits. With `mk`, the masked forward instead: padded
// rows zeroed after the embedding and after each norm (model_forward_hidden_
// masked, :392-519), the masked attention, the head on the last real
// position, and the rings left for the caller to reset. Returns the launches.
static int enqueue_prefill(dz_cuda_cache_t* c, const uint32_t* ids_dev, long long ld, int T, const int* lens_dev,
                           const PrefillMask* mk = nullptr) {
    dz_cuda_model_t* m = c->model;
    const int D = (int)m->desc.embedding_dim, V = (int)m->desc.vocab_size;
    const int H = m->Hl, dl = m->dl, F = m->Fl;   // this rank's heads, attention width, FFN width
    const int hd = D / (int)m->desc.num_heads, B = c->B, cap = c->cap;
    cudaStream_t st = c->stream;
    const int S = (int)prefill_group(c, (size_t)T);
    int launches = 0;
    {
        const int rows = S * T;
        dz_prefill_rowoff_kernel<<<(rows + 255) / 256, 256, 0, st>>>(c->pf_rowoff, rows, T, cap, dl);
        launches++;
    }
    for (int s0 = 0; s0 < B; s0 += S) {
        const int ns = std::min(S, B - s0), R = ns * T;
        const int* lens = lens_dev ? lens_dev + s0 : nullptr;
        const uint8_t* pad = (mk && mk->pad) ? mk->pad + (long long)s0 * T : nullptr;
        const uint8_t* att = (mk && mk->att) ? mk->att + (long long)s0 * T * T : nullptr;
        auto zero_padded = [&](float* x) {
            if (!pad) return;
            dz_zero_padded_rows_kernel<<<R, 128, 0, st>>>(x, pad, D);
            launches++;
        };
        {
            ProfScope prof(DZ_KERNEL_STEP_BEGIN, (double)R * D * 12, 0, st);
            dz_prefill_embed_kernel<<<R, 128, 0, st>>>(ids_dev + (long long)s0 * ld, ld, T, m->emb,
                                                       m->rope ? nullptr : m->pe, m->pe_rows, c->pf_hidden, D, V, lens,
                                                       mk ? nullptr : c->seen + (long long)s0 * c->seen_words,
                                                       c->seen_words);
        }
        launches++;
        zero_padded(c->pf_hidden);
        bool hidden_limbs = false;   // the previous norm wrote the limbs of the product reading c->pf_hidden
        for (size_t l = 0; l < m->layers.size(); l++) {
            DevLayer& L = m->layers[l];
            float* Kl = c->keys + l * (size_t)B * cap * dl + (size_t)s0 * cap * dl;
            float* Vl = c->values + l * (size_t)B * cap * dl + (size_t)s0 * cap * dl;
            if (L.fused_qkv) {
                QmvEpilogue ep = plain_epilogue(L.qkv, c->pf_q, dl);
                ep.nseg = 3;
                ep.seg_start[0] = 0; ep.seg_start[1] = dl; ep.seg_start[2] = 2 * dl; ep.seg_start[3] = 3 * dl;
                ep.seg_ptr[1] = Kl; ep.seg_ld[1] = 0; ep.seg_row_off[1] = c->pf_rowoff;
                ep.seg_ptr[2] = Vl; ep.seg_ld[2] = 0; ep.seg_row_off[2] = c->pf_rowoff;
                launches += launch_qmv(L.qkv, c->pf_hidden, D, R, ep, st, c->pf_scratch, c->status, hidden_limbs);
            } else {
                QmvEpilogue eq = plain_epilogue(L.q, c->pf_q, dl);
                launches += launch_qmv(L.q, c->pf_hidden, D, R, eq, st, c->pf_scratch, c->status);
                QmvEpilogue ek = plain_epilogue(L.k, Kl, 0);
                ek.seg_row_off[0] = c->pf_rowoff;
                launches += launch_qmv(L.k, c->pf_hidden, D, R, ek, st, c->pf_scratch, c->status);
                QmvEpilogue ev = plain_epilogue(L.v, Vl, 0);
                ev.seg_row_off[0] = c->pf_rowoff;
                launches += launch_qmv(L.v, c->pf_hidden, D, R, ev, st, c->pf_scratch, c->status);
            }
            if (m->rope) {
                dz_rope_prefill_kernel<<<R, 128, 0, st>>>(c->pf_q, Kl, (long long)cap * dl, T, dl, hd, m->rope_tab,
                                                          m->pe_rows);
                launches++;
            }
            {
                const double ctx_pairs = (double)ns * H * T * (T + 1) / 2.0;
                ProfScope prof(DZ_KERNEL_ATTENTION, 8.0 * (double)R * dl + 8.0 * (double)ns * T * dl,
                               4.0 * ctx_pairs * hd, st);
                const dim3 grid((unsigned)((T + PF_QT - 1) / PF_QT), (unsigned)H, (unsigned)ns);
                const size_t smem = dz_prefill_att_smem(hd);
                if ((!mk || (!pad && !att)) && (hd == 128 || hd == 64) && prefill_attn_tensor_cores()) {
                    dz_pfattn_launch(c->pf_q, Kl, Vl, lens, c->pf_concat, T, dl, cap, hd, H, ns, st);
                } else if (mk) {
                    if (hd == 128)
                        dz_attention_prefill_kernel<4, true><<<grid, PF_THREADS, smem, st>>>(
                            c->pf_q, Kl, Vl, nullptr, c->pf_concat, T, dl, cap, pad, att);
                    else if (hd == 64)
                        dz_attention_prefill_kernel<2, true><<<grid, PF_THREADS, smem, st>>>(
                            c->pf_q, Kl, Vl, nullptr, c->pf_concat, T, dl, cap, pad, att);
                    else
                        dz_attention_prefill_kernel<1, true><<<grid, PF_THREADS, smem, st>>>(
                            c->pf_q, Kl, Vl, nullptr, c->pf_concat, T, dl, cap, pad, att);
                } else if (hd == 128)
                    dz_attention_prefill_kernel<4><<<grid, PF_THREADS, smem, st>>>(c->pf_q, Kl, Vl, lens,
                                                                                  c->pf_concat, T, dl, cap);
                else if (hd == 64)
                    dz_attention_prefill_kernel<2><<<grid, PF_THREADS, smem, st>>>(c->pf_q, Kl, Vl, lens,
                                                                                  c->pf_concat, T, dl, cap);
                else
                    dz_attention_prefill_kernel<1><<<grid, PF_THREADS, smem, st>>>(c->pf_q, Kl, Vl, lens,
                                                                                  c->pf_concat, T, dl, cap);
            }
            launches++;
            QmvEpilogue eo = plain_epilogue(L.wo, c->pf_attn_raw, D);
            launches += launch_qmv(L.wo, c->pf_concat, dl, R, eo, st, c->pf_scratch, c->status);
            tp_allreduce(m, c->pf_attn_raw, (size_t)R * D, st);
            // (no fusion with padded rows: they are zeroed after the norm)
            const bool ffn_limbs = !pad && norm_limbs_ok(m, L.w1, R, D) &&
                                   (!L.wg.codes || norm_limbs_ok(m, L.wg, R, D)) &&
                                   norm_limbs_aligned(c->pf_attn_raw, c->pf_hidden, L.g1, L.be1, c->pf_attn_norm);
            {
                ProfScope prof(DZ_KERNEL_LAYERNORM, 12.0 * R * D + 8.0 * D + (ffn_limbs ? 3.0 * R * D : 0.0), 0, st);
                if (ffn_limbs)
                    launch_norm_limbs(c->pf_attn_raw, c->pf_hidden, L.g1, L.be1, c->pf_attn_norm, R, D, L.w1,
                                      c->pf_scratch, st);
                else
                    launch_norm(m, c->pf_attn_raw, c->pf_hidden, L.g1, L.be1, c->pf_attn_norm, R, D, st);
            }
            launches++;
            zero_padded(c->pf_attn_norm);
            const long long ldf = m->swiglu ? 2LL * F : F;
            launches += launch_ffn_up(m, L, c->pf_attn_norm, D, R, c->pf_ff, ldf, F, st, c->pf_scratch, c->status,
                                      ffn_limbs);
            QmvEpilogue e2 = plain_epilogue(L.w2, c->pf_ff_raw, D);
            if (m->tp_rank == 0) {
                e2.bias = L.b2;
                e2.residual = c->pf_attn_norm;
                e2.ld_res = D;
            }
            launches += launch_qmv(L.w2, c->pf_ff, ldf, R, e2, st, c->pf_scratch, c->status);
            tp_allreduce(m, c->pf_ff_raw, (size_t)R * D, st);
            // the next layer's fused QKV reads c->pf_hidden (the head reads
            // the gathered last positions instead)
            const DevQMat* next =
                l + 1 < m->layers.size() && m->layers[l + 1].fused_qkv ? &m->layers[l + 1].qkv : nullptr;
            hidden_limbs = !pad && next && norm_limbs_ok(m, *next, R, D) &&
                           norm_limbs_aligned(c->pf_ff_raw, nullptr, L.g2, L.be2, c->pf_hidden);
            {
                ProfScope prof(DZ_KERNEL_LAYERNORM, 8.0 * R * D + 8.0 * D + (hidden_limbs ? 3.0 * R * D : 0.0), 0, st);
                if (hidden_limbs)
                    launch_norm_limbs(c->pf_ff_raw, nullptr, L.g2, L.be2, c->pf_hidden, R, D, *next, c->pf_scratch,
                                      st);
                else
                    launch_norm(m, c->pf_ff_raw, nullptr, L.g2, L.be2, c->pf_hidden, R, D, st);
            }
            launches++;
            zero_padded(c->pf_hidden);
        }
        dz_prefill_gather_kernel<<<ns, 256, 0, st>>>(c->pf_hidden, mk ? mk->last + s0 : lens, T, D,
                                                     c->hidden + (size_t)s0 * D);
        launches++;
    }
    if (!mk) {
        dz_prefill_ring_kernel<<<(B + 255) / 256, 256, 0, st>>>(c->start, c->length, c->total, lens_dev, T, B);
        launches++;
    }
    launches += launch_head(c, st);
    return launches;
}

// Generation jobs above this many launches are enqueued directly instead of
// through a cached CUDA graph.
constexpr size_t GRAPH_MAX_LAUNCHES = 40000;

// The whole generation loop, enqueued on the cache's stream. Returns launches.
static int enqueue_generate(dz_cuda_cache_t* c, const uint32_t* prompts, size_t plen, size_t n_new,
                            const dz_sampling_t* s, const uint64_t* seeds, uint32_t* out,
                            const GenControls* ctl = nullptr) {
    int launches = 0;
    const bool controls = ctl && ctl->on;
    if (!controls && use_seqgen(c, s)) {
        dz_reset_kernel<<<(c->B + 255) / 256, 256, 0, c->stream>>>(c->start, c->length, c->total, nullptr, c->B);
        c->seen_valid = false;   // the fused kernel keeps no token history
        return 1 + launch_seqgen(c, prompts, plen, n_new, s, seeds, out);
    }
    const bool sampled = seeds != nullptr;
    if (sampled) {
        dz_seed_kernel<<<(c->B + 127) / 128, 128, 0, c->stream>>>(seeds, c->rng, c->B, DZ_RNG_STREAM_SAMPLING);
        launches++;
    }
    dz_reset_kernel<<<(c->B + 255) / 256, 256, 0, c->stream>>>(c->start, c->length, c->total, nullptr, c->B);
    dz_seen_clear_kernel<<<dim3((unsigned)((c->seen_words + 255) / 256), (unsigned)c->B), 256, 0, c->stream>>>(
        c->seen, c->seen_words, nullptr);
    c->seen_valid = true;
    launches += 2;
    SelectControls sc = select_controls(c, ctl, true);
    if (controls) {
        dz_gen_init_kernel<<<(c->B + 127) / 128, 128, 0, c->stream>>>(c->gen_state, c->B);
        launches++;
    }
    if (use_batched_prefill(c, plen)) {
        launches += enqueue_prefill(c, prompts, (long long)plen, (int)plen, nullptr);
    } else {
        for (size_t t = 0; t < plen; t++) launches += enqueue_step(c, prompts + t, (long long)plen);
    }
    for (size_t i = 0; i < n_new; i++) {
        launches += enqueue_select(c, s, sampled ? c->rng : nullptr, out + i, (long long)n_new, c->tok,
                                   controls ? &sc : nullptr);
        if (i + 1 < n_new) launches += enqueue_step(c, c->tok, 1);
    }
    return launches;
}

extern "C" size_t dz_cuda_generate_launches(const dz_cuda_cache_t* c, size_t plen, size_t n_new,
                                            const dz_sampling_t* s) {
    if (!c) return 0;
    const dz_cuda_model_t* m = c->model;
    if (use_seqgen(c, s)) return 2;
    const int B = (int)c->B;
    size_t step = 1 + (size_t)head_launches(m, B);   // step begin, head
    for (const auto& L : m->layers) step += layer_launches(m, L, B);
    const size_t seeded = (s && s->strategy != 0 && s->temperature > 0.0f) ? 1 : 0;
    const size_t prefill = use_batched_prefill(c, plen) ? prefill_launches(c, plen) : plen * step;
    return seeded + 2 + prefill + n_new + (n_new ? n_new - 1 : 0) * step;   // + ring reset, history clear
}

static int generate_async(dz_cuda_cache_t* c, const uint32_t* prompts, size_t plen, size_t n_new,
                          const dz_sampling_t* s, const uint64_t* seeds, uint32_t* out, const GenControls* ctl) {
    if (!c || !prompts || !out || plen == 0 || n_new == 0)
        return fail(DZ_E_INVALID, "generate: null buffer or empty prompt/decode length");
    int rc = check_sampling(c, s);
    if (rc) return rc;
    DeviceGuard g(c->model->device);
    if ((rc = ensure_masked(c, s))) return rc;
    const bool fused = !(ctl && ctl->on) && use_seqgen(c, s);
    if (!fused && use_batched_prefill(c, plen) && (rc = ensure_prefill(c, plen))) return rc;
    c->seen_valid = !fused;   // the fused kernel keeps no token history
    if (s && s->n_masked)
        DZ_CUDA(cudaMemcpyAsync(c->masked, s->masked_ids, s->n_masked * 4, cudaMemcpyHostToDevice, c->stream));
    const bool sampled = seeds && s && s->strategy != 0 && s->temperature > 0.0f;
    GenKey key;
    key.plen = plen;
    key.n_new = n_new;
    key.strategy = s ? s->strategy : 0;
    key.temperature = s ? s->temperature : 0.0f;
    key.top_p = s ? s->top_p : 0.0f;
    key.top_k = s ? s->top_k : 0;
    key.masked = s && s->n_masked ? std::vector<uint32_t>(s->masked_ids, s->masked_ids + s->n_masked)
                                  : std::vector<uint32_t>();
    if (ctl) key.ctl = *ctl;
    key.prompts = prompts;
    key.seeds = sampled ? seeds : nullptr;
    key.out = out;
    if (dz_cuda_generate_launches(c, plen, n_new, s) > GRAPH_MAX_LAUNCHES) {
        // jobs this long launch directly: a graph of this many nodes costs more to build than it saves
        enqueue_generate(c, prompts, plen, n_new, s, sampled ? seeds : nullptr, out, ctl);
        DZ_CUDA(cudaGetLastError());
        return DZ_OK;
    }
    auto it = c->gen_graphs.find(key);
    if (it == c->gen_graphs.end()) {
        cudaGraph_t graph;
        DZ_CUDA(cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeThreadLocal));
        enqueue_generate(c, prompts, plen, n_new, s, sampled ? seeds : nullptr, out, ctl);
        cudaError_t e = cudaStreamEndCapture(c->stream, &graph);
        if (e != cudaSuccess) return fail(DZ_E_DEVICE, "capture: %s", cudaGetErrorString(e));
        cudaGraphExec_t exec;
        e = cudaGraphInstantiate(&exec, graph, 0);
        cudaGraphDestroy(graph);
        if (e != cudaSuccess) return fail(DZ_E_DEVICE, "instantiate: %s", cudaGetErrorString(e));
        it = c->gen_graphs.emplace(key, exec).first;
    }
    DZ_CUDA(cudaGraphLaunch(it->second, c->stream));
    return DZ_OK;
}

extern "C" int dz_cuda_generate_async(dz_cuda_cache_t* c, const uint32_t* prompts, size_t plen, size_t n_new,
                                      const dz_sampling_t* s, const uint64_t* seeds, uint32_t* out) {
    return generate_async(c, prompts, plen, n_new, s, seeds, out, nullptr);
}

// The controls of a generation on the host (validated the way
// options_are_valid does, src/cli/generation.c:84-112) and their stop
// sequences copied to the device (buffers grown outside any capture).
static int prepare_controls(dz_cuda_cache_t* c, const dz_generation_controls_t* in, GenControls* out) {
    out->on = false;
    if (!in) return DZ_OK;
    const uint32_t V = (uint32_t)c->model->desc.vocab_size;
    if (!(in->repetition_penalty >= 1.0f) || !(in->repetition_penalty <= 3.402823466e38f))
        return fail(DZ_E_INVALID, "repetition penalty must be finite and >= 1");
    if (in->n_stops > 64 || (in->n_stops && (!in->stop_tokens || !in->stop_lengths)))
        return fail(DZ_E_INVALID, "stop sequences: at most 64, with their tokens and lengths");
    if (in->minimum_new_tokens > (size_t)1 << 30) return fail(DZ_E_INVALID, "minimum_new_tokens too large");
    out->on = true;
    out->penalty = in->repetition_penalty;
    out->eos_id = in->eos_id;
    out->mask_from = in->mask_from;
    out->min_new = (int)in->minimum_new_tokens;
    out->stop_tok.clear();
    out->stop_off.assign(1, 0);
    for (size_t q = 0; q < in->n_stops; q++) {
        const size_t len = in->stop_lengths[q];
        if (len == 0 || len > 256) return fail(DZ_E_INVALID, "stop sequence %zu: length must be 1..256", q);
        for (size_t j = 0; j < len; j++) {
            const uint32_t t = in->stop_tokens[out->stop_tok.size()];
            if (t >= V) return fail(DZ_E_INVALID, "stop sequence %zu: token %u out of the vocabulary", q, t);
            out->stop_tok.push_back(t);
        }
        out->stop_off.push_back((int)out->stop_tok.size());
    }
    const size_t nt = std::max<size_t>(1, out->stop_tok.size()), no = out->stop_off.size();
    if (nt > c->stop_tok_cap || no > c->stop_off_cap) {
        clear_graphs(c);   // captured graphs hold the old pointers
        cudaFree(c->stop_tok);
        cudaFree(c->stop_off);
        c->stop_tok = nullptr;
        c->stop_off = nullptr;
        c->stop_tok_cap = c->stop_off_cap = 0;
        DZ_CUDA(cudaMalloc(&c->stop_tok, std::max<size_t>(nt, 64) * 4));
        DZ_CUDA(cudaMalloc(&c->stop_off, std::max<size_t>(no, 65) * 4));
        c->stop_tok_cap = std::max<size_t>(nt, 64);
        c->stop_off_cap = std::max<size_t>(no, 65);
    }
    if (!out->stop_tok.empty())
        DZ_CUDA(cudaMemcpyAsync(c->stop_tok, out->stop_tok.data(), out->stop_tok.size() * 4, cudaMemcpyHostToDevice,
                                c->stream));
    DZ_CUDA(cudaMemcpyAsync(c->stop_off, out->stop_off.data(), out->stop_off.size() * 4, cudaMemcpyHostToDevice,
                            c->stream));
    return DZ_OK;
}

extern "C" int dz_cuda_generate(dz_cuda_cache_t* c, const uint32_t* prompts, size_t plen, size_t n_new,
                                const dz_sampling_t* s, const uint64_t* seeds, uint32_t* out_tokens) {
    return dz_cuda_generate_ex(c, prompts, plen, n_new, s, nullptr, seeds, out_tokens, nullptr);
}

extern "C" int dz_cuda_generate_ex(dz_cuda_cache_t* c, const uint32_t* prompts, size_t plen, size_t n_new,
                                   const dz_sampling_t* s, const dz_generation_controls_t* controls,
                                   const uint64_t* seeds, uint32_t* out_tokens, dz_generation_result_t* results) {
    if (!c || !prompts || !out_tokens || plen == 0 || n_new == 0)
        return fail(DZ_E_INVALID, "generate: null buffer or empty prompt/decode length");
    if (plen > (size_t)c->cap) return fail(DZ_E_INVALID, "prompt longer than the cache capacity");
    DeviceGuard g(c->model->device);
    const size_t B = c->B;
    if (B * plen > c->gen_prompts_cap) {
        clear_graphs(c);
        cudaFree(c->gen_prompts);
        c->gen_prompts = nullptr;
        c->gen_prompts_cap = 0;
        DZ_CUDA(cudaMalloc(&c->gen_prompts, B * plen * 4));
        c->gen_prompts_cap = B * plen;
    }
    if (B * n_new > c->gen_out_cap) {
        clear_graphs(c);
        cudaFree(c->gen_out);
        c->gen_out = nullptr;
        c->gen_out_cap = 0;
        DZ_CUDA(cudaMalloc(&c->gen_out, B * n_new * 4));
        c->gen_out_cap = B * n_new;
    }
    DZ_CUDA(cudaMemcpyAsync(c->gen_prompts, prompts, B * plen * 4, cudaMemcpyHostToDevice, c->stream));
    if (seeds) DZ_CUDA(cudaMemcpyAsync(c->gen_seeds, seeds, B * 8, cudaMemcpyHostToDevice, c->stream));
    GenControls ctl;
    int rc = prepare_controls(c, controls, &ctl);
    if (rc) return rc;
    rc = generate_async(c, c->gen_prompts, plen, n_new, s, seeds ? c->gen_seeds : nullptr, c->gen_out,
                        ctl.on ? &ctl : nullptr);
    if (rc) return rc;
    DZ_CUDA(cudaMemcpyAsync(out_tokens, c->gen_out, B * n_new * 4, cudaMemcpyDeviceToHost, c->stream));
    if (ctl.on && results)
        DZ_CUDA(cudaMemcpyAsync(c->host_gen, c->gen_state, B * DZ_GEN_WORDS * 4, cudaMemcpyDeviceToHost, c->stream));
    DZ_CUDA(cudaMemcpyAsync(c->host_status, c->status, 4, cudaMemcpyDeviceToHost, c->stream));
    DZ_CUDA(cudaStreamSynchronize(c->stream));
    if (*c->host_status != 0) {
        cudaMemsetAsync(c->status, 0, 4, c->stream);
        cudaStreamSynchronize(c->stream);
        return fail(DZ_E_TIMEOUT, "generate: a weight-copy wait gave up on the device");
    }
    if (results) {
        for (size_t b = 0; b < B; b++) {
            dz_generation_result_t& r = results[b];
            if (ctl.on) {
                const uint32_t* gsv = c->host_gen + b * DZ_GEN_WORDS;
                r.new_count = gsv[GEN_NEW];
                r.emitted_count = gsv[GEN_EMITTED];
                r.stopped_on_eos = gsv[GEN_EOS];
                r.stopped_on_stop_sequence = gsv[GEN_STOP];
                r.stop_sequence_index = gsv[GEN_STOP_INDEX];
            } else {
                r.new_count = r.emitted_count = (uint32_t)n_new;
                r.stopped_on_eos = r.stopped_on_stop_sequence = 0;
                r.stop_sequence_index = 0xffffffffu;
            }
        }
    }
    return DZ_OK;
}

extern "C" int dz_cuda_cache_set_prefill(dz_cuda_cache_t* c, int mode) {
    if (!c || mode < DZ_PREFILL_AUTO || mode > DZ_PREFILL_BATCHED) return fail(DZ_E_INVALID, "bad prefill mode");
    if (mode == DZ_PREFILL_BATCHED && !prefill_eligible(c))
        return fail(DZ_E_UNSUPPORTED, "batched prefill needs a head dimension of 32, 64 or 128");
    if (mode != c->prefill) {
        DeviceGuard g(c->model->device);
        clear_graphs(c);
    }
    c->prefill = mode;
    return DZ_OK;
}

extern "C" int dz_cuda_prefill(dz_cuda_cache_t* c, const uint32_t* ids, const uint32_t* lens, size_t prompt_len,
                               float* logits_out) {
    if (!c || !ids || prompt_len == 0) return fail(DZ_E_INVALID, "prefill: null ids or empty prompt");
    if (prompt_len > (size_t)c->cap) return fail(DZ_E_INVALID, "prefill: prompt longer than the cache capacity");
    if (!prefill_eligible(c)) return fail(DZ_E_UNSUPPORTED, "batched prefill needs a head dimension of 32, 64 or 128");
    const size_t B = c->B;
    std::vector<int> lv;
    if (lens) {
        lv.resize(B);
        for (size_t b = 0; b < B; b++) {
            if (lens[b] == 0 || lens[b] > prompt_len) return fail(DZ_E_INVALID, "prefill: lens must be 1..prompt_len");
            lv[b] = (int)lens[b];
        }
    }
    DeviceGuard g(c->model->device);
    int rc = ensure_prefill(c, prompt_len);
    if (rc) return rc;
    if (B * prompt_len > c->pf_ids_cap) {
        cudaFree(c->pf_ids);
        cudaFree(c->pf_lens);
        c->pf_ids = nullptr;
        c->pf_lens = nullptr;
        c->pf_ids_cap = 0;
        DZ_CUDA(cudaMalloc(&c->pf_ids, B * prompt_len * 4));
        DZ_CUDA(cudaMalloc(&c->pf_lens, B * 4));
        c->pf_ids_cap = B * prompt_len;
    }
    DZ_CUDA(cudaMemcpyAsync(c->pf_ids, ids, B * prompt_len * 4, cudaMemcpyHostToDevice, c->stream));
    if (lens) DZ_CUDA(cudaMemcpyAsync(c->pf_lens, lv.data(), B * 4, cudaMemcpyHostToDevice, c->stream));
    dz_reset_kernel<<<(c->B + 255) / 256, 256, 0, c->stream>>>(c->start, c->length, c->total, nullptr, c->B);
    dz_seen_clear_kernel<<<dim3((unsigned)((c->seen_words + 255) / 256), (unsigned)c->B), 256, 0, c->stream>>>(
        c->seen, c->seen_words, nullptr);
    c->seen_valid = true;
    enqueue_prefill(c, c->pf_ids, (long long)prompt_len, (int)prompt_len, lens ? c->pf_lens : nullptr);
    DZ_CUDA(cudaGetLastError());
    if (logits_out)
        DZ_CUDA(cudaMemcpyAsync(logits_out, c->logits, B * c->model->desc.vocab_size * 4, cudaMemcpyDeviceToHost,
                                c->stream));
    DZ_CUDA(cudaStreamSynchronize(c->stream));
    return DZ_OK;
}

extern "C" int dz_cuda_forward_masked(dz_cuda_cache_t* c, const uint32_t* ids, size_t seq_len,
                                      const uint8_t* padding_mask, const uint8_t* attention_mask,
                                      float* logits_out) {
    if (!c || !ids || !logits_out || seq_len == 0)
        return fail(DZ_E_INVALID, "forward_masked: null ids or logits, or seq_len 0");
    const dz_cuda_model_t* m = c->model;
    if (seq_len > m->desc.max_seq_len) return fail(DZ_E_INVALID, "forward_masked: seq_len above max_seq_len");
    if (seq_len > (size_t)c->cap) return fail(DZ_E_INVALID, "forward_masked: seq_len above the cache capacity");
    if (!prefill_eligible(c))
        return fail(DZ_E_UNSUPPORTED, "the masked forward needs a head dimension of 32, 64 or 128");
    const size_t B = c->B, T = seq_len;
    // the last real position of each sequence (model_forward_masked,
    // src/core/transformer.c:535-545): a padding mask with none is rejected
    std::vector<int> last(B, (int)T);
    if (padding_mask) {
        for (size_t b = 0; b < B; b++) {
            int l = 0;
            for (size_t i = 0; i < T; i++)
                if (padding_mask[b * T + i]) l = (int)i + 1;
            if (l == 0) return fail(DZ_E_INVALID, "forward_masked: sequence %zu has no real position", b);
            last[b] = l;
        }
    }
    DeviceGuard g(m->device);
    int rc = ensure_prefill(c, T);
    if (rc) return rc;
    if (B * T > c->pf_ids_cap) {
        cudaFree(c->pf_ids);
        cudaFree(c->pf_lens);
        c->pf_ids = nullptr;
        c->pf_lens = nullptr;
        c->pf_ids_cap = 0;
        DZ_CUDA(cudaMalloc(&c->pf_ids, B * T * 4));
        DZ_CUDA(cudaMalloc(&c->pf_lens, B * 4));
        c->pf_ids_cap = B * T;
    }
    const size_t pad_bytes = padding_mask ? B * T : 0, att_bytes = attention_mask ? B * T * T : 0;
    const size_t mk_bytes = ((pad_bytes + 15) & ~(size_t)15) + att_bytes;
    if (mk_bytes > c->mk_cap) {
        cudaFree(c->mk_buf);
        c->mk_buf = nullptr;
        c->mk_cap = 0;
        DZ_CUDA(cudaMalloc(&c->mk_buf, mk_bytes));
        c->mk_cap = mk_bytes;
    }
    PrefillMask mk;
    DZ_CUDA(cudaMemcpyAsync(c->pf_ids, ids, B * T * 4, cudaMemcpyHostToDevice, c->stream));
    DZ_CUDA(cudaMemcpyAsync(c->pf_lens, last.data(), B * 4, cudaMemcpyHostToDevice, c->stream));
    mk.last = c->pf_lens;
    if (padding_mask) {
        DZ_CUDA(cudaMemcpyAsync(c->mk_buf, padding_mask, pad_bytes, cudaMemcpyHostToDevice, c->stream));
        mk.pad = c->mk_buf;
    }
    if (attention_mask) {
        uint8_t* d = c->mk_buf + ((pad_bytes + 15) & ~(size_t)15);
        DZ_CUDA(cudaMemcpyAsync(d, attention_mask, att_bytes, cudaMemcpyHostToDevice, c->stream));
        mk.att = d;
    }
    enqueue_prefill(c, c->pf_ids, (long long)T, (int)T, nullptr, &mk);
    // the rings served as working storage: leave every sequence empty
    dz_reset_kernel<<<(c->B + 255) / 256, 256, 0, c->stream>>>(c->start, c->length, c->total, nullptr, c->B);
    dz_seen_clear_kernel<<<dim3((unsigned)((c->seen_words + 255) / 256), (unsigned)c->B), 256, 0, c->stream>>>(
        c->seen, c->seen_words, nullptr);
    c->seen_valid = true;
    DZ_CUDA(cudaGetLastError());
    DZ_CUDA(cudaMemcpyAsync(logits_out, c->logits, B * m->desc.vocab_size * 4, cudaMemcpyDeviceToHost, c->stream));
    DZ_CUDA(cudaStreamSynchronize(c->stream));
    return DZ_OK;
}

extern "C" int dz_cuda_cache_set_path(dz_cuda_cache_t* c, int path) {
    if (!c || path < DZ_PATH_AUTO || path > DZ_PATH_FUSED) return fail(DZ_E_INVALID, "bad path");
    if (path == DZ_PATH_FUSED && !c->model->seq_ok)
        return fail(DZ_E_UNSUPPORTED, "the fused path cannot run this model");
    DeviceGuard g(c->model->device);
    clear_graphs(c);
    c->path = path;
    return DZ_OK;
}

extern "C" int dz_cuda_cache_uses_fused(const dz_cuda_cache_t* c, const dz_sampling_t* s) {
    return c ? (int)use_seqgen(c, s) : 0;
}

extern "C" int dz_cuda_profile_generate(dz_cuda_cache_t* c, const uint32_t* prompts, size_t plen, size_t n_new,
                                        const dz_sampling_t* s, const uint64_t* seeds, uint32_t* out,
                                        dz_kernel_stat_t* stats, size_t n_stats) {
    if (!c || !prompts || !out || !stats || plen == 0 || n_new == 0)
        return fail(DZ_E_INVALID, "profile_generate: null buffer or empty lengths");
    int rc = check_sampling(c, s);
    if (rc) return rc;
    DeviceGuard g(c->model->device);
    if ((rc = ensure_masked(c, s))) return rc;
    if (s && s->n_masked)
        DZ_CUDA(cudaMemcpyAsync(c->masked, s->masked_ids, s->n_masked * 4, cudaMemcpyHostToDevice, c->stream));
    const bool sampled = seeds && s && s->strategy != 0 && s->temperature > 0.0f;
    std::vector<ProfRec> recs;
    DZ_CUDA(cudaMemsetAsync(c->phase_ns, 0, SEQ_PHASES * 8, c->stream));
    g_prof = &recs;
    // eager launches, each bracketed by events; the decode attention's byte
    // count uses the mean context of the decode steps it serves: every step
    // of a token-by-token run, or the draws after a batched prefill (contexts
    // plen + 1 .. plen + n_new - 1); all sequences move in step
    const dz_cuda_model_t* m = c->model;
    const double D = (double)m->dl;   // this rank's K / V width
    const double total_steps = (double)plen + (double)(n_new - 1);
    double mean_ctx = use_batched_prefill(c, plen) ? (double)plen + (double)n_new / 2.0 : (total_steps + 1.0) / 2.0;
    if (mean_ctx > c->cap) mean_ctx = c->cap;
    c->prof_ctx_bytes_per_layer = 8.0 * D * mean_ctx * c->B;
    c->prof_ctx_flops_per_layer = 4.0 * D * mean_ctx * c->B;
    enqueue_generate(c, prompts, plen, n_new, s, sampled ? seeds : nullptr, out);
    g_prof = nullptr;
    cudaError_t e = cudaStreamSynchronize(c->stream);
    for (size_t k = 0; k < n_stats; k++) {
        stats[k].kind = (uint32_t)k;
        stats[k].launches = 0;
        stats[k].total_ms = 0;
        stats[k].bytes = 0;
        stats[k].flops = 0;
    }
    for (auto& r : recs) {
        float ms = 0;
        if (e == cudaSuccess) e = cudaEventElapsedTime(&ms, r.a, r.b);
        if (r.kind >= 0 && (size_t)r.kind < n_stats) {
            stats[r.kind].launches++;
            stats[r.kind].total_ms += ms;
            stats[r.kind].bytes += r.bytes;
            stats[r.kind].flops += r.flops;
        }
        cudaEventDestroy(r.a);
        cudaEventDestroy(r.b);
    }
    if (e != cudaSuccess) return fail(DZ_E_DEVICE, "profile: %s", cudaGetErrorString(e));
    if (use_seqgen(c, s) && n_stats > (size_t)DZ_PHASE_EMBED) {
        unsigned long long ph[SEQ_PHASES];
        DZ_CUDA(cudaMemcpy(ph, c->phase_ns, sizeof(ph), cudaMemcpyDeviceToHost));
        for (int k = 0; k < SEQ_PHASES && (size_t)(DZ_PHASE_EMBED + k) < n_stats; k++) {
            stats[DZ_PHASE_EMBED + k].launches = 0;
            stats[DZ_PHASE_EMBED + k].total_ms = (double)ph[k] * 1e-6;
        }
    }
    return DZ_OK;
}

// ------------------------------------------------ allocation-free matmul

// Scratch of dz_cuda_matmul_quantized_noalloc, laid out as every product
// scratch (qmv_scratch_bytes): the tensor-core GEMV's per-tile counters, then
// the activation split or limbs and the GEMV's partial sums. Every GPU that
// loads this library holds it until the process exits. It is shared by all
// calls on a device and keeps the last call's contents: the kernels overwrite
// every byte of split, limbs and partials that they then read, and each call
// zeroes the counter block before its kernels run, since the GEMV relies on
// counters that start at zero.
static __device__ __align__(256) unsigned char g_noalloc_scratch[DZ_NOALLOC_SCRATCH_BYTES];

static std::mutex g_noalloc_mutex;
static void* g_noalloc_addr[256];   // device address of g_noalloc_scratch, per device ordinal

// The array's device address for `device` (current at the call). In host code
// the symbol names a host-side stand-in, not device memory, so the address is
// looked up once per device and cached.
static int noalloc_scratch(int device, void** out) {
    std::lock_guard<std::mutex> lock(g_noalloc_mutex);
    if (device < 0 || device >= 256) return fail(DZ_E_INVALID, "device ordinal %d out of range", device);
    if (!g_noalloc_addr[device]) {
        void* addr = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&addr, g_noalloc_scratch);
        if (e != cudaSuccess || !addr)
            return fail(DZ_E_DEVICE, "cudaGetSymbolAddress(static scratch) on device %d: %s", device,
                        cudaGetErrorString(e));
        g_noalloc_addr[device] = addr;
    }
    *out = g_noalloc_addr[device];
    return DZ_OK;
}

extern "C" int dz_cuda_matmul_quantized_noalloc(const float* A, const dz_cuda_qmatrix_t* q, float* C, size_t m,
                                                size_t k, void* stream) {
    if (!q || !A || !C || m == 0 || k != (size_t)q->m.K || m > (1u << 24))
        return fail(DZ_E_INVALID, "matmul_quantized_noalloc: bad arguments (k must equal the matrix rows)");
    // a fixed budget: no split-K partials (sizing and launch alike)
    struct NoSplit {
        NoSplit() { g_no_split_k = true; }
        ~NoSplit() { g_no_split_k = false; }
    } no_split;
    const size_t need = qmv_scratch_bytes(q->m, (int)m);
    if (need > (size_t)DZ_NOALLOC_SCRATCH_BYTES)
        return fail(DZ_E_INVALID,
                    "matmul_quantized_noalloc: m=%zu rows x k=%zu need %zu bytes of scratch, above the static "
                    "limit of %u bytes",
                    m, k, need, (unsigned)DZ_NOALLOC_SCRATCH_BYTES);
    DeviceGuard g(q->device);
    if (!g.ok) return fail(DZ_E_DEVICE, "cannot select device %d", q->device);
    void* scratch = nullptr;
    int rc = noalloc_scratch(q->device, &scratch);
    if (rc) return rc;
    // counters from an earlier call that stopped part-way must not leak into this one
    DZ_CUDA(cudaMemsetAsync(scratch, 0, SCRATCH_COUNTERS, (cudaStream_t)stream));
    QmvEpilogue ep = plain_epilogue(q->m, C, q->m.N);
    launch_qmv(q->m, A, (long long)k, (int)m, ep, (cudaStream_t)stream, scratch, q->status);
    DZ_CUDA(cudaGetLastError());
    return DZ_OK;
}
