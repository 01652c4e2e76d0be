// Fused generation kernel for small models: one CTA runs a whole sequence -
// prompt prefill, every decode step, every layer, the vocabulary head and the
// draw - without leaving the kernel. It is the same arithmetic as the layered
// path (qmv.cuh, decode.cuh, select.cuh: src/core/transformer.c:686-858,
// src/cli/sampling.c:38-207, src/cli/generation.c:231-295), scheduled for
// models whose every projection fits a shared-memory buffer (d = 128 at INT4
// or INT8: 32 / 64 KB per matrix).
//
// Weights stream from L2/HBM into two shared-memory buffers with TMA bulk
// copies (cp.async.bulk ... mbarrier::complete_tx): while the CTA computes
// matrix i from one buffer, matrix i+1 lands in the other. One thread issues
// the copies; waits on the mbarriers are bounded and, if one gives up, the CTA
// records DZ_SEQ_TIMEOUT in the status word, lets its copies in flight land and
// returns.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

#include "qmma.cuh"
#include "qmv.cuh"
#include "select.cuh"

namespace dz {

constexpr int SEQ_THREADS = 512;
constexpr int SEQ_WARPS = SEQ_THREADS / 32;
constexpr unsigned SEQ_WAIT_LIMIT = 1u << 30;  // poll bound behind the time bound
constexpr uint64_t SEQ_WAIT_NS = 1000000000ull;  // a wait gives up after ~1 s
constexpr int DZ_SEQ_TIMEOUT = 1;

// One matrix as the fused kernel streams it: a contiguous blob of
// [codes (strip layout) | column scales (Np floats) | extras], each section
// 16-byte aligned. Extras: the bias of W1 / W2 / head, and for W_o and W2 the
// gamma and beta of the LayerNorm that follows them. The TMA copy brings the
// whole blob into shared memory, so epilogues read nothing from global memory.
struct SeqMat {
    const uint8_t* blob;       // codes in the MMA-fragment layout (qmma.cuh) first
    int K, N, nkg, ntiles;
    unsigned bytes;            // whole blob
    unsigned scale_off;        // byte offset of the column scales
    unsigned bias_off;         // byte offset of the bias (0: none)
    unsigned gamma_off;        // byte offset of gamma, beta follows at +4*D bytes (0: none)
};

struct SeqLayer {
    SeqMat qkv, wo, w1, w2;
};

struct SeqParams {
    const SeqLayer* layers;
    int L, D, H, V, cap, bits;
    SeqMat head;
    const float* emb;
    const float* pe;
    long long pe_rows;
    const float* out_bias;
    float* keys;               // [L][B][cap][D]
    float* values;
    int* start;                // ring state per sequence, read at entry, written at exit
    int* length;
    long long* total;
    const uint32_t* prompts;   // [B][plen]
    int plen;
    uint32_t* out;             // [B][n_new]
    int n_new;
    const uint64_t* seeds;     // [B] or nullptr (greedy)
    int strategy;
    float temperature;
    int top_k;
    float top_p;
    const uint32_t* masked;
    int n_masked;
    int* status;
    int buf_bytes;             // bytes of each weight buffer
    int B;
    unsigned long long* phase_ns;  // optional [SEQ_PHASES]: CTA 0 accumulates time per phase
    int kv_smem;               // stage each layer's K/V rows in shared memory
};

enum { SEQ_PH_EMBED = 0, SEQ_PH_WAIT, SEQ_PH_QMV, SEQ_PH_ATTENTION, SEQ_PH_NORM, SEQ_PH_SELECT, SEQ_PHASES };

// ----------------------------------------------------------- PTX helpers

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return done != 0;
}

__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Phase clock of CTA 0, thread 0 (profiling only).
struct SeqClock {
    unsigned long long* acc;
    uint64_t t;
    __device__ explicit SeqClock(unsigned long long* a) : acc(blockIdx.x == 0 && threadIdx.x == 0 ? a : nullptr) {
        t = acc ? global_ns() : 0;
    }
    __device__ void mark(int phase) {
        if (!acc) return;
        const uint64_t n = global_ns();
        acc[phase] += n - t;
        t = n;
    }
};

// Bounded wait (about one second); returns false when the limit ran out. The
// timer is read only after the first tries fail (a global-timer read costs far
// more than a try_wait that succeeds).
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
#pragma unroll 1
    for (int i = 0; i < 4; i++)
        if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_ns();
    for (unsigned i = 0; i < SEQ_WAIT_LIMIT; i++) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 255u) == 255u && global_ns() - t0 > SEQ_WAIT_NS) return false;
    }
    return false;
}

// Global -> shared bulk copy completing on `bar` (16-byte aligned, size % 16 == 0).
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void fence_proxy_async() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// --------------------------------------------------------- the kernel

struct SeqSmem {
    uint8_t* wbuf[2];
    uint64_t* bar;     // [3]: weight buffers 0 and 1, K/V staging
    float *x, *q, *att, *an, *fr, *hid, *logits, *scores, *red, *ev, *part, *part2;
    float *ks, *vs;   // this layer's K / V rows staged in shared memory (or nullptr)
    __half* xs[2];     // fp16 hi/mid/lo splits of the matvec inputs, two alternating buffers
    int* xsh;          // [2] exponent undoing each buffer's row scaling
    uint64_t* keys;
    int* flag;         // [0] abort, [1] token broadcast, [2] top-p count, [3] drawn position
    SeqLayer* layers;  // the layer table, copied from global memory at entry
};

// Matrices in consumption order within a step: per layer qkv, wo, w1, w2; then head.
__device__ __forceinline__ const SeqMat& seq_mat(const SeqParams& p, const SeqLayer* layers, int idx) {
    const int layer = idx >> 2;
    if (layer >= p.L) return p.head;
    const SeqLayer& L = layers[layer];
    switch (idx & 3) {
        case 0: return L.qkv;
        case 1: return L.wo;
        case 2: return L.w1;
        default: return L.w2;
    }
}

// Weight pipeline: matrix number `seq` (monotone over the whole job) lives in
// buffer seq & 1; its barrier phase is (seq >> 1) & 1.
struct SeqPipe {
    int per_step;      // matrices per step: 4L + 1
    int in_step;       // issued % per_step, kept incrementally
    long long issued;  // next matrix to issue
    long long total;   // matrices the job consumes
};

__device__ __forceinline__ void seq_issue(const SeqParams& p, SeqSmem& s, SeqPipe& pipe) {
    // thread 0 only; buffer (issued & 1) must be free
    if (pipe.issued >= pipe.total) return;
    const SeqMat& m = seq_mat(p, s.layers, pipe.in_step);
    const int b = (int)(pipe.issued & 1);
    mbar_expect_tx(&s.bar[b], m.bytes);
    const uint8_t* src = m.blob;
    uint8_t* dst = s.wbuf[b];
    for (unsigned off = 0; off < m.bytes; off += 32768u) {
        const unsigned n = (m.bytes - off) < 32768u ? (m.bytes - off) : 32768u;
        bulk_g2s(dst + off, src + off, n, &s.bar[b]);
    }
    pipe.issued++;
    if (++pipe.in_step == pipe.per_step) pipe.in_step = 0;
}

// Block-level quantized matvec on the tensor cores from the shared-memory copy
// of matrix `m`: y[n] = epi(n, sum_k x[k] * level(k, n) * scale[n]). x enters
// as its fp16 hi/mid/lo split of x * 2^-xshift (three arrays of `xs_stride`
// elements, zero past K); B column g < 3 of each m16n8k16 MMA carries split
// g, the others are zero. Work units are (n-tile, k-part); k-parts combine
// through `red`.
template <int BITS, typename Epi>
__device__ __forceinline__ void seq_qmv(const SeqMat& m, const uint8_t* wsm, const __half* xs, int xs_stride,
                                        int xshift, float* red, Epi epi) {
    constexpr int KT = FragGeom<BITS>::KT;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, t = lane & 3;
    int kp = 1;
    while (kp < SEQ_WARPS && m.ntiles * kp * 2 <= SEQ_WARPS && m.nkg >= kp * 2) kp *= 2;
    const int per = (m.nkg + kp - 1) / kp;
    const int units = m.ntiles * kp;
    const float* scale = reinterpret_cast<const float*>(wsm + m.scale_off);
    const bool feeds = g < 3;
    const uint32_t* xw = reinterpret_cast<const uint32_t*>(xs + (feeds ? g : 0) * xs_stride);
    // INT4 outputs n+8 carry 16x (dz_deq4)
    const int sh_lo = xshift, sh_hi = BITS == 4 ? xshift - 4 : xshift;
    for (int u0 = 0; u0 < units; u0 += SEQ_WARPS) {
        const int unit = u0 + warp;
        const bool active = unit < units;
        const int nt = active ? unit / kp : 0, kpart = active ? unit % kp : 0;
        float d[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
        if (active) {
            const int kg1 = min((kpart + 1) * per, m.nkg);
            for (int kg = kpart * per; kg < kg1; kg++) {
                const uint4 w = reinterpret_cast<const uint4*>(wsm + ((size_t)nt * m.nkg + kg) * 512)[lane];
                const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
                for (int kt = 0; kt < KT; kt++) {
                    const int k0 = (kg * KT + kt) * 16;
                    const uint32_t b0 = feeds ? xw[(k0 >> 1) + t] : 0u;
                    const uint32_t b1 = feeds ? xw[(k0 >> 1) + t + 4] : 0u;
                    uint32_t af[4];
                    if (BITS == 4) dz_deq4(ww[kt], af);
                    else dz_deq8(ww[2 * kt], ww[2 * kt + 1], af);
                    dz_mma_f16(d[kt & 1], af, b0, b1);
                }
            }
        }
        // columns 0..2 (hi, mid, lo of the one row) sit in lanes t = 0 (cols 0, 1) and t = 1 (col 2)
        float v0 = (d[0][0] + d[0][1]) + (d[1][0] + d[1][1]);
        float v1 = (d[0][2] + d[0][3]) + (d[1][2] + d[1][3]);
        v0 += __shfl_xor_sync(0xffffffffu, v0, 1);
        v1 += __shfl_xor_sync(0xffffffffu, v1, 1);
        if (active && t == 0) {
            if (kp == 1) {
                const int n0 = nt * 16 + g;
                if (n0 < m.N) epi(n0, dz_mul_pow2(v0, sh_lo) * scale[n0]);
                if (n0 + 8 < m.N) epi(n0 + 8, dz_mul_pow2(v1, sh_hi) * scale[n0 + 8]);
            } else {
                red[(nt * kp + kpart) * 16 + g] = v0;
                red[(nt * kp + kpart) * 16 + g + 8] = v1;
            }
        }
    }
    if (kp > 1) {
        __syncthreads();
        for (int n = threadIdx.x; n < m.ntiles * 16; n += SEQ_THREADS) {
            const int nt = n >> 4, c = n & 15;
            float sum = 0.0f;
            for (int q = 0; q < kp; q++) sum += red[(nt * kp + q) * 16 + c];
            if (n < m.N) epi(n, dz_mul_pow2(sum, c < 8 ? sh_lo : sh_hi) * scale[n]);
        }
    }
}

// fp16 hi / mid / lo split of v * 2^sh into element i of a split buffer.
__device__ __forceinline__ void seq_split_store(__half* xs, int stride, int i, float v, int sh) {
    const DzSplit3 p = dz_split3(dz_mul_pow2(v, sh));
    xs[i] = p.h;
    xs[stride + i] = p.m;
    xs[2 * stride + i] = p.l;
}

// Split the n values of src (complete and visible to the block) into a split
// buffer with the row's exponent shift; block-wide, ends with the buffer
// written but not yet behind a barrier (the next acquire() is one).
__device__ __forceinline__ void seq_split_block(const float* src, int n, __half* xs, int stride, int* shift_slot,
                                                float* red) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float mx = 0.0f;
    for (int i = threadIdx.x; i < n; i += SEQ_THREADS) mx = fmaxf(mx, fabsf(src[i]));
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
    if (lane == 0) red[warp] = mx;
    __syncthreads();
    float amax = 0.0f;
#pragma unroll
    for (int w = 0; w < SEQ_WARPS; w++) amax = fmaxf(amax, red[w]);
    const int sh = dz_row_shift(amax);
    for (int i = threadIdx.x; i < n; i += SEQ_THREADS) seq_split_store(xs, stride, i, src[i], sh);
    if (threadIdx.x == 0) *shift_slot = -sh;
}

// Attention of one decode position over ctx ring rows (transformer.c:686-713)
// followed by the fp16 split of its output (the input of W_o). The warps of a
// head (up to four) split its keys: a lane takes one key and computes its
// whole q.k (float4 reads in a lane-rotated order, so the lanes' rows do not
// fall into one bank), the warp keeps an online softmax (running max m and
// sum l), and accumulates p.v with its lanes over the head dimension. After
// one barrier the warps of each head merge (m, l, vector); the merged output
// goes straight into the split. exp is expf of the difference to the running
// maximum, as in the reference's softmax; the normalisation divides the
// accumulated vector once. `scratch` holds wph x D floats, `red` 48.
__device__ __forceinline__ void seq_attention(int H, int hd, int D, int cap, int ctx, int start, const float* Ksrc,
                                              const float* Vsrc, const float* q, float denom, float* scratch,
                                              float* red, float* att, __half* xs, int xs_stride, int* shift_slot) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const float NEG_INF = __int_as_float(0xff800000);
    const int wph = H >= SEQ_WARPS ? 1 : min(4, SEQ_WARPS / H);   // warps per head
    const int hpr = SEQ_WARPS / wph;                                // heads per round
    const bool vec = (hd & 3) == 0 && (D & 3) == 0;
    const int nv = vec ? hd / 4 : hd;                               // float4s (or floats) per row
    const int rot = lane % nv;
    float* mw = red;               // [SEQ_WARPS] running max per warp
    float* lw = red + SEQ_WARPS;   // [SEQ_WARPS] running sum per warp
    const bool fused_split = H <= hpr && D <= SEQ_THREADS;
    float out = 0.0f;
    for (int h0 = 0; h0 < H; h0 += hpr) {
        const int h = h0 + warp / wph, w = warp % wph;
        if (warp < hpr * wph && h < H) {
            const int j0 = w * ctx / wph, j1 = (w + 1) * ctx / wph;
            const float* qh = q + h * hd;
            float m = NEG_INF, l = 0.0f;
            float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
            for (int c0 = j0; c0 < j1; c0 += 32) {
                const int j = c0 + lane;
                float sc = NEG_INF;
                if (j < j1) {
                    int phys = start + j;
                    if (phys >= cap) phys -= cap;
                    const float* kr = Ksrc + (long long)phys * D + h * hd;
                    float dot = 0.0f;
                    if (vec) {
                        const float4* k4 = reinterpret_cast<const float4*>(kr);
                        const float4* q4 = reinterpret_cast<const float4*>(qh);
                        for (int c = 0; c < nv; c++) {
                            int cc = rot + c;
                            if (cc >= nv) cc -= nv;
                            const float4 kv = k4[cc], qv = q4[cc];
                            dot = fmaf(qv.x, kv.x, dot);
                            dot = fmaf(qv.y, kv.y, dot);
                            dot = fmaf(qv.z, kv.z, dot);
                            dot = fmaf(qv.w, kv.w, dot);
                        }
                    } else {
                        for (int c = 0; c < nv; c++) {
                            int cc = rot + c;
                            if (cc >= nv) cc -= nv;
                            dot = fmaf(qh[cc], kr[cc], dot);
                        }
                    }
                    sc = dot / denom;
                }
                float cmax = sc;
#pragma unroll
                for (int off = 16; off >= 1; off >>= 1) cmax = fmaxf(cmax, __shfl_xor_sync(0xffffffffu, cmax, off));
                const float mn = fmaxf(m, cmax);
                const float pj = j < j1 ? expf(sc - mn) : 0.0f;
                const float corr = expf(m - mn);
                float ps = pj;
#pragma unroll
                for (int off = 16; off >= 1; off >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, off);
                l = l * corr + ps;
#pragma unroll
                for (int i = 0; i < 4; i++) acc[i] *= corr;
                const int n = min(32, j1 - c0);
                for (int u = 0; u < n; u++) {
                    const float pu = __shfl_sync(0xffffffffu, pj, u);
                    int phys = start + c0 + u;
                    if (phys >= cap) phys -= cap;
                    const float* vr = Vsrc + (long long)phys * D + h * hd;
#pragma unroll
                    for (int i = 0; i < 4; i++) {
                        const int e = lane + 32 * i;
                        if (e < hd) acc[i] = fmaf(pu, vr[e], acc[i]);
                    }
                }
                m = mn;
            }
            if (lane == 0) {
                mw[warp] = m;
                lw[warp] = l;
            }
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const int e = lane + 32 * i;
                if (e < hd) scratch[w * D + h * hd + e] = acc[i];
            }
        }
        __syncthreads();
        // merge the warps of each head of this round
        for (int i = threadIdx.x; i < D; i += SEQ_THREADS) {
            const int h = i / hd;
            if (h < h0 || h >= h0 + hpr) continue;
            const int wb = (h - h0) * wph;
            float M = NEG_INF;
            for (int w = 0; w < wph; w++) M = fmaxf(M, mw[wb + w]);
            float num = 0.0f, den = 0.0f;
            for (int w = 0; w < wph; w++) {
                const float f = expf(mw[wb + w] - M);
                num = fmaf(f, scratch[w * D + i], num);
                den = fmaf(f, lw[wb + w], den);
            }
            const float o = num / den;
            if (fused_split) out = o;
            else att[i] = o;
        }
        if (!fused_split) __syncthreads();   // the next round reuses mw / lw / scratch
    }
    if (!fused_split) {
        seq_split_block(att, D, xs, xs_stride, shift_slot, red + 2 * SEQ_WARPS);
        return;
    }
    // split of the merged output (held by threads 0..D-1): block max, then
    // each thread stores its element's hi / mid / lo
    float mx = threadIdx.x < D ? fabsf(out) : 0.0f;
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
    float* wred = red + 2 * SEQ_WARPS;
    if (lane == 0) wred[warp] = mx;
    __syncthreads();
    float amax = 0.0f;
#pragma unroll
    for (int w = 0; w < SEQ_WARPS; w++) amax = fmaxf(amax, wred[w]);
    const int sh = dz_row_shift(amax);
    if (threadIdx.x < D) seq_split_store(xs, xs_stride, threadIdx.x, out, sh);
    if (threadIdx.x == 0) *shift_slot = -sh;
}

// LayerNorm (src/core/tensor_ops.c:88-111) of D values in shared memory, by
// warp 0 (shuffle reductions, no block barrier until the output is written).
__device__ __forceinline__ void seq_layernorm(const float* in, float* out, const float* gamma, const float* beta,
                                              int D, __half* xs, int xs_stride, int* shift_slot) {
    constexpr int R = 8;   // elements per lane kept in registers (D <= 256)
    if (threadIdx.x < 32 && D <= 32 * R) {
        // the same arithmetic, with the lane's inputs, gamma and beta loaded
        // once up front instead of re-read from shared memory per pass
        const int lane = threadIdx.x;
        float xv[R], gv[R], bv[R], yv[R];
#pragma unroll
        for (int j = 0; j < R; j++) {
            const int i = lane + 32 * j;
            xv[j] = i < D ? in[i] : 0.0f;
            gv[j] = i < D ? gamma[i] : 0.0f;
            bv[j] = i < D ? beta[i] : 0.0f;
        }
        float s = 0.0f;
#pragma unroll
        for (int j = 0; j < R; j++)
            if (lane + 32 * j < D) s += xv[j];
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
        const float mean = s / (float)D;
        float v = 0.0f;
#pragma unroll
        for (int j = 0; j < R; j++)
            if (lane + 32 * j < D) {
                const float d = xv[j] - mean;
                v = fmaf(d, d, v);
            }
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
        const float sd = sqrtf(v / (float)D + 1e-6f);
        float mx = 0.0f;
#pragma unroll
        for (int j = 0; j < R; j++) {
            const int i = lane + 32 * j;
            yv[j] = 0.0f;
            if (i < D) {
                const float y = gv[j] * ((xv[j] - mean) / sd) + bv[j];
                out[i] = y;
                yv[j] = y;
                mx = fmaxf(mx, fabsf(y));
            }
        }
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
        const int sh = dz_row_shift(mx);
#pragma unroll
        for (int j = 0; j < R; j++)
            if (lane + 32 * j < D) seq_split_store(xs, xs_stride, lane + 32 * j, yv[j], sh);
        if (lane == 0) *shift_slot = -sh;
    } else if (threadIdx.x < 32) {
        const int lane = threadIdx.x;
        float s = 0.0f;
        for (int i = lane; i < D; i += 32) s += in[i];
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
        const float mean = s / (float)D;
        float v = 0.0f;
        for (int i = lane; i < D; i += 32) {
            const float d = in[i] - mean;
            v = fmaf(d, d, v);
        }
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
        const float sd = sqrtf(v / (float)D + 1e-6f);
        float mx = 0.0f;
        for (int i = lane; i < D; i += 32) {
            const float y = gamma[i] * ((in[i] - mean) / sd) + beta[i];
            out[i] = y;
            mx = fmaxf(mx, fabsf(y));
        }
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
        const int sh = dz_row_shift(mx);
        for (int i = lane; i < D; i += 32) seq_split_store(xs, xs_stride, i, out[i], sh);
        if (lane == 0) *shift_slot = -sh;
    }
    __syncthreads();
}

// Ascending bitonic sort of the n keys of a (n a power of two), the network of
// dz_bitonic_sort with its keys held in registers for n <= 2 * SEQ_THREADS:
// element i = e * SEQ_THREADS + threadIdx.x, padded to SEQ_THREADS with the
// largest key (a holds at least SEQ_THREADS entries). Partners closer than 32
// are exchanged by warp shuffles, partners up to SEQ_THREADS / 2 apart through
// a[] (two barriers per stage), the partner SEQ_THREADS away sits in the same
// thread. Larger n go to dz_bitonic_sort.
static __device__ void seq_sort_keys(uint64_t* a, int n) {
    if (n > 2 * SEQ_THREADS) {
        dz_bitonic_sort(a, n);
        return;
    }
    const int m = n < SEQ_THREADS ? SEQ_THREADS : n;
    const int E = m / SEQ_THREADS;   // keys per thread: 1 or 2
    const int tid = threadIdx.x;
    uint64_t v[2];
#pragma unroll
    for (int e = 0; e < 2; e++) {
        const int i = e * SEQ_THREADS + tid;
        v[e] = (e < E && i < n) ? a[i] : ~0ull;
    }
    for (int size = 2; size <= m; size <<= 1) {
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            if (stride >= SEQ_THREADS) {   // E == 2: elements tid and tid + SEQ_THREADS
                const bool up = (tid & size) == 0;
                if ((v[0] > v[1]) == up) {
                    const uint64_t t = v[0];
                    v[0] = v[1];
                    v[1] = t;
                }
                continue;
            }
            uint64_t w[2];
            if (stride >= 32) {
                __syncthreads();   // earlier readers of a[] are done
#pragma unroll
                for (int e = 0; e < 2; e++)
                    if (e < E) a[e * SEQ_THREADS + tid] = v[e];
                __syncthreads();
#pragma unroll
                for (int e = 0; e < 2; e++) w[e] = e < E ? a[(e * SEQ_THREADS + tid) ^ stride] : 0ull;
            } else {
#pragma unroll
                for (int e = 0; e < 2; e++) w[e] = __shfl_xor_sync(0xffffffffu, v[e], stride);
            }
#pragma unroll
            for (int e = 0; e < 2; e++) {
                if (e >= E) continue;
                const int i = e * SEQ_THREADS + tid;
                const bool take_min = ((i & stride) == 0) == ((i & size) == 0);
                const bool less = v[e] < w[e];
                v[e] = take_min ? (less ? v[e] : w[e]) : (less ? w[e] : v[e]);
            }
        }
    }
    __syncthreads();
#pragma unroll
    for (int e = 0; e < 2; e++) {
        const int i = e * SEQ_THREADS + tid;
        if (e < E && i < n) a[i] = v[e];
    }
    __syncthreads();
}

// Selection over the logits in shared memory; returns the token on every thread.
static __device__ uint32_t seq_select(const SeqParams& p, SeqSmem& s, uint64_t* rng) {
    const int V = p.V;
    float* lg = s.logits;
    for (int m = threadIdx.x; m < p.n_masked; m += SEQ_THREADS) {
        const uint32_t id = p.masked[m];
        if (id < (uint32_t)V) lg[id] = -3.402823466e38f;
    }
    __syncthreads();
    const bool greedy = p.strategy == 0 || !(p.temperature > 0.0f) || rng == nullptr ||
                        (p.strategy == 1 && p.top_k == 0) ||
                        (p.strategy == 2 && (p.top_p <= 0.0f || p.top_p > 1.0f)) ||
                        (p.strategy != 1 && p.strategy != 2);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (greedy) {
        uint64_t best = ~0ull;
        for (int i = threadIdx.x; i < V; i += SEQ_THREADS) {
            const uint64_t k = dz_desc_key(lg[i], (uint32_t)i);
            best = k < best ? k : best;
        }
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) {
            const uint64_t o = __shfl_xor_sync(0xffffffffu, best, off);
            best = o < best ? o : best;
        }
        if (lane == 0) s.keys[warp] = best;
        __syncthreads();
        if (threadIdx.x == 0) {
            uint64_t mn = s.keys[0];
            for (int w = 1; w < SEQ_WARPS; w++) mn = s.keys[w] < mn ? s.keys[w] : mn;
            s.flag[1] = (int)(mn & 0xffffffffu);
        }
        __syncthreads();
        const uint32_t tok = (uint32_t)s.flag[1];
        __syncthreads();
        return tok;
    }
    const float inv_t = 1.0f / p.temperature;
    int P = 1;
    while (P < V) P <<= 1;
    for (int i = threadIdx.x; i < P; i += SEQ_THREADS)
        s.keys[i] = i < V ? dz_desc_key(lg[i] * inv_t, (uint32_t)i) : ~0ull;
    __syncthreads();
    seq_sort_keys(s.keys, P);
    const int nexp = p.strategy == 1 ? (p.top_k < V ? p.top_k : V) : V;
    const float top = dz_key_value(s.keys[0]);
    for (int i = threadIdx.x; i < nexp; i += SEQ_THREADS) s.ev[i] = dz_expf(dz_key_value(s.keys[i]) - top);
    __syncthreads();
    // The reference's running sums (sampling.c:80-94, :137-170) are sequential
    // fp32 chains. One thread builds them as prefix arrays - every "acc +=
    // e[i]" loop of the reference reads a prefix of the same chain P - with
    // explicit round-to-nearest adds and multiplies (no FMA contraction, as
    // the reference's x86 build has none); the searches then run in parallel.
    float* Pre = s.part;                   // prefix sums of e
    float* C = s.part2;                    // running sum of e[i] * (1/sum_all)
    if (threadIdx.x == 0) {
        // blocks of 8: loads first (they do not depend on the chain), then the
        // dependent adds, then the stores
        const float* ev = s.ev;
        float acc = 0.0f;
        int i = 0;
        for (; i + 8 <= nexp; i += 8) {
            float e8[8], o8[8];
#pragma unroll
            for (int u = 0; u < 8; u++) e8[u] = ev[i + u];
#pragma unroll
            for (int u = 0; u < 8; u++) { acc = __fadd_rn(acc, e8[u]); o8[u] = acc; }
#pragma unroll
            for (int u = 0; u < 8; u++) Pre[i + u] = o8[u];
        }
        for (; i < nexp; i++) {
            acc = __fadd_rn(acc, ev[i]);
            Pre[i] = acc;
        }
        if (p.strategy == 2) {
            const float inv = __fdiv_rn(1.0f, acc);
            float cum = 0.0f;
            i = 0;
            for (; i + 8 <= nexp; i += 8) {
                float e8[8], o8[8];
#pragma unroll
                for (int u = 0; u < 8; u++) e8[u] = __fmul_rn(ev[i + u], inv);
#pragma unroll
                for (int u = 0; u < 8; u++) { cum = __fadd_rn(cum, e8[u]); o8[u] = cum; }
#pragma unroll
                for (int u = 0; u < 8; u++) C[i + u] = o8[u];
            }
            for (; i < nexp; i++) {
                cum = __fadd_rn(cum, __fmul_rn(ev[i], inv));
                C[i] = cum;
            }
        }
        s.flag[2] = nexp;   // top-p candidate count, refined below
        s.flag[3] = -1;     // selected position
    }
    __syncthreads();
    if (p.strategy == 2) {
        // cand = first i with C[i] >= top_p, plus one (nexp when none)
        for (int i = threadIdx.x; i < nexp; i += SEQ_THREADS)
            if (C[i] >= p.top_p) atomicMin(&s.flag[2], i + 1);
        __syncthreads();
    }
    const int cand = s.flag[2];
    if (threadIdx.x == 0) {
        const float total = Pre[cand - 1];
        s.red[0] = __fmul_rn((float)dz_rng_unit(rng), total);
    }
    __syncthreads();
    const float r = s.red[0];
    int* pos = &s.flag[3];
    for (int i = threadIdx.x; i < cand; i += SEQ_THREADS)
        if (Pre[i] >= r) atomicMin(reinterpret_cast<unsigned int*>(pos), (unsigned int)i);
    __syncthreads();
    if (threadIdx.x == 0) {
        const int at = s.flag[3] < 0 ? 0 : s.flag[3];   // no crossing: the reference keeps pairs[0]
        s.flag[1] = (int)(s.keys[at] & 0xffffffffu);
    }
    __syncthreads();
    const uint32_t tok = (uint32_t)s.flag[1];
    __syncthreads();
    return tok;
}

template <int BITS>
__global__ void __launch_bounds__(SEQ_THREADS, 1) dz_seqgen_kernel(SeqParams p) {
    extern __shared__ __align__(128) unsigned char seq_smem[];
    const int b = blockIdx.x;
    const int D = p.D, H = p.H, hd = D / H, F = 4 * D, V = p.V, cap = p.cap;

    SeqSmem s;
    unsigned char* cur = seq_smem;
    s.wbuf[0] = cur; cur += p.buf_bytes;
    s.wbuf[1] = cur; cur += p.buf_bytes;
    s.bar = reinterpret_cast<uint64_t*>(cur); cur += 32;
    s.flag = reinterpret_cast<int*>(cur); cur += 16;
    s.xsh = reinterpret_cast<int*>(cur); cur += 16;
    s.layers = reinterpret_cast<SeqLayer*>(cur); cur += (sizeof(SeqLayer) * p.L + 15) & ~(size_t)15;
    int P = 1;
    while (P < V) P <<= 1;
    s.keys = reinterpret_cast<uint64_t*>(cur); cur += 8 * (P > SEQ_THREADS ? P : SEQ_THREADS);
    // float arrays, each rounded up to 16 bytes (bulk-copy destinations and
    // float4 activation reads need the alignment); seq_smem_bytes mirrors this
    float* f = reinterpret_cast<float*>(cur);
    auto take = [&](int n) { float* r = f; f += (n + 3) & ~3; return r; };
    s.x = take(D);
    s.q = take(D);
    s.att = take(D);
    s.an = take(D);
    s.fr = take(D);
    s.hid = take(F);
    s.logits = take(V);
    s.ev = take(V);
    s.scores = take(H * cap);
    s.red = take(64);
    const int pv = V > SEQ_THREADS ? V : SEQ_THREADS;
    s.part = take(pv);
    s.part2 = take(pv);
    if (p.kv_smem) {
        s.ks = take(cap * D);
        s.vs = take(cap * D);
    } else {
        s.ks = s.vs = nullptr;
    }
    const int xs_stride = ((F + 63) / 64) * 64;   // longest matvec input, padded to a k-group
    s.xs[0] = reinterpret_cast<__half*>(take(3 * xs_stride / 2));
    s.xs[1] = reinterpret_cast<__half*>(take(3 * xs_stride / 2));
    for (int i = threadIdx.x; i < 3 * xs_stride; i += SEQ_THREADS) {
        s.xs[0][i] = __float2half_rn(0.0f);
        s.xs[1][i] = __float2half_rn(0.0f);
    }

    for (int i = threadIdx.x; i < (int)(sizeof(SeqLayer) * p.L / 4); i += SEQ_THREADS)
        reinterpret_cast<uint32_t*>(s.layers)[i] = reinterpret_cast<const uint32_t*>(p.layers)[i];
    if (threadIdx.x == 0) {
        mbar_init(&s.bar[0], 1);
        mbar_init(&s.bar[1], 1);
        mbar_init(&s.bar[2], 1);
        s.flag[0] = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();

    SeqPipe pipe;
    pipe.per_step = 4 * p.L + 1;
    const long long steps = (long long)p.plen + (p.n_new > 0 ? p.n_new - 1 : 0);
    pipe.total = steps * pipe.per_step;
    pipe.issued = 0;
    pipe.in_step = 0;
    if (threadIdx.x == 0) {
        seq_issue(p, s, pipe);
        seq_issue(p, s, pipe);
    }
    long long consumed = 0;

    int start = p.start[b], length = p.length[b];
    long long total = p.total[b];
    uint64_t rng_state = 0;
    uint64_t* rng = nullptr;
    if (p.seeds) {
        uint64_t st = dz_splitmix64(p.seeds[b] ^ dz_splitmix64(0x94d049bb133111ebull));
        rng_state = st ? st : 0x9e3779b97f4a7c15ull;
        rng = &rng_state;
    }
    const float denom = sqrtf((float)hd);
    bool aborted = false;
    unsigned kv_uses = 0;   // completed phases of the K/V staging barrier
    bool kv_pending = false; // a K/V staging copy is in flight

    // wait for matrix `consumed`, returns false on timeout (CTA-uniform)
    SeqClock clk(p.phase_ns);
    auto acquire = [&]() -> bool {
        const int bi = (int)(consumed & 1);
        const uint32_t parity = (uint32_t)((consumed >> 1) & 1);
        if (threadIdx.x == 0 && !mbar_wait(&s.bar[bi], parity)) s.flag[0] = 1;
        __syncthreads();
        clk.mark(SEQ_PH_WAIT);
        return s.flag[0] == 0;
    };
    // matrix `consumed` no longer read: refill its buffer with the one after next
    auto release = [&](bool after_barrier = false) {
        // every thread is past its reads of this buffer; the next TMA write
        // into it is issued after the barrier (the LayerNorm that ends W_o's
        // and W2's phases ends with one already)
        if (!after_barrier) __syncthreads();
        if (threadIdx.x == 0) seq_issue(p, s, pipe);
        consumed++;
        clk.mark(SEQ_PH_QMV);
    };

    auto forward = [&](uint32_t tok) -> bool {
        const long long pos = total;
        int slot, ctx;
        if (length < cap) {
            slot = (start + length) % cap;
            ctx = length + 1;
        } else {
            slot = start;
            start = (start + 1) % cap;
            ctx = cap;
        }
        if (tok >= (uint32_t)V) tok = 0;
        const float* e = p.emb + (long long)tok * D;
        if (pos < p.pe_rows) {
            const float* pr = p.pe + pos * D;
            for (int i = threadIdx.x; i < D; i += SEQ_THREADS) {
                s.x[i] = e[i] + pr[i];
            }
        } else {
            const float ln_base = logf(10000.0f);
            for (int i = threadIdx.x; i < D; i += SEQ_THREADS) {
                const float sc = expf(-((2.0f * (float)i) / (float)D) * ln_base);
                const float ang = (float)pos * sc;
                s.x[i] = e[i] + ((i % 2 == 0) ? sinf(ang) : cosf(ang));
            }
        }
        __syncthreads();
        seq_split_block(s.x, D, s.xs[0], xs_stride, &s.xsh[0], s.red);
        clk.mark(SEQ_PH_EMBED);
        for (int l = 0; l < p.L; l++) {
            const SeqLayer& Ly = s.layers[l];
            float* Kl = p.keys + (((long long)l * p.B + b) * cap) * D;
            float* Vl = p.values + (((long long)l * p.B + b) * cap) * D;
            // Stage the K/V rows this step attends to, except the new slot, into
            // shared memory; the copy overlaps the QKV product below.
            const int old_rows = ctx - 1 < cap ? (length < cap ? length : cap) : cap;
            const bool staged = s.ks != nullptr && old_rows > 0;
            kv_pending = staged;
            if (staged && threadIdx.x == 0) {
                // rows [0, old_rows) hold the retained tokens; the slot row is excluded
                const int lo_rows = slot < old_rows ? slot : old_rows;
                const int hi_first = slot + 1, hi_rows = old_rows - hi_first;
                const unsigned bytes = (unsigned)((lo_rows + (hi_rows > 0 ? hi_rows : 0)) * D * 4) * 2u;
                // order earlier generic writes (ring rows in global, last layer's
                // reads of the staging area) before the async-proxy copy
                asm volatile("fence.proxy.async;" ::: "memory");
                mbar_expect_tx(&s.bar[2], bytes);
                if (lo_rows > 0) {
                    bulk_g2s(s.ks, Kl, (unsigned)(lo_rows * D * 4), &s.bar[2]);
                    bulk_g2s(s.vs, Vl, (unsigned)(lo_rows * D * 4), &s.bar[2]);
                }
                if (hi_rows > 0) {
                    bulk_g2s(s.ks + (long long)hi_first * D, Kl + (long long)hi_first * D, (unsigned)(hi_rows * D * 4),
                             &s.bar[2]);
                    bulk_g2s(s.vs + (long long)hi_first * D, Vl + (long long)hi_first * D, (unsigned)(hi_rows * D * 4),
                             &s.bar[2]);
                }
            }
            // QKV: q to shared memory, k and v into the ring slot (global, and
            // the staged copy)
            if (!acquire()) return false;
            float* ksm = s.ks;
            float* vsm = s.vs;
            seq_qmv<BITS>(Ly.qkv, s.wbuf[consumed & 1], s.xs[0], xs_stride, s.xsh[0], s.part, [&](int n, float y) {
                if (n < D) {
                    s.q[n] = y;
                } else if (n < 2 * D) {
                    Kl[(long long)slot * D + (n - D)] = y;
                    if (ksm) ksm[slot * D + (n - D)] = y;
                } else {
                    Vl[(long long)slot * D + (n - 2 * D)] = y;
                    if (vsm) vsm[slot * D + (n - 2 * D)] = y;
                }
            });
            release();
            if (staged) {
                if (threadIdx.x == 0 && !mbar_wait(&s.bar[2], kv_uses & 1u)) s.flag[0] = 1;
                kv_uses++;
                __syncthreads();
                if (s.flag[0]) return false;
            }
            kv_pending = false;
            const float* Ksrc = ksm ? ksm : Kl;
            const float* Vsrc = vsm ? vsm : Vl;
            // attention over the ring (transformer.c:686-713), then the fp16
            // split of its output for W_o
            seq_attention(H, hd, D, cap, ctx, start, Ksrc, Vsrc, s.q, denom, s.hid, s.red, s.att, s.xs[1],
                          xs_stride, &s.xsh[1]);
            clk.mark(SEQ_PH_ATTENTION);
            // W_o, + residual, then LayerNorm with the gamma/beta carried in W_o's blob
            if (!acquire()) return false;
            {
                const uint8_t* wb = s.wbuf[consumed & 1];
                seq_qmv<BITS>(Ly.wo, wb, s.xs[1], xs_stride, s.xsh[1], s.part,
                              [&](int n, float y) { s.fr[n] = y + s.x[n]; });
                __syncthreads();
                const float* g = reinterpret_cast<const float*>(wb + Ly.wo.gamma_off);
                seq_layernorm(s.fr, s.an, g, g + D, D, s.xs[0], xs_stride, &s.xsh[0]);
            }
            release(true);
            clk.mark(SEQ_PH_NORM);
            // FFN up + bias + ReLU
            if (!acquire()) return false;
            {
                const uint8_t* wb = s.wbuf[consumed & 1];
                const float* bias = reinterpret_cast<const float*>(wb + Ly.w1.bias_off);
                seq_qmv<BITS>(Ly.w1, wb, s.xs[0], xs_stride, s.xsh[0], s.part, [&](int n, float y) {
                    const float pre = y + bias[n];
                    s.hid[n] = pre > 0.0f ? pre : 0.0f;
                });
            }
            release();
            seq_split_block(s.hid, F, s.xs[1], xs_stride, &s.xsh[1], s.red);
            // FFN down + bias + residual, LayerNorm
            if (!acquire()) return false;
            {
                const uint8_t* wb = s.wbuf[consumed & 1];
                const float* bias = reinterpret_cast<const float*>(wb + Ly.w2.bias_off);
                seq_qmv<BITS>(Ly.w2, wb, s.xs[1], xs_stride, s.xsh[1], s.part,
                              [&](int n, float y) { s.fr[n] = y + bias[n] + s.an[n]; });
                __syncthreads();
                const float* g = reinterpret_cast<const float*>(wb + Ly.w2.gamma_off);
                seq_layernorm(s.fr, s.x, g, g + D, D, s.xs[0], xs_stride, &s.xsh[0]);
            }
            release(true);
            clk.mark(SEQ_PH_NORM);
        }
        if (!acquire()) return false;
        {
            const uint8_t* wb = s.wbuf[consumed & 1];
            const float* bias = reinterpret_cast<const float*>(wb + p.head.bias_off);
            seq_qmv<BITS>(p.head, wb, s.xs[0], xs_stride, s.xsh[0], s.part,
                          [&](int n, float y) { s.logits[n] = y + bias[n]; });
        }
        release();
        __syncthreads();
        if (length < cap) length++;
        total++;
        return true;
    };

    for (int t = 0; t < p.plen && !aborted; t++)
        if (!forward(p.prompts[(long long)b * p.plen + t])) aborted = true;
    for (int i = 0; i < p.n_new && !aborted; i++) {
        const uint32_t tok = seq_select(p, s, rng);
        clk.mark(SEQ_PH_SELECT);
        if (threadIdx.x == 0) p.out[(long long)b * p.n_new + i] = tok;
        if (i + 1 < p.n_new && !forward(tok)) aborted = true;
    }

    if (aborted) {
        // let copies in flight land before the CTA's shared memory goes away
        if (threadIdx.x == 0) {
            p.status[0] = DZ_SEQ_TIMEOUT;
            for (long long m = consumed; m < pipe.issued; m++)
                mbar_wait(&s.bar[m & 1], (uint32_t)((m >> 1) & 1));
            if (kv_pending) mbar_wait(&s.bar[2], kv_uses & 1u);
        }
        __syncthreads();
        return;
    }
    if (threadIdx.x == 0) {
        p.start[b] = start;
        p.length[b] = length;
        p.total[b] = total;
    }
}

// Host side (seqgen.cu): the dynamic shared-memory limit and one launch.
cudaError_t dz_seqgen_set_smem(int bits, int bytes);
cudaError_t dz_seqgen_launch(const SeqParams& p, int bits, int blocks, size_t smem, cudaStream_t st);

}  // namespace dz
