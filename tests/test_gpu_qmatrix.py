"""Quantized weight matrices on the device: layout round trip (bit-exact codes
and unpack), and C = A . deq(W) against the reference's outputs and the oracle
(tolerance of src/tests/core/test_quantized_matmul.c:79: 1e-4 * (1 + max|ref|))."""
import numpy as np
import pytest

from conftest import golden

pytestmark = pytest.mark.gpu


def _tol_ok(c, ref):
    err = np.abs(c - ref).max()
    return err <= 1e-4 * (1 + np.abs(ref).max()), err


@pytest.mark.parametrize("shape", [(1, 1), (7, 3), (33, 47), (64, 257), (128, 384), (4096, 32000 // 16),
                                   (600, 50257 // 8), (1000, 130)])
@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("gran", [0, 1, 2])
def test_layout_round_trip_bit_exact(gpu, shape, bits, gran):
    rng = np.random.RandomState(shape[0] * 7 + shape[1])
    w = (rng.randn(*shape) * 0.02).astype(np.float32)
    s, p = gpu.quantize_pack(w, bits, gran)
    q = gpu.QuantizedWeightMatrix(s, p, shape[0], shape[1], bits, gran)
    np.testing.assert_array_equal(q.codes(), p)
    ref = gpu.quantize_unpack(s, p, shape[0], shape[1], bits, gran)
    np.testing.assert_array_equal(q.unpack().view(np.uint32), ref.view(np.uint32))
    q.close()


def test_matmul_reference_test_shapes(gpu):
    g = golden("qmm.npz")
    for n in range(int(g["count"])):
        m, k, nn, bits, gran = (int(x) for x in g[f"t{n}_meta"])
        q = gpu.QuantizedWeightMatrix.encode(g[f"t{n}_b"], bits, gran)
        ok, err = _tol_ok(q.matmul(g[f"t{n}_a"]), g[f"t{n}_c"])
        assert ok, (m, k, nn, bits, gran, err)
        q.close()


@pytest.mark.parametrize("bits", [8, 4])
def test_matmul_c3_reference_outputs(gpu, bits):
    """C3 K=N=4096, M=8 and M=1 against the reference's matmul_quantized_weight."""
    st = np.array([gpu.rng_stream(3, gpu.STREAM_TESTING)], np.uint64)
    x = gpu.synth_gaussian(st, 512 * 4096, 1.0).reshape(512, 4096)
    w = gpu.synth_gaussian(st, 4096 * 4096, 0.02).reshape(4096, 4096)
    ref = golden("qmm.npz")[f"c3_m8_int{bits}"]
    q = gpu.QuantizedWeightMatrix.encode(w, bits)
    ok, err = _tol_ok(q.matmul(x[:8]), ref)
    assert ok, err
    ok1, err1 = _tol_ok(q.matmul(x[:1]), ref[:1])
    assert ok1, err1
    q.close()


@pytest.mark.parametrize("N", [4096, 11008, 32000])
@pytest.mark.parametrize("bits", [8, 4])
def test_matmul_c3_sweep_vs_oracle(gpu, oracle, N, bits):
    """Every C3 (M, N) at K=4096; the oracle checks a seeded sample of columns
    (column scales make a column slice quantize to the same codes)."""
    st = np.array([gpu.rng_stream(3, gpu.STREAM_TESTING)], np.uint64)
    x = gpu.synth_gaussian(st, 512 * 4096, 1.0).reshape(512, 4096)
    w = gpu.synth_gaussian(st, 4096 * N, 0.02).reshape(4096, N)
    q = gpu.QuantizedWeightMatrix.encode(w, bits)
    cols = np.sort(np.random.RandomState(N + bits).choice(N, 96, replace=False))
    s_sub, p_sub = oracle.quantize_pack(np.ascontiguousarray(w[:, cols]), bits, 2)
    for M in (1, 8, 64, 512):
        c = q.matmul(x[:M])
        assert c.shape == (M, N) and np.isfinite(c).all()
        ref = oracle.matmul_quantized(x[:M], 4096, len(cols), s_sub, p_sub, bits, 2)
        ok, err = _tol_ok(c[:, cols], ref)
        assert ok, (M, err)
    q.close()


def test_matmul_ragged_and_unaligned(gpu, oracle):
    rng = np.random.RandomState(1)
    for (m, k, n) in [(13, 100, 77), (3, 9, 5), (1, 4095, 33), (9, 4104, 1)]:
        for bits in (4, 8):
            w = (rng.randn(k, n) * 0.05).astype(np.float32)
            buf = rng.randn(m * k + 1).astype(np.float32)
            a = buf[1:].reshape(m, k)                      # not 16-byte aligned
            q = gpu.QuantizedWeightMatrix.encode(w, bits)
            s, p = oracle.quantize_pack(w, bits, 2)
            ref = oracle.matmul_quantized(np.ascontiguousarray(a), k, n, s, p, bits, 2)
            ok, err = _tol_ok(q.matmul(a), ref)
            assert ok, (m, k, n, bits, err)
            q.close()


@pytest.mark.parametrize("gran", [0, 1, 2])
def test_matmul_many_rows_ragged(gpu, oracle, gran):
    """Row counts above the matvec kernels' limit (the tensor-core GEMM for
    INT8), ragged K / N, every granularity, against the oracle."""
    rng = np.random.RandomState(7 + gran)
    for (m, k, n) in [(17, 100, 77), (130, 300, 257), (200, 4104, 129), (64, 64, 16)]:
        for bits in (8, 4):
            w = (rng.randn(k, n) * 0.05).astype(np.float32)
            a = rng.randn(m, k).astype(np.float32)
            q = gpu.QuantizedWeightMatrix.encode(w, bits, gran)
            s, p = oracle.quantize_pack(w, bits, gran)
            ref = oracle.matmul_quantized(a, k, n, s, p, bits, gran)
            ok, err = _tol_ok(q.matmul(a), ref)
            assert ok, (m, k, n, bits, gran, err)
            q.close()


def test_matmul_many_rows_dynamic_range_and_nonfinite(gpu, oracle):
    """Rows whose elements span 2^-30 .. 2^20, and a row holding inf / NaN
    (which reads NaN, as the reference's fp32 sums do), at M = 40."""
    rng = np.random.RandomState(11)
    m, k, n = 40, 512, 300
    w = (rng.randn(k, n) * 0.05).astype(np.float32)
    a = (rng.randn(m, k) * np.exp2(rng.randint(-30, 20, size=(m, k)))).astype(np.float32)
    a[5] *= 1e-30
    for bits in (8, 4):
        q = gpu.QuantizedWeightMatrix.encode(w, bits)
        s, p = oracle.quantize_pack(w, bits, 2)
        ref = oracle.matmul_quantized(a, k, n, s, p, bits, 2)
        c = q.matmul(a)
        for r in range(m):
            ok, err = _tol_ok(c[r], ref[r])
            assert ok, (bits, r, err)
        bad = a.copy()
        bad[3, 7] = np.inf
        bad[9, 100] = np.nan
        c = q.matmul(bad)
        assert np.isnan(c[9]).all() and not np.isfinite(c[3]).any()
        assert np.isfinite(np.delete(c, [3, 9], axis=0)).all()
        q.close()


def test_matmul_rejects_bad_k(gpu):
    q = gpu.QuantizedWeightMatrix.encode(np.ones((8, 4), np.float32), 8)
    with pytest.raises(gpu.DzError):
        q.matmul(np.ones((2, 7), np.float32))
    q.close()


@pytest.mark.parametrize("gran", [0, 1, 2])
def test_matmul_tensor_core_gemv_ragged(gpu, oracle, gran):
    """8..16 rows on matrices of at least 2^20 codes (the tcgen05 GEMV):
    ragged K and N, every granularity, activations from an aligned buffer and
    from a device buffer off the 16-byte grid (the split's scalar path),
    against the oracle."""
    torch = pytest.importorskip("torch")
    rng = np.random.RandomState(23 + gran)
    for (m, k, n) in [(8, 1100, 1000), (16, 4104, 300), (13, 2048, 1031)]:
        for bits in (8, 4):
            w = (rng.randn(k, n) * 0.05).astype(np.float32)
            buf = rng.randn(m * k + 1).astype(np.float32)
            q = gpu.QuantizedWeightMatrix.encode(w, bits, gran)
            s, p = oracle.quantize_pack(w, bits, gran)
            a = np.ascontiguousarray(buf[1:].reshape(m, k))
            ref = oracle.matmul_quantized(a, k, n, s, p, bits, gran)
            ok, err = _tol_ok(q.matmul(a), ref)
            assert ok, (m, k, n, bits, gran, err)
            # the same rows from a device buffer 4 bytes past a 16-byte boundary
            xd = torch.from_numpy(buf).cuda()
            cd = torch.empty((m, n), dtype=torch.float32, device="cuda")
            q.matmul_async(xd.data_ptr() + 4, cd.data_ptr(), m, torch.cuda.current_stream().cuda_stream)
            torch.cuda.synchronize()
            ok, err = _tol_ok(cd.cpu().numpy(), ref)
            assert ok, ("unaligned", m, k, n, bits, gran, err)
            q.close()


@pytest.mark.parametrize("bits", [8, 4])
def test_matmul_tensor_core_gemv_large(gpu, oracle, bits):
    """3..16 rows on a matrix of more than 2^25 codes (the GEMV from 3 rows),
    K = 4096, N = 8300 (not a multiple of the 128-column tile); the oracle
    checks a seeded sample of columns."""
    st = np.array([gpu.rng_stream(5, gpu.STREAM_TESTING)], np.uint64)
    K, N = 4096, 8300
    x = gpu.synth_gaussian(st, 16 * K, 1.0).reshape(16, K)
    w = gpu.synth_gaussian(st, K * N, 0.02).reshape(K, N)
    q = gpu.QuantizedWeightMatrix.encode(w, bits)
    cols = np.sort(np.random.RandomState(bits).choice(N, 128, replace=False))
    cols[-1] = N - 1
    s_sub, p_sub = oracle.quantize_pack(np.ascontiguousarray(w[:, cols]), bits, 2)
    for M in (3, 5, 8, 11, 16):
        c = q.matmul(x[:M])
        assert c.shape == (M, N) and np.isfinite(c).all()
        ref = oracle.matmul_quantized(np.ascontiguousarray(x[:M]), K, len(cols), s_sub, p_sub, bits, 2)
        ok, err = _tol_ok(c[:, cols], ref)
        assert ok, (M, err)
    q.close()


def test_matmul_tensor_core_gemv_dynamic_range_and_nonfinite(gpu, oracle):
    """The GEMV at M = 12: rows spanning 2^-30 .. 2^20, a tiny row, and rows
    holding inf / NaN (NaN out, the other rows unaffected)."""
    rng = np.random.RandomState(12)
    m, k, n = 12, 1536, 1000
    w = (rng.randn(k, n) * 0.05).astype(np.float32)
    a = (rng.randn(m, k) * np.exp2(rng.randint(-30, 20, size=(m, k)))).astype(np.float32)
    a[5] *= 1e-30
    for bits in (8, 4):
        q = gpu.QuantizedWeightMatrix.encode(w, bits)
        s, p = oracle.quantize_pack(w, bits, 2)
        ref = oracle.matmul_quantized(a, k, n, s, p, bits, 2)
        c = q.matmul(a)
        for r in range(m):
            ok, err = _tol_ok(c[r], ref[r])
            assert ok, (bits, r, err)
        bad = a.copy()
        bad[3, 7] = np.inf
        bad[9, 100] = np.nan
        c = q.matmul(bad)
        assert np.isnan(c[9]).all() and not np.isfinite(c[3]).any()
        assert np.isfinite(np.delete(c, [3, 9], axis=0)).all()
        q.close()


@pytest.mark.parametrize("shape", [(256, 2048, 2048), (96, 8192, 2048), (64, 4096, 4096), (64, 4096, 1000)])
@pytest.mark.parametrize("bits", [8, 4])
def test_split_k_gemm_is_bit_identical(gpu, oracle, shape, bits):
    """Grids of fewer 128 x 128 tiles than half the SMs run split-K (the
    tile's k blocks in parts, int64 partial totals added by the last part).
    The totals are exact integers, so the result equals the unsplit GEMM's
    (the allocation-free entry point never splits) bit for bit, and the
    reference's tolerance against the oracle."""
    import torch
    from dranzer_b200 import _native
    L = _native.lib()
    m, k, n = shape
    rng = np.random.RandomState(m + k + n + bits)
    w = (rng.randn(k, n) * 0.02).astype(np.float32)
    a = rng.randn(m, k).astype(np.float32)
    q = gpu.QuantizedWeightMatrix.encode(w, bits)
    ad = torch.from_numpy(a).cuda()
    c_split = torch.zeros((m, n), dtype=torch.float32, device="cuda")
    c_plain = torch.full((m, n), float("nan"), dtype=torch.float32, device="cuda")
    stream = torch.cuda.Stream()
    for _ in range(2):   # the per-tile counters are zero again after a launch
        _native.check(L.dz_cuda_matmul_quantized_async(ad.data_ptr(), q.handle, c_split.data_ptr(), m, k,
                                                       stream.cuda_stream), "async")
        _native.check(L.dz_cuda_matmul_quantized_noalloc(ad.data_ptr(), q.handle, c_plain.data_ptr(), m, k,
                                                         stream.cuda_stream), "noalloc")
        stream.synchronize()
        np.testing.assert_array_equal(c_split.cpu().numpy().view(np.uint32), c_plain.cpu().numpy().view(np.uint32))
    s, p = oracle.quantize_pack(w, bits, 2)
    ref = oracle.matmul_quantized(a, k, n, s, p, bits, 2)
    ok, err = _tol_ok(c_split.cpu().numpy(), ref)
    assert ok, err
    q.close()


@pytest.mark.parametrize("bits", [8, 4])
def test_gemv_and_gemm_rows_bit_identical(gpu, bits):
    """The tensor-core GEMV (16 rows) and the tensor-core GEMM (17 rows)
    compute the same exact integer sums with one rounding: the 16 shared rows
    agree bit for bit."""
    st = np.array([gpu.rng_stream(9, gpu.STREAM_TESTING)], np.uint64)
    K, N = 4096, 2000
    x = gpu.synth_gaussian(st, 17 * K, 1.0).reshape(17, K)
    w = gpu.synth_gaussian(st, K * N, 0.02).reshape(K, N)
    q = gpu.QuantizedWeightMatrix.encode(w, bits)
    gemv = q.matmul(x[:16])
    gemm = q.matmul(x)
    np.testing.assert_array_equal(gemv, gemm[:16])
    q.close()
