"""The allocation-free quantized matmul (dz_cuda_matmul_quantized_noalloc).

Some hosts budget all device memory at start-up and give the library no right
to call cudaMalloc afterwards; they multiply through this entry point, which
takes its scratch from a fixed static device array instead of growing a buffer.
These tests check that it gives the product of dz_cuda_matmul_quantized_async,
on two calls in a row (the array keeps the previous call's contents), on the
CUDA-core matvec path and on the tensor-core GEMV path (whose tile counters
live in the array), and that calls too large for the array are refused.
This file is collected last on purpose: a failure here leaves every other test
already run."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _tol_ok(c, ref):
    # the tolerance of src/tests/core/test_quantized_matmul.c:79
    return np.abs(c - ref).max() <= 1e-4 * (1 + np.abs(ref).max())


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("shape", [(1000, 3000, (5, 3)), (4096, 8300, (12, 9))])
def test_noalloc_matches_allocating_entry_point(gpu, bits, shape):
    import torch
    from dranzer_b200 import _native
    L = _native.lib()
    K, N, ms = shape
    rng = np.random.RandomState(bits)
    w = (rng.randn(K, N) * 0.02).astype(np.float32)
    q = gpu.QuantizedWeightMatrix.encode(w, bits)
    stream = torch.cuda.Stream()
    for call, m in enumerate(ms):   # two calls in a row on the shared array
        a = torch.from_numpy(rng.randn(m, K).astype(np.float32)).cuda()
        c_ref = torch.zeros((m, N), dtype=torch.float32, device="cuda")
        c_new = torch.full((m, N), float("nan"), dtype=torch.float32, device="cuda")
        torch.cuda.synchronize()
        _native.check(L.dz_cuda_matmul_quantized_async(a.data_ptr(), q.handle, c_ref.data_ptr(), m, K,
                                                       stream.cuda_stream), "async")
        _native.check(L.dz_cuda_matmul_quantized_noalloc(a.data_ptr(), q.handle, c_new.data_ptr(), m, K,
                                                         stream.cuda_stream), "noalloc")
        stream.synchronize()
        ref, new = c_ref.cpu().numpy(), c_new.cpu().numpy()
        assert np.isfinite(new).all(), call
        assert _tol_ok(new, ref), (call, np.abs(new - ref).max())
    q.close()


@pytest.mark.parametrize("bits", [4, 8])
def test_noalloc_first_call_gemm_and_no_growth(gpu, bits):
    """A fresh matrix whose first product goes through the allocation-free
    entry point, at 64 rows (the tensor-core GEMM, its limbs and TMA map in
    the static array), then 1 row (the M <= 2 matvec); both against the
    allocating entry point afterwards, and a repeated call leaves the
    device's free memory unchanged."""
    import torch
    from dranzer_b200 import _native
    L = _native.lib()
    K, N = 4096, 8300
    rng = np.random.RandomState(40 + bits)
    w = (rng.randn(K, N) * 0.02).astype(np.float32)
    q = gpu.QuantizedWeightMatrix.encode(w, bits)
    stream = torch.cuda.Stream()
    for m in (64, 1):
        a = torch.from_numpy(rng.randn(m, K).astype(np.float32)).cuda()
        c_new = torch.full((m, N), float("nan"), dtype=torch.float32, device="cuda")
        c_ref = torch.zeros((m, N), dtype=torch.float32, device="cuda")
        torch.cuda.synchronize()
        _native.check(L.dz_cuda_matmul_quantized_noalloc(a.data_ptr(), q.handle, c_new.data_ptr(), m, K,
                                                         stream.cuda_stream), "noalloc")
        stream.synchronize()
        free0 = torch.cuda.mem_get_info()[0]
        _native.check(L.dz_cuda_matmul_quantized_noalloc(a.data_ptr(), q.handle, c_new.data_ptr(), m, K,
                                                         stream.cuda_stream), "noalloc")
        stream.synchronize()
        assert torch.cuda.mem_get_info()[0] == free0, m
        _native.check(L.dz_cuda_matmul_quantized_async(a.data_ptr(), q.handle, c_ref.data_ptr(), m, K,
                                                       stream.cuda_stream), "async")
        stream.synchronize()
        ref, new = c_ref.cpu().numpy(), c_new.cpu().numpy()
        assert np.isfinite(new).all(), m
        assert _tol_ok(new, ref), (m, np.abs(new - ref).max())
    q.close()


def test_noalloc_rejects_oversized_calls(gpu):
    from dranzer_b200 import _native
    L = _native.lib()
    import torch
    q = gpu.QuantizedWeightMatrix.encode(np.ones((4096, 16), np.float32), 8)
    a = torch.zeros((300, 4096), dtype=torch.float32, device="cuda")
    c = torch.zeros((300, 16), dtype=torch.float32, device="cuda")
    # 150 row pairs x 16 x 4096 bytes of split activations are above the 8 MiB array
    st = L.dz_cuda_matmul_quantized_noalloc(a.data_ptr(), q.handle, c.data_ptr(), 300, 4096, None)
    assert st == -1
    assert "static" in _native.last_error()[1]
    q.close()
