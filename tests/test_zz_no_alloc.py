"""The allocation-free quantized matmul (dz_cuda_matmul_quantized_noalloc).

Callers that cannot allocate device memory when they call - code recording a
CUDA graph, hosts with no allocation rights after start-up - get the same
product as dz_cuda_matmul_quantized_async from a fixed static scratch array.
This file is collected last on purpose: a failure here leaves every other test
already run."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _tol_ok(c, ref):
    # the tolerance of src/tests/core/test_quantized_matmul.c:79
    return np.abs(c - ref).max() <= 1e-4 * (1 + np.abs(ref).max())


@pytest.mark.parametrize("bits", [4, 8])
def test_noalloc_matches_allocating_entry_point(gpu, bits):
    import torch
    from dranzer_b200 import _native
    L = _native.lib()
    K, N = 1000, 3000
    rng = np.random.RandomState(bits)
    w = (rng.randn(K, N) * 0.02).astype(np.float32)
    q = gpu.QuantizedWeightMatrix.encode(w, bits)
    stream = torch.cuda.Stream()
    for call, m in enumerate((5, 3)):   # two calls in a row on the shared array
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


def test_noalloc_rejects_oversized_calls(gpu):
    from dranzer_b200 import _native
    L = _native.lib()
    import torch
    q = gpu.QuantizedWeightMatrix.encode(np.ones((4096, 16), np.float32), 8)
    a = torch.zeros((171, 4096), dtype=torch.float32, device="cuda")
    c = torch.zeros((171, 16), dtype=torch.float32, device="cuda")
    # 86 row pairs x 16 x 4096 bytes of split activations are above the 4 MiB array
    st = L.dz_cuda_matmul_quantized_noalloc(a.data_ptr(), q.handle, c.data_ptr(), 171, 4096, None)
    assert st == -1
    assert "static" in _native.last_error()[1]
    q.close()
