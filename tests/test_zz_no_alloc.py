"""GPU: acfun_gemm_epi_noalloc, the GEMM entry point that allocates no device memory.

It exists for callers that cannot call cudaMalloc — a process that has reserved all device
memory in its own pool, code running inside an out-of-memory handler or an allocator
callback, a latency-critical loop in which cudaMalloc / cudaFree would synchronise the
device.  Its scratch is a fixed array compiled into the library, so the caller passes only
device inputs and outputs.  This test checks, through the C ABI, that two calls in a row
give the same result as the allocating entry point acfun_gemm_epi (within the fp32
tolerance the other tests use), that the second call is not polluted by what the first
left in the shared array, and that sizes beyond the array and host pointers are rejected
with an error instead of being staged.

The file is named so that pytest collects it last: a failure here never hides another test.
"""
import numpy as np
import pytest

from helpers import TOL_F32, max_rel

pytestmark = pytest.mark.gpu


def _dev(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _reference_result(acf, A, B, bias, act):
    """The existing (allocating) entry point on the same device tensors."""
    import torch
    M, K = A.shape
    N = B.shape[1]
    C = torch.empty((M, N), dtype=torch.float32, device="cuda")
    acf.lib().acfun_gemm_epi(M, N, K, A.data_ptr(), B.data_ptr(), C.data_ptr(),
                             bias.data_ptr() if bias is not None else None, act)
    acf.synchronize()
    acf.check()
    return C.cpu().numpy()


def _noalloc_result(acf, A, B, bias, act):
    import torch
    M, K = A.shape
    N = B.shape[1]
    C = torch.full((M, N), float("nan"), dtype=torch.float32, device="cuda")
    rc = acf.lib().acfun_gemm_epi_noalloc(M, N, K, A.data_ptr(), B.data_ptr(), C.data_ptr(),
                                          bias.data_ptr() if bias is not None else None, act)
    assert rc == 0, acf.lib().acfun_last_error().decode()
    return C.cpu().numpy()


def test_noalloc_matches_allocating_gemm_on_two_calls(acf):
    g = np.random.default_rng(11)
    # first call: the BASELINE SGEMM size (fills most of the 16 MiB array)
    A1 = _dev(g.uniform(-1, 1, (1024, 1024)).astype(np.float32))
    B1 = _dev(g.uniform(-1, 1, (1024, 1024)).astype(np.float32))
    b1 = _dev(g.uniform(-1, 1, 1024).astype(np.float32))
    got1 = _noalloc_result(acf, A1, B1, b1, 1)
    ref1 = _reference_result(acf, A1, B1, b1, 1)
    assert np.isfinite(got1).all()
    assert max_rel(got1, ref1) < TOL_F32, max_rel(got1, ref1)
    # second call right after: a smaller, ragged problem without bias on the same array
    A2 = _dev(g.uniform(-1, 1, (333, 129)).astype(np.float32))
    B2 = _dev(g.uniform(-1, 1, (129, 47)).astype(np.float32))
    got2 = _noalloc_result(acf, A2, B2, None, 0)
    ref2 = _reference_result(acf, A2, B2, None, 0)
    assert np.isfinite(got2).all()
    assert max_rel(got2, ref2) < TOL_F32, max_rel(got2, ref2)


def test_noalloc_rejects_oversize_and_host_memory(acf):
    import torch
    L = acf.lib()
    big = torch.zeros((2048, 2048), dtype=torch.float32, device="cuda")
    out = torch.zeros((2048, 2048), dtype=torch.float32, device="cuda")
    rc = L.acfun_gemm_epi_noalloc(2048, 2048, 2048, big.data_ptr(), big.data_ptr(), out.data_ptr(), None, 0)
    assert rc == 1 and "maximum" in L.acfun_last_error().decode()
    L.acfun_clear_error()
    h = np.zeros((8, 8), np.float32)
    rc = L.acfun_gemm_epi_noalloc(8, 8, 8, acf.ptr(h), acf.ptr(h), acf.ptr(h), None, 0)
    assert rc == 1 and "device pointers" in L.acfun_last_error().decode()
    L.acfun_clear_error()
