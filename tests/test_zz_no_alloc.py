"""GPU: acfun_gemm_epi_noalloc, the GEMM entry point that allocates no device memory.

It exists for callers that cannot call cudaMalloc — a process that has reserved all device
memory in its own pool, code running inside an out-of-memory handler or an allocator
callback, a latency-critical loop in which cudaMalloc / cudaFree would synchronise the
device.  Its scratch is a fixed array compiled into the library, so the caller passes only
device inputs and outputs.  This test checks, through the C ABI, on calls made back to back
on the shared array: the result against the CPU oracle (within the fp32 tolerance the other
tests use) and bit for bit against the allocating entry point acfun_gemm_epi in 3xTF32 mode,
whose arithmetic it shares; every tile width it can choose (32, 64 and 128 columns); and that
sizes beyond the array, host pointers and pointers on no device are rejected with an error
instead of being staged.

The file is named so that pytest collects it last: a failure here never hides another test.
"""
import numpy as np
import pytest

from helpers import TOL_F32, assert_bits_equal, max_rel

pytestmark = pytest.mark.gpu


def _dev(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _reference_result(acf, A, B, bias, act):
    """The existing (allocating) entry point on the same device tensors, in 3xTF32 mode (the
    no-alloc entry point's arithmetic); the process-wide mode is restored afterwards."""
    import torch
    M, K = A.shape
    N = B.shape[1]
    C = torch.empty((M, N), dtype=torch.float32, device="cuda")
    L = acf.lib()
    assert L.acfun_set_fp32_math(1) == 0
    try:
        L.acfun_gemm_epi(M, N, K, A.data_ptr(), B.data_ptr(), C.data_ptr(),
                         bias.data_ptr() if bias is not None else None, act)
        acf.synchronize()
        acf.check()
    finally:
        L.acfun_set_fp32_math(0)
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


def _oracle_result(orc, A, B, bias, act):
    a, b = A.cpu().numpy(), B.cpu().numpy()
    M, K = a.shape
    N = b.shape[1]
    out = np.empty((M, N), np.float32)
    bb = None if bias is None else bias.cpu().numpy()
    orc.oracle().orc_gemm_f32(M, N, K, a, b, out, None if bb is None else bb.ctypes.data, act)
    return out


# (M, N, K, bias, act): the BASELINE SGEMM size (BN = 128 tiles would be too few: 64-column
# tiles), a ragged problem without bias (32-column tiles), and 4096 x 1024 x 256, which has
# enough 128-column tiles for the 128-wide variant and fills most of the 16 MiB array
SHAPES = [(1024, 1024, 1024, True, 1), (333, 29, 129, False, 0), (4096, 1024, 256, True, 0)]


def test_noalloc_matches_oracle_and_allocating_gemm_on_calls_in_a_row(acf, orc):
    g = np.random.default_rng(11)
    for M, N, K, has_bias, act in SHAPES:
        A = _dev(g.uniform(-1, 1, (M, K)).astype(np.float32))
        B = _dev(g.uniform(-1, 1, (K, N)).astype(np.float32))
        b = _dev(g.uniform(-1, 1, N).astype(np.float32)) if has_bias else None
        got = _noalloc_result(acf, A, B, b, act)
        assert np.isfinite(got).all()
        ref = _oracle_result(orc, A, B, b, act)
        assert max_rel(got, ref) < TOL_F32, ((M, N, K), max_rel(got, ref))
        assert_bits_equal(got, _reference_result(acf, A, B, b, act), f"{M}x{N}x{K} vs acfun_gemm_epi")


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
