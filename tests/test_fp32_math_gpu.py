"""GPU: measured error of the two fp32 tensor-core modes (3xTF32, 3xBF16) against float64,
on the SGEMM, FC and conv shapes of the BASELINE configs.  Both must stay inside the fp32
parity tolerance (max-rel 1e-4 after scaling by max|ref|); the measured values justify the
default choice written in acfun.h."""
import numpy as np
import pytest

from helpers import TOL_F32, max_rel

pytestmark = pytest.mark.gpu


def _conv_ref64(x, w, b, KH, stride, pad, act):
    N, H, W, Cin = x.shape
    Cout = w.shape[1]
    OH, OW = (H + 2 * pad - KH) // stride + 1, (W + 2 * pad - KH) // stride + 1
    xp = np.pad(x.astype(np.float64), ((0, 0), (pad, pad), (pad, pad), (0, 0)))
    wk = w.astype(np.float64).reshape(KH, KH, Cin, Cout)
    out = np.zeros((N, OH, OW, Cout)) + b
    for kh in range(KH):
        for kw in range(KH):
            out += np.einsum("nhwc,co->nhwo", xp[:, kh:kh + stride * OH:stride, kw:kw + stride * OW:stride, :], wk[kh, kw])
    return np.maximum(out, 0) if act else out


@pytest.mark.parametrize("mode,name", [(1, "tf32x3"), (2, "bf16x3")])
def test_fp32_modes_measured_error(acf, mode, name):
    L = acf.lib()
    assert L.acfun_set_fp32_math(mode) == 0
    try:
        g = np.random.default_rng(31)
        errs = {}
        A = g.uniform(-1, 1, (1024, 1024)).astype(np.float32)
        B = g.uniform(-1, 1, (1024, 1024)).astype(np.float32)
        errs["sgemm1024"] = max_rel(acf.gemm(A, B), A.astype(np.float64) @ B.astype(np.float64))
        x = g.uniform(-1, 1, (16, 3072)).astype(np.float32)
        w = (g.uniform(-1, 1, (3072, 512)) / 30).astype(np.float32)
        bb = g.uniform(-0.1, 0.1, 512).astype(np.float32)
        errs["fc3072"] = max_rel(acf.fc(x, w, bb, 1), np.maximum(x.astype(np.float64) @ w + bb, 0))
        xc = g.uniform(0, 1, (2, 28, 28, 64)).astype(np.float32)
        wc = g.uniform(-np.sqrt(6 / 576), np.sqrt(6 / 576), (576, 64)).astype(np.float32)
        bc = g.uniform(-0.1, 0.1, 64).astype(np.float32)
        errs["conv3x3"] = max_rel(acf.conv2d(xc, wc, bc, 3, 3, 64, 1, 1, 1), _conv_ref64(xc, wc, bc, 3, 1, 1, 1))
        print(f"measured max-rel vs float64 ({name}):", {k: f"{v:.2e}" for k, v in errs.items()})
        for k, v in errs.items():
            assert v < TOL_F32, (name, k, v)
    finally:
        L.acfun_set_fp32_math(0)
