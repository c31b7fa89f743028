"""CPU: pin the oracle (oracle/acfun_oracle.c + oracle/model_oracle.py) against the golden
vectors the reference produced (tests/golden, see make_golden.py), and — when the reference
library was built here (oracle/_ref) — against fresh reference runs on new seeds."""
import glob
import os

import numpy as np
import pytest

from helpers import TOL_BF16, TOL_F32, assert_bits_equal, max_rel

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def load(name):
    return dict(np.load(os.path.join(GOLD, name + ".npz")))


def names(prefix):
    return sorted(os.path.basename(p)[:-4] for p in glob.glob(os.path.join(GOLD, prefix + "*.npz")))


def test_golden_inventory():
    assert len(names("")) >= 40


@pytest.mark.parametrize("name", [n for n in names("gemm_int8_") if "_epi_" not in n])
def test_oracle_gemm_int8(orc, name):
    d = load(name)
    M, K = d["A"].shape
    N = d["B"].shape[1]
    C = np.empty((M, N), np.int32)
    orc.oracle().orc_gemm_int8(M, N, K, d["A"], d["B"], C)
    assert_bits_equal(C, d["C"], name)


@pytest.mark.parametrize("name", names("gemm_int8_epi_"))
def test_oracle_gemm_int8_epi(orc, name):
    d = load(name)
    M, K = d["A"].shape
    N = d["B"].shape[1]
    C = np.empty((M, N), np.float32)
    orc.oracle().orc_gemm_int8_epi(M, N, K, d["A"], d["B"], C, d["alpha"], d["beta"], int(d["act"]))
    assert_bits_equal(C, d["C"], name)


@pytest.mark.parametrize("name", names("gemm_s8_requant"))
def test_oracle_s8_requant(orc, name):
    d = load(name)
    M, K = d["A"].shape
    N = d["B"].shape[1]
    C = np.empty((M, N), np.int8)
    orc.oracle().orc_gemm_s8_requant(M, N, K, d["A"], d["B"], d["bias"].ctypes.data, d["scale"], C,
                                     int(d["act"]))
    assert_bits_equal(C, d["C"], name)
    # saturation is the common case at BASELINE value ranges
    assert (np.abs(C.astype(int)) == 127).mean() > 0.3 or int(d["act"]) == 1


def test_oracle_quantize(orc):
    d = load("quantize_u8")
    q = np.empty(d["x"].size, np.uint8)
    orc.oracle().orc_quantize_u8(d["x"], q, q.size, np.float32(1.0), 128, 1)
    assert_bits_equal(q, d["q"], "quantize_u8 (rne)")


@pytest.mark.parametrize("name", names("conv_int8_"))
def test_oracle_conv_int8(orc, name):
    d = load(name)
    N, H, W, Cin, KH, KW, Cout, st, pd, act = (int(v) for v in d["shape"])
    ws = np.empty(Cout, np.float32)
    wq = np.empty((KH * KW * Cin, Cout), np.int8)
    orc.oracle().orc_quantize_weights(d["w"], KH * KW * Cin, Cout, ws, wq)
    assert_bits_equal(wq, d["wq"], name + " wq")
    assert_bits_equal(ws, d["ws"], name + " ws")
    out = orc.orc_conv2d_int8(d["x"], wq, ws, d["b"], N, H, W, Cin, KH, KW, Cout, st, pd, act)
    assert_bits_equal(out, d["out"], name)


def test_int8_winograd_is_an_exact_integer_conv(orc):
    """The identity the GPU int8-Winograd route relies on: with G~ = 2G integral, the
    reference's transform pipeline equals fmaf(4*(float)sum((xq-128)*wq), wso, bias)."""
    d = load("conv_int8_wino_a1")
    N, H, W, Cin, KH, KW, Cout, st, pd, act = (int(v) for v in d["shape"])
    x = d["x"]
    maxa = np.float32(np.abs(x).max())
    inv_s = np.float32(127.0) / maxa
    sa = maxa / np.float32(127.0)
    t = (x * inv_s).astype(np.float32)
    cvec = Cin & ~15
    q = np.empty_like(t, dtype=np.int64)
    r = (t + np.copysign(np.float32(0.5), t).astype(np.float32)).astype(np.float32)
    q[..., :cvec] = np.trunc(r[..., :cvec]).astype(np.int64)
    tail = t[..., cvec:].astype(np.float64)
    q[..., cvec:] = (np.sign(tail) * np.floor(np.abs(tail) + 0.5)).astype(np.int64)
    xq = np.clip(q + 128, 0, 255) - 128           # centred, zero padding == zp padding
    xp = np.pad(xq, ((0, 0), (1, 1), (1, 1), (0, 0)))
    wq = d["wq"].astype(np.int64).reshape(3, 3, Cin, Cout)
    acc = np.zeros((N, H, W, Cout), np.int64)
    for kh in range(3):
        for kw in range(3):
            acc += np.einsum("nhwc,co->nhwo", xp[:, kh:kh + H, kw:kw + W, :], wq[kh, kw])
    wso = (sa * np.float32(0.25)) * d["ws"]
    y = (4 * acc).astype(np.float32)
    # fmaf in float64 then one rounding is exact for these magnitudes (|y*wso| < 2^24 ulps)
    v = (y.astype(np.float64) * wso.astype(np.float64) + d["b"].astype(np.float64)).astype(np.float32)
    v = np.where(v > 0, v, np.float32(0))
    assert_bits_equal(v, d["out"], "int8 winograd == exact integer correlation")


@pytest.mark.parametrize("name", names("gemm_f32_"))
def test_oracle_gemm_f32_and_bf16(orc, name):
    d = load(name)
    M, K = d["A"].shape
    N = d["B"].shape[1]
    C = np.empty((M, N), np.float32)
    orc.oracle().orc_gemm_f32(M, N, K, d["A"], d["B"], C, d["bias"].ctypes.data, 1)
    assert max_rel(C, d["C_epi_relu"]) < TOL_F32
    Cb = np.empty((M, N), np.float32)
    orc.oracle().orc_gemm_bf16(M, N, K, d["A"], d["B"], Cb)
    assert max_rel(Cb, d["C_bf16"]) < TOL_BF16


@pytest.mark.parametrize("name", names("conv_f32_") + names("conv_dw") + names("conv_grp"))
def test_oracle_conv_f32(orc, name):
    d = load(name)
    N, H, W, Cin, KH, KW, Cout, st, pd, act, groups = (int(v) for v in d["shape"])
    OH, OW = orc.conv_out_hw(H, W, KH, KW, st, pd)
    out = np.empty((N, OH, OW, Cout), np.float32)
    orc.oracle().orc_conv2d(d["x"], N, H, W, Cin, np.ascontiguousarray(d["w"]), d["b"].ctypes.data,
                            KH, KW, Cout, st, pd, groups, out, act)
    assert max_rel(out, d["out"]) < TOL_F32, name
    if orc.oracle().orc_conv2d_route(N, H, W, Cin, KH, KW, Cout, st, pd, groups) in (1, 2):
        # depthwise and grouped-direct routes: the oracle restates the AVX-512 / AVX2 fma chains
        assert_bits_equal(out, d["out"], name)
    if name == "conv_f32_wino23":
        o2 = np.empty_like(out)
        orc.oracle().orc_winograd23(d["x"], N, H, W, Cin, d["w"], d["b"].ctypes.data, Cout, o2, act)
        assert max_rel(o2, d["out"]) < 1e-6
    if name == "conv_f32_wino43":
        o2 = np.empty_like(out)
        orc.oracle().orc_winograd43(d["x"], N, H, W, Cin, d["w"], d["b"].ctypes.data, Cout, o2, act)
        assert max_rel(o2, d["out"]) < 1e-5


@pytest.mark.parametrize("name", names("maxpool_"))
def test_oracle_maxpool(orc, name):
    d = load(name)
    N, H, W, C, pool, st, pd, post = (int(v) for v in d["shape"])
    out = np.empty_like(d["out"])
    orc.oracle().orc_maxpool(d["x"], N, H, W, C, pool, st, pd, out, post)
    assert_bits_equal(out, d["out"], name)


def test_oracle_softmax_bn_fc(orc):
    O = orc.oracle()
    d = load("softmax")
    out = np.empty_like(d["x"])
    O.orc_softmax(d["x"], 3, 1000, out)
    assert max_rel(out, d["out"]) < 1e-6
    d = load("batchnorm")
    x = d["x"].copy()
    O.orc_batchnorm(x, x.size, 12, d["mean"], d["var"], d["gamma"].ctypes.data, d["beta"].ctypes.data,
                    np.float32(1e-5))
    assert_bits_equal(x, d["out"], "batchnorm")
    d = load("fc")
    o = np.empty((5, 70), np.float32)
    O.orc_fc(d["x"], 5, 300, d["w"], d["b"].ctypes.data, 70, o, 0)
    assert max_rel(o, d["out"]) < TOL_F32
    O.orc_fc(d["x"], 5, 300, d["w"], d["b"].ctypes.data, 70, o, 1)
    assert max_rel(o, d["out_relu"]) < TOL_F32


def test_oracle_model_demo(orc):
    from oracle.model_oracle import OracleModel
    d = load("model_demo")
    m = OracleModel(d["blob"].tobytes())
    for k in range(d["x"].shape[0]):
        y = m.infer(d["x"][k])
        assert y.shape == d["out"][k].shape
        assert max_rel(y, d["out"][k]) < TOL_F32


# ---------------------------------------------------------------- live reference (optional)
ref_only = pytest.mark.skipif(not os.path.exists(os.path.join(os.path.dirname(GOLD), "..", "oracle", "_ref",
                                                              "libacfun_ref.so")),
                              reason="reference library not built on this host")


@ref_only
@pytest.mark.parametrize("seed", [1, 2, 3])
def test_oracle_conv_int8_vs_reference_fresh_seeds(orc, seed):
    g = np.random.default_rng(seed)
    O = orc.oracle()
    for (N, H, W, Cin, KH, KW, Cout, st, pd) in [(1, 7, 9, 16, 3, 3, 12, 1, 1), (2, 6, 6, 5, 3, 3, 8, 1, 1),
                                                 (1, 9, 8, 4, 5, 5, 6, 2, 2), (1, 5, 5, 70, 1, 1, 9, 1, 0),
                                                 (1, 8, 8, 24, 3, 3, 10, 2, 1)]:
        x = g.uniform(-2, 2, (N, H, W, Cin)).astype(np.float32)
        w = g.uniform(-0.3, 0.3, (KH * KW * Cin, Cout)).astype(np.float32)
        ws = np.empty(Cout, np.float32)
        wq = np.empty((KH * KW * Cin, Cout), np.int8)
        O.orc_quantize_weights(w, KH * KW * Cin, Cout, ws, wq)
        b = g.uniform(-1, 1, Cout).astype(np.float32)
        for act in (0, 1):
            a = orc.orc_conv2d_int8(x, wq, ws, b, N, H, W, Cin, KH, KW, Cout, st, pd, act)
            r = orc.ref_conv2d_int8(x, wq, ws, b, N, H, W, Cin, KH, KW, Cout, st, pd, act)
            assert_bits_equal(a, r, f"seed {seed} {(N, H, W, Cin, KH, KW, Cout, st, pd, act)}")


@ref_only
@pytest.mark.parametrize("case", [
    # (N, H, W, Cin, Cout, groups, K, stride, pad, act): BASELINE cfg4 shapes (fewer images),
    # plus the AVX-512 masked channel tail (C % 16 != 0) and Cout_per >= 16 / < 8 / = 8
    (2, 56, 56, 144, 144, 144, 3, 1, 1, 1), (2, 13, 11, 21, 21, 21, 3, 2, 1, 0),
    (4, 14, 14, 24, 48, 6, 3, 1, 1, 1), (4, 14, 14, 24, 48, 6, 3, 2, 1, 1),
    (2, 9, 9, 16, 80, 4, 3, 1, 1, 0), (2, 7, 7, 6, 60, 3, 3, 2, 1, 1), (2, 9, 9, 8, 12, 4, 3, 1, 1, 1),
])
def test_oracle_dw_grouped_vs_reference_exact(orc, case):
    """Depthwise and grouped-direct routes: the oracle equals the compiled reference bit for bit
    (the fma chains of dw_avx512.cpp and group_conv_avx512.cpp / _avx2.cpp)."""
    N, H, W, Cin, Cout, gr, K, st, pd, act = case
    g = np.random.default_rng(sum(case))
    x = g.uniform(-1, 1, (N, H, W, Cin)).astype(np.float32)
    if gr == Cin == Cout:
        w = g.uniform(-1, 1, (Cin, K, K)).astype(np.float32)
    else:
        w = g.uniform(-1, 1, (gr, K * K * (Cin // gr), Cout // gr)).astype(np.float32)
    b = g.uniform(-0.1, 0.1, Cout).astype(np.float32)
    OH, OW = orc.conv_out_hw(H, W, K, K, st, pd)
    a = np.empty((N, OH, OW, Cout), np.float32)
    r = np.empty_like(a)
    orc.oracle().orc_conv2d(x, N, H, W, Cin, w, b.ctypes.data, K, K, Cout, st, pd, gr, a, act)
    orc.ref().acfun_conv2d_g(x, N, H, W, Cin, w, b.ctypes.data, K, K, Cout, st, pd, gr, r, act)
    assert_bits_equal(a, r, str(case))


@ref_only
def test_oracle_model_vs_reference_vgg_small(orc, tmp_path):
    from acfun_b200 import acfun0
    from oracle.model_oracle import OracleModel
    blob = acfun0.vgg11(seed=3, in_hw=32, width_div=16, fc_dims=(64, 32, 10)).tobytes()
    p = tmp_path / "v.acfun"
    p.write_bytes(blob)
    R = orc.ref()
    h = R.acfun_model_load(str(p).encode())
    assert h
    x = np.random.default_rng(4).uniform(0, 1, (32, 32, 3)).astype(np.float32)
    o = np.empty(10, np.float32)
    assert R.acfun_model_infer(h, x, o) == 10
    R.acfun_model_destroy(h)
    y = OracleModel(blob).infer(x)
    assert max_rel(y, o) < TOL_F32


@ref_only
def test_int8_model_composition_oracle_vs_reference(tmp_path):
    """The int8 VGG composition (quantize_weights + conv2d_int8 per dense conv, per image) in
    the oracle equals the same composition run on the reference library, bit for bit; the
    fp32 harness equals the reference's own acfun_model_infer."""
    from acfun_b200 import acfun0
    from oracle import pyoracle as P
    from oracle.model_oracle import OracleModel
    R = P.ref()
    blob = acfun0.vgg11(seed=3, in_hw=32, width_div=16, fc_dims=(64, 32, 10)).tobytes()
    path = tmp_path / "v.acfun"
    path.write_bytes(blob)
    om = OracleModel(blob)
    h = R.acfun_model_load(str(path).encode())
    try:
        for seed in (1, 2):
            x = np.random.default_rng(seed).uniform(-1, 2, (32, 32, 3)).astype(np.float32)
            o = np.empty(10, np.float32)
            R.acfun_model_infer(h, x, o)
            np.testing.assert_array_equal(om.ref_infer(R, x), o)
            np.testing.assert_array_equal(om.infer(x, int8=True).view(np.int32),
                                          om.ref_infer(R, x, int8=True).view(np.int32))
    finally:
        R.acfun_model_destroy(h)
