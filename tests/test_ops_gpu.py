"""GPU parity: bandwidth kernels (ReLU/ReLU6, max-pool, softmax, batch-norm, u8 quantise,
depthwise, grouped) against the golden vectors and the oracle."""
import os

import numpy as np
import pytest

from helpers import TOL_F32, assert_bits_equal, max_rel

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def load(name):
    return dict(np.load(os.path.join(GOLD, name + ".npz")))


def test_relu_relu6(acf, orc):
    g = np.random.default_rng(0)
    x = g.uniform(-10, 10, 100003).astype(np.float32)
    x[:4] = [-0.0, 0.0, 6.0, -1e-30]
    for six, fn in ((0, "acfun_relu"), (1, "acfun_relu6")):
        y = x.copy()
        getattr(acf.lib(), fn)(acf.ptr(y), y.size)
        acf.check()
        r = x.copy()
        (orc.oracle().orc_relu6 if six else orc.oracle().orc_relu)(r, r.size)
        assert_bits_equal(y, r, fn)


@pytest.mark.parametrize("name", ["maxpool_mp2", "maxpool_mp3", "maxpool_mp2_c64"])
def test_maxpool_golden(acf, name):
    d = load(name)
    N, H, W, C, pool, st, pd, post = (int(v) for v in d["shape"])
    assert_bits_equal(acf.maxpool(d["x"], pool, st, pd, post), d["out"], name)


@pytest.mark.parametrize("shape", [(2, 224, 224, 64, 2, 2, 0), (1, 15, 13, 7, 3, 2, 1), (4, 14, 14, 512, 2, 2, 0),
                                   (1, 9, 9, 12, 2, 1, 0), (1, 5, 5, 16, 3, 3, 2)])
def test_maxpool_vs_oracle(acf, orc, shape):
    N, H, W, C, pool, st, pd = shape
    x = np.random.default_rng(C).uniform(-1, 1, (N, H, W, C)).astype(np.float32)
    for post in (0, 1):
        OH, OW = orc.conv_out_hw(H, W, pool, pool, st, pd)
        r = np.empty((N, OH, OW, C), np.float32)
        orc.oracle().orc_maxpool(x, N, H, W, C, pool, st, pd, r, post)
        assert_bits_equal(acf.maxpool(x, pool, st, pd, post), r, f"maxpool {shape} post={post}")


def test_softmax_golden(acf):
    d = load("softmax")
    assert max_rel(acf.softmax(d["x"]), d["out"]) < TOL_F32
    x = np.random.default_rng(3).uniform(-30, 30, (256, 1000)).astype(np.float32)
    ref = np.empty_like(x)
    from oracle import pyoracle
    pyoracle.oracle().orc_softmax(x, 256, 1000, ref)
    assert max_rel(acf.softmax(x), ref) < TOL_F32


def test_batchnorm_exact(acf):
    d = load("batchnorm")
    x = d["x"].copy()
    acf.lib().acfun_batchnorm(acf.ptr(x), x.size, 12, acf.ptr(d["mean"]), acf.ptr(d["var"]),
                              acf.ptr(d["gamma"]), acf.ptr(d["beta"]), 1e-5)
    acf.check()
    assert_bits_equal(x, d["out"], "batchnorm")


def test_quantize_u8_exact(acf, orc):
    d = load("quantize_u8")
    q = np.empty(d["x"].size, np.uint8)
    acf.lib().acfun_quantize_u8(acf.ptr(d["x"]), acf.ptr(q), q.size, 1.0, 128)
    acf.check()
    assert_bits_equal(q, d["q"], "quantize golden (ties to even, out-of-range -> 0)")
    x = np.random.default_rng(9).uniform(-2, 2, 1 << 20 | 3).astype(np.float32)
    for inv in (63.5, 127.0 / 1.999):
        r = np.empty(x.size, np.uint8)
        orc.oracle().orc_quantize_u8(x, r, x.size, np.float32(inv), 128, 1)
        acf.lib().acfun_quantize_u8(acf.ptr(x), acf.ptr(q := np.empty(x.size, np.uint8)), x.size, inv, 128)
        acf.check()
        assert_bits_equal(q, r, f"quantize inv_s={inv}")


@pytest.mark.parametrize("name", ["conv_dw_s1", "conv_dw_s2"])
def test_depthwise_golden_exact(acf, name):
    d = load(name)
    N, H, W, C, KH, KW, _, st, pd, act, _ = (int(v) for v in d["shape"])
    got = acf.conv2d_dw(d["x"], np.ascontiguousarray(d["w"]), d["b"], KH, KW, st, pd, act)
    assert_bits_equal(got, d["out"], name)      # same FMA chain as the AVX-512 kernel


def test_depthwise_cfg4_size(acf, orc):
    """BASELINE cfg4 depthwise: N=32, 56x56x144, 3x3 s1 p1, bias + ReLU; every image bit for
    bit against the oracle (the kernel keeps the reference's per-output fma chain)."""
    g = np.random.default_rng(44)
    N, H, W, C = 32, 56, 56, 144
    x = g.uniform(0, 1, (N, H, W, C)).astype(np.float32)
    w = g.uniform(-np.sqrt(6 / 9), np.sqrt(6 / 9), (C, 3, 3)).astype(np.float32)
    b = g.uniform(-0.1, 0.1, C).astype(np.float32)
    got = acf.conv2d_dw(x, w, b, 3, 3, 1, 1, 1)
    ref = np.empty_like(x)
    orc.oracle().orc_conv2d(x, N, H, W, C, w, b.ctypes.data, 3, 3, C, 1, 1, C, ref, 1)
    assert_bits_equal(got, ref, "cfg4 depthwise")


@pytest.mark.parametrize("N,H,W,C,bias,act", [
    (4, 112, 112, 32, True, 1),   # 128 tiles of 7 rows x 56 columns: the TMA-fed kernel
    (2, 17, 13, 12, True, 1),     # odd width narrower than a column strip, ragged last row strip
    (1, 30, 33, 40, False, 0),    # no bias, no ReLU
    (3, 16, 250, 8, True, 1),     # a 250-column strip (box row of 252 pixels)
    (2, 6, 9, 512, True, 1),      # C > 256: channel groups, fewer rows than a strip
    (1, 9, 10, 144, True, 0),
    (32, 56, 56, 8, True, 1),     # more tiles than SMs: the register-window kernel
])
def test_depthwise_tma_route_exact(acf, orc, N, H, W, C, bias, act):
    """3x3 s1 p1 depthwise maps whose tiles fit one wave of CTAs run k_dw3_tma (TMA halo boxes
    into shared memory, dw_tma.cu), the others k_dw3_roll; both keep the reference's per-output
    fma chain, so every element equals the oracle bit for bit, borders and ragged strips included."""
    g = np.random.default_rng(N * 1000 + H * 10 + W + C)
    x = g.uniform(-1, 1, (N, H, W, C)).astype(np.float32)
    w = g.uniform(-0.8, 0.8, (C, 3, 3)).astype(np.float32)
    b = g.uniform(-0.1, 0.1, C).astype(np.float32) if bias else None
    got = acf.conv2d_dw(x, w, b, 3, 3, 1, 1, act)
    ref = np.empty_like(x)
    orc.oracle().orc_conv2d(x, N, H, W, C, w, b.ctypes.data if bias else None, 3, 3, C, 1, 1, C, ref, act)
    assert_bits_equal(got, ref, f"depthwise {N}x{H}x{W}x{C}")


@pytest.mark.parametrize("st", [1, 2])
def test_grouped_cfg4_size_exact(acf, orc, st):
    """BASELINE cfg4 grouped conv at its own shape: N=32, 14x14, 24 -> 48, groups 6, 3x3 pad 1,
    bias + ReLU, He-uniform weights, inputs U[0,1); every image bit for bit against the oracle."""
    g = np.random.default_rng(600 + st)
    N, H, W, Cin, Cout, gr = 32, 14, 14, 24, 48, 6
    x = g.uniform(0, 1, (N, H, W, Cin)).astype(np.float32)
    fan = 9 * (Cin // gr)
    w = g.uniform(-np.sqrt(6 / fan), np.sqrt(6 / fan), (gr, fan, Cout // gr)).astype(np.float32)
    b = g.uniform(-0.1, 0.1, Cout).astype(np.float32)
    got = acf.conv2d(x, w, b, 3, 3, Cout, st, 1, 1, groups=gr)
    ref = np.empty_like(got)
    orc.oracle().orc_conv2d(x, N, H, W, Cin, w, b.ctypes.data, 3, 3, Cout, st, 1, gr, ref, 1)
    assert_bits_equal(got, ref, f"cfg4 grouped s{st}")


@pytest.mark.parametrize("name", ["conv_grp_s1", "conv_grp_s2", "conv_grp_narrow"])
def test_grouped_golden(acf, name):
    d = load(name)
    N, H, W, Cin, KH, KW, Cout, st, pd, act, gr = (int(v) for v in d["shape"])
    got = acf.conv2d(d["x"], np.ascontiguousarray(d["w"]), d["b"], KH, KW, Cout, st, pd, act, groups=gr)
    assert_bits_equal(got, d["out"], name)


@pytest.mark.parametrize("st", [1, 2])
def test_grouped_cout16_vs_oracle(acf, orc, st):
    """Cout/g = 16 (the 16-accumulator grouped kernel) against the oracle's restatement."""
    g = np.random.default_rng(16 + st)
    N, H, W, Cin, Cout, gr = 2, 9, 11, 12, 48, 3
    x = g.uniform(-1, 1, (N, H, W, Cin)).astype(np.float32)
    w = g.uniform(-0.5, 0.5, (gr, 9 * (Cin // gr), Cout // gr)).astype(np.float32)
    b = g.uniform(-0.1, 0.1, Cout).astype(np.float32)
    got = acf.conv2d(x, w, b, 3, 3, Cout, st, 1, 1, groups=gr)
    ref = np.empty_like(got)
    orc.oracle().orc_conv2d(x, N, H, W, Cin, w, b.ctypes.data, 3, 3, Cout, st, 1, gr, ref, 1)
    assert max_rel(got, ref) < TOL_F32
