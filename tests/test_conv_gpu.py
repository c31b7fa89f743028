"""GPU parity: fp32 conv routes (tolerance) and int8 conv routes (bit-exact) through the
C ABI, against the reference's golden vectors and the oracle, plus BASELINE-size cases."""
import glob
import os
import zlib

import numpy as np
import pytest

from helpers import TOL_F32, assert_bits_equal, max_rel

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def load(name):
    return dict(np.load(os.path.join(GOLD, name + ".npz")))


def gnames(prefix):
    return sorted(os.path.basename(p)[:-4] for p in glob.glob(os.path.join(GOLD, prefix + "*.npz")))


@pytest.mark.parametrize("name", gnames("conv_f32_") + ["conv_grp_split"])
def test_conv_f32_golden(acf, name):
    d = load(name)
    N, H, W, Cin, KH, KW, Cout, st, pd, act, groups = (int(v) for v in d["shape"])
    w = np.ascontiguousarray(d["w"])
    if name == "conv_f32_wino43":  # internal entry point of the F(4,3) route
        got = np.empty_like(d["out"])
        acf.lib().acfun_winograd43_conv3x3(acf.ptr(d["x"]), N, H, W, Cin, acf.ptr(w), acf.ptr(d["b"]), Cout,
                                           acf.ptr(got), act)
        acf.check()
    else:
        got = acf.conv2d(d["x"], w, d["b"], KH, KW, Cout, st, pd, act, groups=groups)
    assert max_rel(got, d["out"]) < TOL_F32, (name, max_rel(got, d["out"]))


def he(g, shape, fan_in):
    lim = np.sqrt(6.0 / fan_in)
    return g.uniform(-lim, lim, size=shape).astype(np.float32)


@pytest.mark.parametrize("cfg", [
    ("cfg3a_f23", 32, 56, 56, 64, 3, 3, 64, 1, 1),       # routed to F(2,3) in the reference
    ("cfg3b_f43", 8, 112, 112, 64, 3, 3, 64, 1, 1),      # routed to F(4,3)
    ("cfg4_pw_s1", 32, 56, 56, 144, 1, 1, 24, 1, 0),     # zero-copy 1x1
    ("cfg4_pw_s2", 32, 56, 56, 32, 1, 1, 64, 2, 0),      # strided 1x1 gather
    ("vgg_l1", 2, 224, 224, 3, 3, 3, 64, 1, 1),          # im2col route (Cin=3 < 4)
    ("odd", 3, 17, 23, 40, 3, 3, 72, 1, 1),
    ("k5s2", 2, 19, 21, 12, 5, 5, 20, 2, 2),
    ("pw_c40", 4, 20, 22, 72, 1, 1, 40, 1, 0),         # CUDA-core route, 48-wide accumulators
    # narrow stride-1 convs (<= 64 -> <= 64 channels): the split pass + resident-weight slab
    # kernel; channel counts off the vector width, pad 0, many images
    ("halo_c20_o24", 3, 15, 17, 20, 3, 3, 24, 1, 1),
    ("halo_c48_o40_p0", 2, 12, 11, 48, 3, 3, 40, 1, 0),
    ("halo_c16_o64", 5, 40, 37, 16, 3, 3, 64, 1, 1),
    ("halo_k1x5", 2, 9, 30, 40, 1, 5, 33, 1, 2),
    # 1x1 stride 1 over >= 148 * 128 pixels: the tensor-core pointwise kernel (ragged last tile,
    # a partial K block, 1..3 K blocks, Cout padded to 16 / 48 / 64)
    ("pwtc_c100_o40", 7, 57, 51, 100, 1, 1, 40, 1, 0),
    ("pwtc_c192_o64", 6, 60, 60, 192, 1, 1, 64, 1, 0),
    ("pwtc_c12_o8", 5, 66, 61, 12, 1, 1, 8, 1, 0),
])
def test_conv_f32_configs_vs_oracle(acf, orc, cfg):
    tag, N, H, W, Cin, KH, KW, Cout, st, pd = cfg
    g = np.random.default_rng(zlib.crc32(tag.encode()))
    x = g.uniform(0, 1, (N, H, W, Cin)).astype(np.float32)
    w = he(g, (KH * KW * Cin, Cout), KH * KW * Cin)
    b = g.uniform(-0.1, 0.1, Cout).astype(np.float32)
    got = acf.conv2d(x, w, b, KH, KW, Cout, st, pd, 1)
    # every image: a persistent kernel's last wave and ragged tiles cover the last images
    OH, OW = orc.conv_out_hw(H, W, KH, KW, st, pd)
    ref = np.empty((N, OH, OW, Cout), np.float32)
    orc.oracle().orc_conv2d(x, N, H, W, Cin, w, b.ctypes.data, KH, KW, Cout, st, pd, 1, ref, 1)
    for n in range(N):
        assert max_rel(got[n], ref[n]) < TOL_F32, (n, max_rel(got[n], ref[n]))
    assert np.isfinite(got).all()


@pytest.mark.parametrize("name", gnames("conv_int8_"))
def test_conv_int8_golden_exact(acf, name):
    d = load(name)
    N, H, W, Cin, KH, KW, Cout, st, pd, act = (int(v) for v in d["shape"])
    ws, wq = acf.quantize_weights(d["w"])
    assert_bits_equal(wq, d["wq"], "wq")
    assert_bits_equal(ws, d["ws"], "ws")
    got = acf.conv2d_int8(d["x"], wq, ws, d["b"], KH, KW, Cout, st, pd, act)
    assert_bits_equal(got, d["out"], name)


@pytest.mark.parametrize("cfg", [
    ("cfg3a_int8", 32, 56, 56, 64, 3, 3, 64, 1, 1, 1),    # Winograd-int8 route at BASELINE size
    ("wino_odd", 2, 13, 9, 48, 3, 3, 40, 1, 1, 1),
    ("direct_s2", 2, 30, 30, 3, 3, 3, 16, 2, 1, 1),
    ("pw", 2, 20, 20, 160, 1, 1, 48, 1, 0, 0),
    ("im2col_s2", 1, 21, 17, 48, 3, 3, 24, 2, 1, 1),
    ("direct_small_cin_s1", 2, 15, 15, 4, 3, 3, 8, 1, 1, 1),
    ("k5p2", 1, 14, 14, 36, 5, 5, 12, 1, 2, 0),
    # K-block / tile-width variants: 128-byte K blocks, 128- and 256-wide tiles
    ("c128_o160", 2, 12, 12, 128, 3, 3, 160, 1, 1, 1),
    ("c200_o300", 1, 10, 11, 200, 3, 3, 300, 1, 1, 0),
    ("im2col_k224_o70", 1, 9, 9, 24, 3, 3, 70, 2, 1, 1),
    ("wide_m_o200", 8, 40, 40, 64, 3, 3, 200, 1, 1, 1),
    # narrow stride-1 convs (<= 64 input, <= 128 output channels) through the resident-weight
    # kernel that stages one slab of input rows per tile: the Winograd route with tail
    # channels, the direct route (pad 0), 1x1 and 1x3, 128-wide tiles, slabs of three boxes
    # (wide rows), many images per tile, 25 resident taps
    ("h8_c20_tail", 2, 15, 17, 20, 3, 3, 24, 1, 1, 1),
    ("h8_pad0", 2, 12, 11, 48, 3, 3, 40, 1, 0, 1),
    ("h8_1x1", 2, 20, 20, 64, 1, 1, 48, 1, 0, 0),
    ("h8_k1x3", 2, 9, 30, 40, 1, 3, 33, 1, 0, 1),
    ("h8_o128", 2, 14, 13, 64, 3, 3, 128, 1, 1, 1),
    ("h8_o96_wide_rows", 1, 9, 100, 32, 3, 3, 96, 1, 1, 0),
    ("h8_many_images", 5, 7, 6, 16, 3, 3, 8, 1, 1, 1),
    ("h8_k5p2", 1, 20, 20, 16, 5, 5, 40, 1, 2, 1),
])
def test_conv_int8_vs_oracle_exact(acf, orc, cfg):
    tag, N, H, W, Cin, KH, KW, Cout, st, pd, act = cfg
    g = np.random.default_rng(zlib.crc32(tag.encode()))
    x = g.uniform(0, 1, (N, H, W, Cin)).astype(np.float32)
    x[..., ::7] -= 0.5
    w = he(g, (KH * KW * Cin, Cout), KH * KW * Cin)
    b = g.uniform(-0.1, 0.1, Cout).astype(np.float32)
    ws, wq = acf.quantize_weights(w)
    got = acf.conv2d_int8(x, wq, ws, b, KH, KW, Cout, st, pd, act)
    ref = orc.orc_conv2d_int8(x, wq, ws, b, N, H, W, Cin, KH, KW, Cout, st, pd, act)
    assert_bits_equal(got, ref, tag)


def test_conv_int8_all_zero_input(acf):
    x = np.zeros((1, 6, 6, 8), np.float32)
    g = np.random.default_rng(1)
    ws, wq = acf.quantize_weights(g.uniform(-1, 1, (72, 8)).astype(np.float32))
    b = np.full(8, 3.0, np.float32)
    got = acf.conv2d_int8(x, wq, ws, b, 3, 3, 8, 1, 1, 1)
    assert (got.view(np.int32) == 0).all()      # conv_int8.cpp:78 writes zeros, not the bias


def test_int8_internal_entry_points(acf, orc):
    """acfun_conv2d_int8_direct / acfun_conv1x1_int8 / acfun_winograd_conv3x3_int8 with
    caller-supplied scales, against the oracle's restatements."""
    g = np.random.default_rng(7)
    O, L = orc.oracle(), acf.lib()
    N, H, W, Cin, Cout = 2, 9, 10, 20, 12
    xq = g.integers(0, 256, (N, H, W, Cin), dtype=np.uint8)
    wq = g.integers(-128, 128, (9 * Cin, Cout), dtype=np.int8)
    al = g.uniform(1e-4, 1e-2, Cout).astype(np.float32)
    be = g.uniform(-3, 3, Cout).astype(np.float32)
    for st in (1, 2):
        OH, OW = orc.conv_out_hw(H, W, 3, 3, st, 1)
        ref = np.empty((N, OH, OW, Cout), np.float32)
        O.orc_conv2d_int8_direct(xq, N, H, W, Cin, wq, al, be, 3, 3, Cout, st, 1, OH, OW, ref, 1)
        got = np.empty_like(ref)
        L.acfun_conv2d_int8_direct(acf.ptr(xq), N, H, W, Cin, acf.ptr(wq), acf.ptr(al), acf.ptr(be), 3, 3,
                                   Cout, st, 1, OH, OW, acf.ptr(got), 1)
        acf.check()
        assert_bits_equal(got, ref, f"direct s{st}")
    A = g.integers(0, 256, (300, Cin), dtype=np.uint8)
    w1 = g.integers(-128, 128, (Cin, Cout), dtype=np.int8)
    ref = np.empty((300, Cout), np.float32)
    O.orc_gemm_int8_epi(300, Cout, Cin, A, w1, ref, al, be, 0)
    got = np.empty_like(ref)
    L.acfun_conv1x1_int8(acf.ptr(A), 300, Cin, Cout, acf.ptr(w1), acf.ptr(al), acf.ptr(be), acf.ptr(got), 0)
    acf.check()
    assert_bits_equal(got, ref, "conv1x1_int8")
    x = g.uniform(-1, 1, (N, H, W, Cin)).astype(np.float32)
    ws = g.uniform(1e-3, 1e-2, Cout).astype(np.float32)
    b = g.uniform(-1, 1, Cout).astype(np.float32)
    ref = np.empty((N, H, W, Cout), np.float32)
    O.orc_winograd_int8(x, N, H, W, Cin, wq, ws, b.ctypes.data, Cout, 0.0083, 120.5, ref, 1)
    got = np.empty_like(ref)
    L.acfun_winograd_conv3x3_int8(acf.ptr(x), N, H, W, Cin, acf.ptr(wq), acf.ptr(ws), acf.ptr(b), Cout,
                                  0.0083, 120.5, acf.ptr(got), 1)
    acf.check()
    assert_bits_equal(got, ref, "winograd_int8 internal")


def test_fc_golden(acf):
    d = load("fc")
    assert max_rel(acf.fc(d["x"], d["w"], d["b"], 0), d["out"]) < TOL_F32
    assert max_rel(acf.fc(d["x"], d["w"], d["b"], 1), d["out_relu"]) < TOL_F32


def test_conv_f32_last_wave_images(acf, orc):
    """8 x 56 x 56, 64 -> 128: 211 implicit-GEMM tiles on 148 persistent CTAs; the second,
    partial wave covers the last images, which are the ones checked here."""
    N, H, W, Cin, Cout = 8, 56, 56, 64, 128
    g = np.random.default_rng(211)
    x = g.uniform(-1, 1, (N, H, W, Cin)).astype(np.float32)
    w = he(g, (9 * Cin, Cout), 9 * Cin)
    b = g.uniform(-0.1, 0.1, Cout).astype(np.float32)
    got = acf.conv2d(x, w, b, 3, 3, Cout, 1, 1, 1)
    ref = np.empty((3, H, W, Cout), np.float32)
    orc.oracle().orc_conv2d(np.ascontiguousarray(x[N - 3:]), 3, H, W, Cin, w, b.ctypes.data, 3, 3, Cout, 1, 1,
                            1, ref, 1)
    assert max_rel(got[N - 3:], ref) < TOL_F32, max_rel(got[N - 3:], ref)


def test_conv_f32_wide_tiles_vs_oracle(acf, orc):
    """16 x 28 x 28, 96 -> 320: 226 implicit-GEMM tiles of 128 x 256 in 64-byte K blocks
    (Cin padded to 128, Cout ragged in the second column tile); first and last images."""
    N, H, W, Cin, Cout = 16, 28, 28, 96, 320
    g = np.random.default_rng(320)
    x = g.uniform(0, 1, (N, H, W, Cin)).astype(np.float32)
    w = he(g, (9 * Cin, Cout), 9 * Cin)
    b = g.uniform(-0.1, 0.1, Cout).astype(np.float32)
    got = acf.conv2d(x, w, b, 3, 3, Cout, 1, 1, 1)
    for sl in (slice(0, 2), slice(N - 2, N)):
        ref = np.empty((2, H, W, Cout), np.float32)
        orc.oracle().orc_conv2d(np.ascontiguousarray(x[sl]), 2, H, W, Cin, w, b.ctypes.data, 3, 3, Cout, 1,
                                1, 1, ref, 1)
        assert max_rel(got[sl], ref) < TOL_F32, max_rel(got[sl], ref)


@pytest.mark.parametrize("N,H,W,Cout", [(12, 56, 56, 96), (14, 50, 50, 48)])
def test_conv_f32_paired_subtiles_vs_oracle(acf, orc, N, H, W, Cout):
    """Implicit GEMMs with two 128-row sub-tiles per CTA sharing each weight stage (Cout 96
    on 128-column tiles, 48 on 64-column tiles); the last images sit in the second wave, and
    at 14 x 52 x 52 padded rows the last tile's second sub-tile is past the end."""
    Cin = 64
    g = np.random.default_rng(N * 1000 + Cout)
    x = g.uniform(0, 1, (N, H, W, Cin)).astype(np.float32)
    w = he(g, (9 * Cin, Cout), 9 * Cin)
    b = g.uniform(-0.1, 0.1, Cout).astype(np.float32)
    got = acf.conv2d(x, w, b, 3, 3, Cout, 1, 1, 1)
    for sl in (slice(0, 1), slice(N - 2, N)):
        n = sl.stop - sl.start
        ref = np.empty((n, H, W, Cout), np.float32)
        orc.oracle().orc_conv2d(np.ascontiguousarray(x[sl]), n, H, W, Cin, w, b.ctypes.data, 3, 3, Cout, 1,
                                1, 1, ref, 1)
        assert max_rel(got[sl], ref) < TOL_F32, max_rel(got[sl], ref)
