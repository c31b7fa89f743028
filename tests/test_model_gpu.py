"""GPU parity: acfun_model_load / acfun_model_infer(_batch) over ACFUN0 against the
reference's golden outputs and the oracle executor."""
import os

import numpy as np
import pytest

from helpers import TOL_F32, assert_bits_equal, max_rel

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def test_model_demo_golden(acf, tmp_path):
    d = dict(np.load(os.path.join(GOLD, "model_demo.npz")))
    p = tmp_path / "demo.acfun"
    p.write_bytes(d["blob"].tobytes())
    m = acf.Model(str(p))
    assert m.in_dims == (32, 32, 3)
    for k in range(d["x"].shape[0]):
        y = m.infer(np.ascontiguousarray(d["x"][k]))
        assert y.shape == d["out"][k].shape
        assert max_rel(y, d["out"][k]) < TOL_F32
    yb = m.infer_batch(np.ascontiguousarray(d["x"]))
    assert max_rel(yb, d["out"]) < TOL_F32
    m.close()


# 4: conv1 has 16 channels -> fused conv + pool; 2: conv2..conv8 run their max-pool in the
# GEMM epilogue (row-pair tiles 32, 16, 8 and 4 columns wide)
@pytest.mark.parametrize("width_div", [8, 4, 2])
def test_model_vgg_small_vs_oracle(acf, tmp_path, width_div):
    from acfun_b200 import acfun0
    from oracle.model_oracle import OracleModel
    blob = acfun0.vgg11(seed=3, in_hw=64, width_div=width_div, fc_dims=(128, 64, 10)).tobytes()
    p = tmp_path / "v.acfun"
    p.write_bytes(blob)
    m = acf.Model(str(p))
    x = np.random.default_rng(4).uniform(0, 1, (3, 64, 64, 3)).astype(np.float32)
    y = m.infer_batch(x)
    om = OracleModel(blob)
    for k in range(3):
        assert max_rel(y[k], om.infer(x[k])) < TOL_F32


def test_model_device_pointers(acf, tmp_path):
    import torch
    d = dict(np.load(os.path.join(GOLD, "model_demo.npz")))
    p = tmp_path / "demo.acfun"
    p.write_bytes(d["blob"].tobytes())
    m = acf.Model(str(p))
    x = torch.from_numpy(np.ascontiguousarray(d["x"])).cuda()
    out = torch.empty((2, 10), device="cuda")
    m.infer_batch(x, out)
    acf.synchronize()
    assert max_rel(out.cpu().numpy(), d["out"]) < TOL_F32


@pytest.mark.parametrize("mutate", ["truncate", "magic", "type", "dims"])
def test_model_load_rejects_corrupt_files(acf, tmp_path, mutate):
    from acfun_b200 import acfun0
    blob = bytearray(acfun0.demo_net(seed=1).tobytes())
    if mutate == "truncate":
        blob = blob[: len(blob) // 2]
    elif mutate == "magic":
        blob[0:6] = b"ACFUN9"
    elif mutate == "type":
        blob[26:30] = (99).to_bytes(4, "little")
    elif mutate == "dims":
        blob[10:14] = (0).to_bytes(4, "little")
    p = tmp_path / "bad.acfun"
    p.write_bytes(bytes(blob))
    L = acf.lib()
    assert not L.acfun_model_load(str(p).encode())
    assert L.acfun_last_error_code() == 5
    L.acfun_clear_error()
    assert L.acfun_model_infer(None, None, None) == 0


def test_model_conv_pool_fusion_vs_oracle(acf, tmp_path):
    """Conv -> MaxPool pairs that run fused (small-K conv, 2x2/2 pool): odd spatial sizes
    (ragged pool edge, image borders), a strided 1x1 conv, a pool with post-ReLU."""
    from acfun_b200.acfun0 import Acfun0Writer, bn_params
    from oracle.model_oracle import OracleModel
    g = np.random.default_rng(11)
    u = lambda *s: g.uniform(-0.3, 0.3, size=s).astype(np.float32)
    Wr = Acfun0Writer(3, 37, 29)
    Wr.conv(u(27, 16), u(16), 3, 3, 16, 1, 1).bn(*bn_params(g, 16)).relu().maxpool(2, 2, 0)   # 18x14
    Wr.conv(u(16, 32), u(32), 1, 1, 32, 2, 0).maxpool(2, 2, 0).relu()                          # 9x7 -> 4x3
    Wr.fc(u(4 * 3 * 32, 10), u(10), 4 * 3 * 32, 10).softmax()
    blob = Wr.tobytes()
    p = tmp_path / "cp.acfun"
    p.write_bytes(blob)
    m = acf.Model(str(p))
    x = np.random.default_rng(12).uniform(-1, 1, (5, 37, 29, 3)).astype(np.float32)
    y = m.infer_batch(x)
    om = OracleModel(blob)
    for k in range(5):
        assert max_rel(y[k], om.infer(x[k])) < TOL_F32
    m.close()


@pytest.mark.parametrize("width_div", [8, 4, 2])   # 2: pooled int8 GEMM epilogues (Cout > 64)
def test_model_int8_mode_vs_oracle(acf, tmp_path, width_div):
    """acfun_model_set_int8: every dense conv through the int8 router with one activation scale
    per image (conv1: u8 im2col route, the rest: int8 Winograd route), FC / pool / softmax fp32.
    Against the oracle's per-image composition (quantize_weights + conv2d_int8 per layer), and
    a batch must give each image exactly what a single-image call gives."""
    from acfun_b200 import acfun0
    from oracle.model_oracle import OracleModel
    blob = acfun0.vgg11(seed=3, in_hw=64, width_div=width_div, fc_dims=(128, 64, 10)).tobytes()
    p = tmp_path / "v8.acfun"
    p.write_bytes(blob)
    m = acf.Model(str(p))
    m.set_int8(True)
    g = np.random.default_rng(41)
    x = g.uniform(0, 1, (3, 64, 64, 3)).astype(np.float32)
    x[1] *= 7.0                     # images with different activation ranges
    x[2] -= 0.5
    y = m.infer_batch(x)
    om = OracleModel(blob)
    for k in range(3):
        assert max_rel(y[k], om.infer(x[k], int8=True)) < TOL_F32
        assert_bits_equal(m.infer_batch(np.ascontiguousarray(x[k:k + 1]))[0], y[k], f"image {k} alone")
    m.set_int8(False)
    assert max_rel(m.infer_batch(x)[0], om.infer(x[0])) < TOL_F32
    m.close()


@pytest.mark.parametrize("st,post_relu,cin,relu", [(1, False, 3, True), (2, True, 3, True),
                                                  (1, True, 7, True), (1, False, 3, False)])
def test_model_int8_conv_pool_fusion_bit_exact(acf, tmp_path, st, post_relu, cin, relu):
    """int8 mode, Conv -> MaxPool(2,2,0) with nothing after it: the fused small-K int8 conv +
    pool kernel must equal the oracle's conv2d_int8 + maxpool bit for bit (odd sizes, borders,
    per-image scales, an all-zero image)."""
    from acfun_b200.acfun0 import Acfun0Writer, bn_params
    from oracle.model_oracle import OracleModel
    g = np.random.default_rng(100 + st + cin)
    u = lambda *s: g.uniform(-0.3, 0.3, size=s).astype(np.float32)
    Wr = Acfun0Writer(cin, 37, 29)
    Wr.conv(u(9 * cin, 32), u(32), 3, 3, 32, st, 1).bn(*bn_params(g, 32))
    if relu:
        Wr.relu()
    Wr.maxpool(2, 2, 0)
    if post_relu:
        Wr.relu()
    blob = Wr.tobytes()
    p = tmp_path / "cp8.acfun"
    p.write_bytes(blob)
    m = acf.Model(str(p))
    m.set_int8(True)
    x = np.random.default_rng(7).uniform(-1, 1, (4, 37, 29, cin)).astype(np.float32)
    x[1] *= 50.0
    x[3] = 0.0                       # max|x| < 1e-12: the conv writes zeros
    y = m.infer_batch(x)
    om = OracleModel(blob)
    for k in range(4):
        assert_bits_equal(y[k], om.infer(x[k], int8=True), f"image {k}")
    m.close()


@pytest.mark.parametrize("cin,k,cout,hw,relu", [(3, 3, 64, (70, 100), True), (3, 3, 48, (33, 65), False),
                                               (4, 2, 16, (18, 40), True), (1, 3, 32, (64, 64), True)])
def test_model_int8_conv_pool_tensor_route_bit_exact(acf, tmp_path, cin, k, cout, hw, relu):
    """int8 mode, small-K stride-1 Conv -> MaxPool(2,2,0) on the tensor-core kernel (K =
    k*k*cin <= 32, tiles of 2 x 16 pooled pixels: ragged last tiles in both directions, several
    tiles per image, Cout 16..64), bit for bit against the oracle, with the per-image maxima the
    next int8 layer would use checked through a second conv."""
    from acfun_b200.acfun0 import Acfun0Writer, bn_params
    from oracle.model_oracle import OracleModel
    g = np.random.default_rng(cin * 100 + k * 10 + cout)
    H, W = hw
    Wr = Acfun0Writer(cin, H, W)
    Wr.conv(g.uniform(-0.3, 0.3, (k * k * cin, cout)).astype(np.float32),
            g.uniform(-0.1, 0.1, cout).astype(np.float32), k, k, cout, 1, 1).bn(*bn_params(g, cout))
    if relu:
        Wr.relu()
    Wr.maxpool(2, 2, 0)
    Wr.conv(g.uniform(-0.1, 0.1, (9 * cout, 24)).astype(np.float32), np.zeros(24, np.float32),
            3, 3, 24, 1, 1)
    blob = Wr.tobytes()
    p = tmp_path / "cp8tc.acfun"
    p.write_bytes(blob)
    m = acf.Model(str(p))
    m.set_int8(True)
    x = np.random.default_rng(11).uniform(-1, 1, (3, H, W, cin)).astype(np.float32)
    x[1] *= 40.0
    y = m.infer_batch(x)
    om = OracleModel(blob)
    for i in range(3):
        assert_bits_equal(y[i], om.infer(x[i], int8=True), f"image {i}")
    m.close()


def test_model_int8_conv_pool_tensor_route_exact_slow_channel(acf, tmp_path):
    """A channel with all-zero weights and zero bias (alpha = 0, beta = 0, no ReLU) sends every
    tile of the tensor-core conv + pool kernel through its exact per-pixel path; bit for bit."""
    from acfun_b200.acfun0 import Acfun0Writer
    from oracle.model_oracle import OracleModel
    g = np.random.default_rng(77)
    w = g.uniform(-0.3, 0.3, (27, 64)).astype(np.float32)
    b = g.uniform(-0.1, 0.1, 64).astype(np.float32)
    w[:, 5] = 0.0
    b[5] = 0.0
    Wr = Acfun0Writer(3, 30, 50)
    Wr.conv(w, b, 3, 3, 64, 1, 1)
    Wr.maxpool(2, 2, 0)
    blob = Wr.tobytes()
    p = tmp_path / "cp8slow.acfun"
    p.write_bytes(blob)
    m = acf.Model(str(p))
    m.set_int8(True)
    x = np.random.default_rng(12).uniform(-1, 1, (2, 30, 50, 3)).astype(np.float32)
    y = m.infer_batch(x)
    om = OracleModel(blob)
    for i in range(2):
        assert_bits_equal(y[i], om.infer(x[i], int8=True), f"image {i}")
    m.close()


@pytest.mark.parametrize("hw", [(224, 224), (37, 29)])
def test_fused_conv1_pool_bit_exact_vs_separate_calls(acf, tmp_path, hw):
    """The fused CUDA-core 3x3 / Cin 3 conv + 2x2 pool kernel (packed f32x2 FMAs; the route
    in 3xTF32 mode, where the tensor-core conv + pool route is off) against acfun_conv2d
    (CUDA-core route, scalar fma chain) followed by acfun_maxpool: identical bits."""
    from acfun_b200.acfun0 import Acfun0Writer
    H, W = hw
    g = np.random.default_rng(H)
    w = g.uniform(-0.5, 0.5, (27, 64)).astype(np.float32)
    b = g.uniform(-0.1, 0.1, 64).astype(np.float32)
    Wr = Acfun0Writer(3, H, W)
    Wr.conv(w, b, 3, 3, 64, 1, 1).maxpool(2, 2, 0)
    p = tmp_path / "c1.acfun"
    p.write_bytes(Wr.tobytes())
    L = acf.lib()
    assert L.acfun_set_fp32_math(1) == 0
    try:
        m = acf.Model(str(p))
        x = g.uniform(-1, 1, (2, H, W, 3)).astype(np.float32)
        y = m.infer_batch(x)
        ref = acf.maxpool(acf.conv2d(x, w, b, 3, 3, 64, 1, 1, 0), 2, 2, 0)
        assert_bits_equal(y, ref.reshape(y.shape), "fused conv1 + pool")
        m.close()
    finally:
        L.acfun_set_fp32_math(0)


@pytest.mark.parametrize("hw,nxt", [((224, 224), False), ((224, 224), True), ((223, 221), True)])
def test_conv1_pool_tensor_route_vs_oracle(acf, tmp_path, hw, nxt):
    """Conv (K = 27) + 2x2 pool on the tensor cores: pooled-order im2col and a 3xBF16 GEMM
    that pools in its epilogue, writing fp32 or (nxt) the next conv's split input; odd sizes
    drop the last row / column like the pool."""
    from acfun_b200.acfun0 import Acfun0Writer
    from oracle.model_oracle import OracleModel
    H, W = hw
    g = np.random.default_rng(H + W + nxt)
    u = lambda *s: g.uniform(-0.5, 0.5, size=s).astype(np.float32)
    Wr = Acfun0Writer(3, H, W)
    Wr.conv(u(27, 64), u(64), 3, 3, 64, 1, 1).relu().maxpool(2, 2, 0)
    if nxt:
        Wr.conv(u(576, 64) * 0.2, u(64), 3, 3, 64, 1, 1).relu()
    blob = Wr.tobytes()
    p = tmp_path / "c1t.acfun"
    p.write_bytes(blob)
    m = acf.Model(str(p))
    x = g.uniform(0, 1, (2, H, W, 3)).astype(np.float32)
    y = m.infer_batch(x)
    om = OracleModel(blob)
    for k in range(2):
        assert max_rel(y[k], om.infer(x[k]).reshape(y[k].shape)) < TOL_F32
    m.close()


@pytest.mark.parametrize("hw,cin,c2,k2,nimg", [((112, 112), 64, 128, 3, 2),  # 128- then 64-wide
                                               ((56, 58), 64, 192, 1, 2),    # 1x1; 64 then 32, odd
                                               ((30, 29), 64, 128, 3, 3),    # 32-wide, odd OW
                                               ((14, 14), 128, 128, 3, 3)])  # 16-wide
def test_model_pooled_conv_vs_oracle(acf, tmp_path, hw, cin, c2, k2, nimg):
    """Conv -> MaxPool(2, 2, 0) as one implicit GEMM with row-pair tiles (the pool in the
    epilogue), fp32 (3xBF16; the pooled output written as the next conv's split input and as
    fp32) and int8 (Winograd and 1x1 routes, per-image scales; bit-exact) against the oracle."""
    from acfun_b200.acfun0 import Acfun0Writer, bn_params
    from oracle.model_oracle import OracleModel
    H, W = hw
    g = np.random.default_rng(H * 7 + c2)
    u = lambda s, *d: g.uniform(-s, s, size=d).astype(np.float32)
    Wr = Acfun0Writer(cin, H, W)
    Wr.conv(u(0.1, k2 * k2 * cin, c2), u(0.1, c2), k2, k2, c2, 1, k2 // 2).bn(*bn_params(g, c2)).relu()
    Wr.maxpool(2, 2, 0)
    Wr.conv(u(0.05, 9 * c2, 128), u(0.1, 128), 3, 3, 128, 1, 1).relu().maxpool(2, 2, 0).relu()
    blob = Wr.tobytes()
    p = tmp_path / "pc.acfun"
    p.write_bytes(blob)
    m = acf.Model(str(p))
    x = np.random.default_rng(5).uniform(0, 1, (nimg, H, W, cin)).astype(np.float32)
    x[-1] *= 9.0
    om = OracleModel(blob)
    y = m.infer_batch(x)
    for k in range(nimg):
        assert max_rel(y[k], om.infer(x[k]).reshape(y[k].shape)) < TOL_F32, k
    m.set_int8(True)
    y8 = m.infer_batch(x)
    for k in range(nimg):
        assert_bits_equal(y8[k], om.infer(x[k], int8=True).reshape(y8[k].shape), f"int8 image {k}")
    assert_bits_equal(m.infer_batch(np.ascontiguousarray(x[-1:]))[0], y8[-1], "int8 last image alone")
    m.close()


def test_parity_strict_off_corrects_the_loader_quirks(acf, tmp_path, monkeypatch):
    """ACFUN_PARITY_STRICT=0: a ReLU before MaxPool is kept (the reference drops it), and
    Conv -> ReLU -> BN applies BN after the activation (the reference folds BN into the conv)."""
    from acfun_b200.acfun0 import Acfun0Writer, bn_params
    g = np.random.default_rng(21)
    w = g.uniform(-0.3, 0.3, (36, 8)).astype(np.float32)
    b = np.where(np.arange(8) % 2 == 0, -10.0, 0.2).astype(np.float32)  # all-negative channels
    x = g.uniform(0, 1, (2, 10, 10, 4)).astype(np.float32)

    def run(Wr, name):
        p = tmp_path / name
        p.write_bytes(Wr.tobytes())
        m = acf.Model(str(p))
        y = m.infer_batch(x)
        m.close()
        return y

    pool_model = lambda: Acfun0Writer(4, 10, 10).conv(w, b, 3, 3, 8, 1, 1).relu().maxpool(2, 2, 0)
    y_strict = run(pool_model(), "a.acfun")
    assert (y_strict < 0).any()                       # the dropped ReLU: pooled negatives
    monkeypatch.setenv("ACFUN_PARITY_STRICT", "0")
    y_fixed = run(pool_model(), "b.acfun")
    assert_bits_equal(y_fixed, np.maximum(y_strict, 0.0), "ReLU kept before MaxPool")

    mean, var, gamma, beta = bn_params(g, 8)
    y_bn = run(Acfun0Writer(4, 10, 10).conv(w, b, 3, 3, 8, 1, 1).relu().bn(mean, var, gamma, beta),
               "c.acfun")
    conv = acf.conv2d(x, w, b, 3, 3, 8, 1, 1, 1).reshape(2, 10, 10, 8)   # ReLU'd conv
    ref = ((conv - mean) / np.sqrt(var + 1e-5) * gamma + beta).reshape(y_bn.shape)  # then BN
    assert max_rel(y_bn, ref) < TOL_F32, max_rel(y_bn, ref)
