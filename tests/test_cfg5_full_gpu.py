"""GPU parity at the end-to-end model configuration itself: the VGG-11 ACFUN0 net at 224x224,
full width, batch 256 -- the workload the benchmark times -- so the paths that only run at
this size are covered: conv1's tensor-core route in L2-sized image chunks, the 16/8/4/2-wide
row-pair pooled tiles at 112/56/28/14 pooled widths, FC1 at K = 25088 inside the model and
the int8 mode's per-image activation scales across a 256-image batch.

Checked images: 0, 1, 254 and 255 of the batch (the first and the last tiles of every
persistent-kernel walk), against the reference library's own acfun_model_infer
(src/model.cpp:274-349 of hit-droid/Acfun, built from its sources into oracle/_ref) and, for
the int8 mode, against the reference's int8 layer composition (acfun_quantize_weights +
acfun_conv2d_int8 per conv, src/conv_int8.cpp:24-148).  When the reference library is absent
the C oracle (pinned to the reference's outputs) stands in.
"""
import os

import numpy as np
import pytest

from helpers import TOL_F32, assert_bits_equal, max_rel

pytestmark = pytest.mark.gpu

BATCH = 256
CHECK = (0, 1, 254, 255)
FC_RECORDS = 6          # fc, relu, fc, relu, fc, softmax at the end of acfun0.vgg11()


@pytest.fixture(scope="module")
def vgg(tmp_path_factory):
    """The benchmark's cfg5 net (acfun0.vgg11(seed=5)) and its conv stack alone (the same
    records without the FC head: output = the last pooled conv tensor, 7x7x512)."""
    from acfun_b200 import acfun0
    d = tmp_path_factory.mktemp("cfg5")
    full = acfun0.vgg11(seed=5)
    pf = str(d / "vgg11.acfun")
    full.save(pf)
    full.records = full.records[:-FC_RECORDS]
    ps = str(d / "vgg11_convs.acfun")
    full.save(ps)
    x = np.random.default_rng(2024).uniform(0, 1, (BATCH, 224, 224, 3)).astype(np.float32)
    return pf, ps, x


def _ref_model_infer(path, imgs):
    """acfun_model_infer of the reference library (or the C oracle's executor) per image."""
    from oracle import pyoracle as P
    if P.ref_available():
        R = P.ref()
        P.ref_set_threads(os.cpu_count() or 1)
        h = R.acfun_model_load(path.encode())
        assert h
        n = R.acfun_model_output_size(h)
        outs = []
        for x in imgs:
            o = np.empty(max(n, 1 << 20) if n <= 0 else n, np.float32)
            k = R.acfun_model_infer(h, np.ascontiguousarray(x), o)
            assert k > 0
            outs.append(o[:k].copy())
        R.acfun_model_destroy(h)
        return outs
    from oracle.model_oracle import OracleModel
    om = OracleModel(open(path, "rb").read())
    return [om.infer(x) for x in imgs]


def _ref_int8_infer(path, imgs):
    """The reference's int8 composition over the fused layer list (reference library when
    built, else the C oracle's restatement of the same calls)."""
    from oracle import pyoracle as P
    from oracle.model_oracle import OracleModel
    om = OracleModel(open(path, "rb").read())
    if P.ref_available():
        R = P.ref()
        P.ref_set_threads(os.cpu_count() or 1)
        return [om.ref_infer(R, x, int8=True) for x in imgs]
    return [om.infer(x, int8=True) for x in imgs]


@pytest.mark.parametrize("which", ["full", "convs"])
def test_cfg5_vgg11_fp32_batch256_vs_reference(acf, vgg, which):
    pf, ps, x = vgg
    path = pf if which == "full" else ps
    m = acf.Model(path)
    y = m.infer_batch(x)
    m.close()
    assert np.isfinite(y).all()
    refs = _ref_model_infer(path, [x[k] for k in CHECK])
    for k, r in zip(CHECK, refs):
        got = y[k].reshape(-1)
        assert got.shape == r.shape, (k, got.shape, r.shape)
        assert max_rel(got, r) < TOL_F32, (which, k, max_rel(got, r))
    if which == "full":
        assert np.allclose(y.sum(axis=1), 1.0, atol=1e-4)     # softmax rows


@pytest.mark.parametrize("which", ["full", "convs"])
def test_cfg5_vgg11_int8_batch256_vs_reference(acf, vgg, which):
    """int8 mode over the whole batch: the conv stack bit for bit (every conv output of these
    images is an exact function of its per-image scale), the softmax output within 1e-4."""
    pf, ps, x0 = vgg
    x = x0.copy()
    x[1] *= 0.25                   # per-image activation ranges differ across the batch
    x[254] *= 3.0
    x[255] = 0.5 - x[255]
    path = pf if which == "full" else ps
    m = acf.Model(path)
    m.set_int8(True)
    y = m.infer_batch(x)
    m.close()
    refs = _ref_int8_infer(path, [x[k] for k in CHECK])
    for k, r in zip(CHECK, refs):
        got = y[k].reshape(-1)
        if which == "convs":
            assert_bits_equal(got, r.reshape(-1), f"int8 conv stack, image {k}")
        else:
            assert max_rel(got, r) < TOL_F32, (k, max_rel(got, r))
