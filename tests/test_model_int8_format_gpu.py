"""GPU: the int8 ACFUN0 record (ConvInt8, type 8 -- an extension of this library; the reference's
int8 path has no model format).  acfun0.quantize_model() stores every dense conv as BN-folded,
quantised weights; loading that file must give the same bits as acfun_model_set_int8 on the
fp32 file (which quantises the same folded weights at run time), and a stored activation range
must give what a measured range of the same value gives."""
import numpy as np
import pytest

from helpers import assert_bits_equal

pytestmark = pytest.mark.gpu


def _run(acf, tmp_path, name, blob, x, int8_mode=False):
    p = tmp_path / name
    p.write_bytes(blob)
    m = acf.Model(str(p))
    if int8_mode:
        m.set_int8(True)
    y = m.infer_batch(x)
    m.close()
    return y


@pytest.mark.parametrize("width_div,head", [(4, True), (2, False)])
def test_saved_int8_model_equals_set_int8(acf, tmp_path, width_div, head):
    """VGG-11 shape at 64x64 (conv1 through the fused small-K int8 conv + pool, the rest through
    the Winograd route with pooled epilogues), with and without the FC / softmax head."""
    from acfun_b200 import acfun0
    W = acfun0.vgg11(seed=3, in_hw=64, width_div=width_div, fc_dims=(128, 64, 10))
    if not head:
        W.records = W.records[:-6]
    blob = W.tobytes()
    blob8 = acfun0.quantize_model(blob)
    assert len(blob8) < len(blob)
    g = np.random.default_rng(77)
    x = g.uniform(0, 1, (4, 64, 64, 3)).astype(np.float32)
    x[1] *= 5.0
    x[3] -= 0.5
    y_mode = _run(acf, tmp_path, "f.acfun", blob, x, int8_mode=True)
    y_file = _run(acf, tmp_path, "q.acfun", blob8, x)
    assert_bits_equal(y_file, y_mode, "int8 file vs set_int8")


@pytest.mark.parametrize("pool", [True, False])
def test_stored_activation_range_equals_measured(acf, tmp_path, pool):
    """act_max > 0: every image's max|x| is the stored value.  Images whose measured maximum is
    exactly that value give identical bits either way (pool: the fused small-K conv + pool
    kernel; otherwise the general int8 router)."""
    from acfun_b200 import acfun0
    from acfun_b200.acfun0 import Acfun0Writer, bn_params
    g = np.random.default_rng(5)
    u = lambda *s: g.uniform(-0.3, 0.3, size=s).astype(np.float32)
    Wr = Acfun0Writer(3, 33, 30)
    Wr.conv(u(27, 32), u(32), 3, 3, 32, 1, 1).bn(*bn_params(g, 32)).relu()
    if pool:
        Wr.maxpool(2, 2, 0)
    Wr.conv(u(9 * 32, 80), u(80), 3, 3, 80, 1, 1).relu()
    blob = Wr.tobytes()
    x = g.uniform(-1, 1, (3, 33, 30, 3)).astype(np.float32)
    x[:, 4, 5, 1] = 1.0            # every image: max|x| = 1 exactly
    dyn = _run(acf, tmp_path, "d.acfun", acfun0.quantize_model(blob), x)
    # the second conv's input range is measured (0); the first is stored as 1.0
    stat = _run(acf, tmp_path, "s.acfun", acfun0.quantize_model(blob, act_max=[1.0, 0.0]), x)
    assert_bits_equal(stat, dyn, "stored range 1.0 vs measured 1.0")
    # a stored range wider than the data quantises more coarsely: a different, finite result
    wide = _run(acf, tmp_path, "w.acfun", acfun0.quantize_model(blob, act_max=[4.0, 0.0]), x)
    assert np.isfinite(wide).all() and not np.array_equal(wide, dyn)


def test_int8_record_rejects_malformed(acf, tmp_path):
    from acfun_b200.acfun0 import Acfun0Writer
    L = acf.lib()
    Wr = Acfun0Writer(4, 8, 8)
    Wr.conv_int8(np.ones((36, 8), np.int8), np.ones(8, np.float32), np.zeros(8, np.float32), 3, 3, 8)
    blob = bytearray(Wr.tobytes())
    p = tmp_path / "t.acfun"
    p.write_bytes(bytes(blob[:-8]))                      # truncated wq
    assert not L.acfun_model_load(str(p).encode())
    assert L.acfun_last_error_code() == 5
    L.acfun_clear_error()
    neg = bytearray(blob)
    neg[26 + 24:26 + 28] = np.float32(-1.0).tobytes()     # negative act_max
    p.write_bytes(bytes(neg))
    assert not L.acfun_model_load(str(p).encode())
    L.acfun_clear_error()
