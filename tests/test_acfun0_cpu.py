"""CPU: the ACFUN0 int8 converter (acfun0.quantize_model) -- its BN fold equals the loader's
(restated by the oracle's orc_fold_bn, model.cpp:69-95) bit for bit, its weights equal the
library's acfun_quantize_weights of those folded weights, and the records parse back."""
import struct

import numpy as np


def test_fold_bn_matches_the_oracle_fold(orc):
    from acfun_b200.acfun0 import bn_params, fold_bn
    g = np.random.default_rng(3)
    K, Cout = 27, 16
    w = g.uniform(-0.5, 0.5, (K, Cout)).astype(np.float32)
    b = g.uniform(-0.1, 0.1, Cout).astype(np.float32)
    stats = bn_params(g, Cout)
    w2, b2 = fold_bn(w.reshape(-1), b, Cout, stats)
    wo, bo = w.reshape(-1).copy(), b.copy()
    mean, var, gamma, beta = (np.ascontiguousarray(s) for s in stats)
    orc.oracle().orc_fold_bn(wo, bo, wo.size, Cout, 0, mean, var, gamma, beta)
    assert np.array_equal(w2.view(np.int32), wo.view(np.int32))
    assert np.array_equal(b2.view(np.int32), bo.view(np.int32))


def test_quantize_model_records():
    import acfun_b200
    from acfun_b200 import acfun0
    W = acfun0.vgg11(seed=3, in_hw=32, width_div=16, fc_dims=(32, 16, 10))
    blob = W.tobytes()
    q = acfun0.quantize_model(blob, act_max=[0.0] * 7 + [2.5])
    assert q[:6] == b"ACFUN0"
    _, inC, inH, inW, num = struct.unpack_from("<5I", q, 6)
    assert (inC, inH, inW) == (3, 32, 32)
    off, prevC, types, convs = 26, 3, [], []
    for _ in range(num):
        t = struct.unpack_from("<I", q, off)[0]
        types.append(t)
        off += 4
        if t == 8:
            KH, KW, Cout, st, pd = struct.unpack_from("<5I", q, off)
            am = struct.unpack_from("<f", q, off + 20)[0]
            off += 24
            ws = np.frombuffer(q, "<f4", Cout, off)
            b = np.frombuffer(q, "<f4", Cout, off + 4 * Cout)
            off += 8 * Cout
            n = KH * KW * prevC * Cout
            wq = np.frombuffer(q, np.int8, n, off).reshape(-1, Cout)
            off += (n + 3) // 4 * 4
            convs.append((prevC, Cout, am, ws.copy(), b.copy(), wq.copy()))
            prevC = Cout
        elif t == 2:
            Cout, inDim = struct.unpack_from("<2I", q, off)
            off += 8 + 4 * (inDim * Cout + Cout)
        elif t == 4:
            off += 12
    assert off == len(q)
    assert types.count(8) == 8 and 1 not in types and 6 not in types     # BNs folded away
    assert [c[2] for c in convs] == [0.0] * 7 + [2.5]
    # the first conv: folded with its BN, quantised by the library's acfun_quantize_weights
    _, _, _, recs = acfun0._parse_records(blob)
    w2, b2 = acfun0.fold_bn(recs[0]["w"], recs[0]["b"], recs[0]["Cout"], recs[1]["stats"])
    ws, wq = acfun_b200.quantize_weights(w2.reshape(-1, recs[0]["Cout"]))
    assert np.array_equal(convs[0][3], ws) and np.array_equal(convs[0][5], wq)
    assert np.array_equal(convs[0][4].view(np.int32), b2.view(np.int32))
