"""ACFUN0 model files: writer and the VGG-11 generator used by the end-to-end benchmark.

Format (little endian; reference src/model.cpp:1-21, encoder tools/gen_model.py:12-44):
    magic "ACFUN0" | u32 version | u32 inC, inH, inW | u32 num_layers | layer records
    1 Conv        u32 KH, KW, Cout, stride, pad | f32 w[KH*KW*Cin*Cout] | f32 b[Cout]
    2 FC          u32 Cout, inDim | f32 w[inDim*Cout] | f32 b[Cout]
    3 ReLU        (no payload)
    4 MaxPool     u32 pool, stride, pad
    5 Softmax     (no payload)
    6 BN          u32 ch | f32 mean[ch], var[ch], gamma[ch], beta[ch]
    7 ConvGrouped u32 KH, KW, Cout, stride, pad, groups | f32 w[...] | f32 b[Cout]
Conv weights are [KH*KW*Cin, Cout]; grouped weights [g][KH*KW*Cin_per][Cout_per]
(the layout the kernels read, group_conv.cpp:137-139); FC weights [inDim, Cout].

Extension of this library (the reference's int8 path has no model format; its loader
rejects the record):
    8 ConvInt8    u32 KH, KW, Cout, stride, pad | f32 act_max | f32 wscale[Cout] |
                  f32 b[Cout] | s8 wq[KH*KW*Cin*Cout] | zero bytes to a multiple of 4
an already quantised dense convolution (acfun_quantize_weights of the BN-folded weights,
conv_int8.cpp:24-37), run through the int8 router at load without re-quantising.
act_max = 0: one activation scale per image from that image's max|x| (the reference's
per-call definition, conv_int8.cpp:75-77); act_max > 0: a stored calibration range used as
every image's max|x|.  quantize_model() turns an fp32 file into this form.
"""
from __future__ import annotations

import struct

import numpy as np

MAGIC = b"ACFUN0"


class Acfun0Writer:
    def __init__(self, in_c: int, in_h: int, in_w: int, version: int = 1):
        self.in_dims = (in_c, in_h, in_w)
        self.version = version
        self.records: list[bytes] = []
        self.c = in_c

    @staticmethod
    def _u32(*v):
        return struct.pack("<" + "I" * len(v), *v)

    @staticmethod
    def _f32(a):
        return np.ascontiguousarray(a, dtype="<f4").tobytes()

    def conv(self, w, b, KH, KW, Cout, stride=1, pad=1):
        assert w.size == KH * KW * self.c * Cout and b.size == Cout
        self.records.append(self._u32(1, KH, KW, Cout, stride, pad) + self._f32(w) + self._f32(b))
        self.c = Cout
        return self

    def conv_g(self, w, b, KH, KW, Cout, groups, stride=1, pad=1):
        assert w.size == KH * KW * (self.c // groups) * Cout and b.size == Cout
        self.records.append(self._u32(7, KH, KW, Cout, stride, pad, groups) + self._f32(w) + self._f32(b))
        self.c = Cout
        return self

    def fc(self, w, b, in_dim, Cout):
        assert w.size == in_dim * Cout and b.size == Cout
        self.records.append(self._u32(2, Cout, in_dim) + self._f32(w) + self._f32(b))
        self.c = Cout
        return self

    def conv_int8(self, wq, wscale, b, KH, KW, Cout, stride=1, pad=1, act_max=0.0):
        """ConvInt8 record: wq [KH*KW*Cin, Cout] int8, wscale / b [Cout] fp32."""
        wq = np.ascontiguousarray(wq, dtype=np.int8)
        assert wq.size == KH * KW * self.c * Cout and wscale.size == Cout and b.size == Cout
        assert act_max >= 0.0
        raw = wq.tobytes()
        raw += b"\0" * (-len(raw) % 4)
        self.records.append(self._u32(8, KH, KW, Cout, stride, pad) + struct.pack("<f", act_max)
                            + self._f32(wscale) + self._f32(b) + raw)
        self.c = Cout
        return self

    def relu(self):
        self.records.append(self._u32(3))
        return self

    def maxpool(self, pool=2, stride=2, pad=0):
        self.records.append(self._u32(4, pool, stride, pad))
        return self

    def softmax(self):
        self.records.append(self._u32(5))
        return self

    def bn(self, mean, var, gamma, beta):
        ch = mean.size
        self.records.append(self._u32(6, ch) + self._f32(mean) + self._f32(var) + self._f32(gamma)
                            + self._f32(beta))
        return self

    def tobytes(self) -> bytes:
        c, h, w = self.in_dims
        return (MAGIC + self._u32(self.version, c, h, w, len(self.records)) + b"".join(self.records))

    def save(self, path: str) -> int:
        blob = self.tobytes()
        with open(path, "wb") as fh:
            fh.write(blob)
        return len(blob)


def he_uniform(g: np.random.Generator, shape, fan_in: int) -> np.ndarray:
    lim = np.sqrt(6.0 / fan_in)
    return g.uniform(-lim, lim, size=shape).astype(np.float32)


def bn_params(g: np.random.Generator, ch: int):
    """BASELINE cfg3/cfg5 BN distributions: gamma U[0.5,1.5], beta U[-0.1,0.1],
    mean U[-0.1,0.1], var U[0.5,1.5]."""
    gamma = g.uniform(0.5, 1.5, ch).astype(np.float32)
    beta = g.uniform(-0.1, 0.1, ch).astype(np.float32)
    mean = g.uniform(-0.1, 0.1, ch).astype(np.float32)
    var = g.uniform(0.5, 1.5, ch).astype(np.float32)
    return mean, var, gamma, beta


VGG11_CONVS = [64, "M", 128, "M", 256, 256, "M", 512, 512, "M", 512, 512, "M"]


def vgg11(seed: int = 5, in_hw: int = 224, width_div: int = 1, fc_dims=(4096, 4096, 1000)) -> Acfun0Writer:
    """VGG-11-style ACFUN0 net of the BASELINE cfg5: Conv3x3 -> BN -> ReLU stacks of
    64,128,256x2,512x2,512x2 with MaxPool(2,2,0) after each stage, then
    FC 25088 -> 4096 -> ReLU -> 4096 -> ReLU -> 1000 -> Softmax.  He-uniform conv / FC
    weights, zero biases, seeded BN statistics.  `width_div` / `in_hw` / `fc_dims` shrink
    the net for tests."""
    g = np.random.default_rng(seed)
    W = Acfun0Writer(3, in_hw, in_hw)
    c, hw = 3, in_hw
    for v in VGG11_CONVS:
        if v == "M":
            W.maxpool(2, 2, 0)
            hw //= 2
            continue
        cout = max(v // width_div, 4)
        W.conv(he_uniform(g, (9 * c, cout), 9 * c), np.zeros(cout, np.float32), 3, 3, cout, 1, 1)
        W.bn(*bn_params(g, cout))
        W.relu()
        c = cout
    dim = hw * hw * c
    d1, d2, d3 = fc_dims
    W.fc(he_uniform(g, (dim, d1), dim), np.zeros(d1, np.float32), dim, d1).relu()
    W.fc(he_uniform(g, (d1, d2), d1), np.zeros(d2, np.float32), d1, d2).relu()
    W.fc(he_uniform(g, (d2, d3), d2), np.zeros(d3, np.float32), d2, d3).softmax()
    return W


def demo_net(seed: int = 7) -> Acfun0Writer:
    """A small net with every layer type (conv, BN, ReLU, depthwise/grouped conv, strided
    conv, max-pool, FC, softmax) in the shape of tools/gen_model.py:46-77, plus a grouped
    conv and a ReLU directly before a max-pool."""
    g = np.random.default_rng(seed)
    W = Acfun0Writer(3, 32, 32)
    u = lambda *s: g.uniform(-0.1, 0.1, size=s).astype(np.float32)
    W.conv(u(27, 16), u(16), 3, 3, 16, 1, 1).bn(*bn_params(g, 16)).relu()
    W.conv_g(u(16, 9), u(16), 3, 3, 16, groups=16).bn(*bn_params(g, 16)).relu()
    W.conv_g(u(4, 9 * 4, 8), u(32), 3, 3, 32, groups=4).relu()
    W.conv(u(9 * 32, 32), u(32), 3, 3, 32, 2, 1).bn(*bn_params(g, 32)).relu()
    W.maxpool(2, 2, 0)
    W.conv(u(32, 24), u(24), 1, 1, 24, 1, 0).relu().maxpool(2, 2, 0).relu()
    W.fc(u(4 * 4 * 24, 10), u(10), 4 * 4 * 24, 10).relu().softmax()
    return W


# ---------------------------------------------------------------- int8 model conversion
def _parse_records(blob: bytes):
    """(inC, inH, inW, [(type, header u32s, payload dict, raw record bytes)]) of an fp32 ACFUN0
    file (types 1-7), with each record's byte range."""
    if blob[:6] != MAGIC:
        raise ValueError("not an ACFUN0 file")
    u32 = lambda o: struct.unpack_from("<I", blob, o)[0]
    _, inC, inH, inW, num = struct.unpack_from("<5I", blob, 6)
    off, prevC, recs = 26, inC, []
    for _ in range(num):
        start, t = off, u32(off)
        off += 4
        rec = {"type": t}
        if t in (1, 7):
            n = 6 if t == 7 else 5
            hdr = struct.unpack_from("<%dI" % n, blob, off)
            off += 4 * n
            KH, KW, Cout, st, pd = hdr[:5]
            g = hdr[5] if t == 7 else 1
            wn = KH * KW * prevC * Cout // g
            rec.update(KH=KH, KW=KW, Cout=Cout, st=st, pd=pd, groups=g, Cin=prevC)
            rec["w"] = np.frombuffer(blob, "<f4", wn, off).copy()
            off += 4 * wn
            rec["b"] = np.frombuffer(blob, "<f4", Cout, off).copy()
            off += 4 * Cout
            prevC = Cout
        elif t == 2:
            Cout, inDim = struct.unpack_from("<2I", blob, off)
            off += 8 + 4 * (inDim * Cout + Cout)
            prevC = Cout
        elif t == 4:
            off += 12
        elif t == 6:
            ch = u32(off)
            rec["ch"] = ch
            rec["stats"] = np.frombuffer(blob, "<f4", 4 * ch, off + 4).copy().reshape(4, ch)
            off += 4 + 16 * ch
        elif t not in (3, 5):
            raise ValueError(f"unsupported layer type {t} for int8 conversion")
        rec["raw"] = blob[start:off]
        recs.append(rec)
    return inC, inH, inW, recs


def fold_bn(w, b, Cout, stats):
    """The loader's BN fold for a dense conv (model.cpp:69-95 expression order, every step one
    float32 rounding, no contraction): scale = gamma / sqrt(var + 1e-5), w *= scale,
    b = b * scale + (beta - mean * scale)."""
    mean, var, gamma, beta = (np.asarray(r, np.float32) for r in stats)
    f = np.float32
    scale = (gamma / np.sqrt((var + f(1e-5)).astype(f)).astype(f)).astype(f)
    shift = (beta - (mean * scale).astype(f)).astype(f)
    w2 = (w.reshape(-1, Cout) * scale).astype(f)
    b2 = ((b * scale).astype(f) + shift).astype(f)
    return w2.reshape(-1), b2


def quantize_model(blob: bytes, act_max=None) -> bytes:
    """An fp32 ACFUN0 file -> the same network with every dense Conv stored as a ConvInt8
    record: the loader's fusion rule (Conv [ReLU] [BN with ch == Cout] folds the BN) applied
    here, the folded weights quantised with the library's acfun_quantize_weights -- exactly what
    acfun_model_set_int8 computes at run time, so the file gives the same bits.  act_max: None
    (every conv measures its input's range per image) or one range per dense conv (0 keeps
    that conv's measured range)."""
    from . import quantize_weights
    inC, inH, inW, recs = _parse_records(blob)
    Wr = Acfun0Writer(inC, inH, inW)
    out = []
    n, i, k = len(recs), 0, 0
    while i < n:
        r = recs[i]
        if r["type"] != 1:
            out.append(r["raw"])
            i += 1
            continue
        w, b, Cout = r["w"], r["b"], r["Cout"]
        j, relu = i + 1, False
        if j < n and recs[j]["type"] == 3:
            relu, j = True, j + 1
        if j < n and recs[j]["type"] == 6 and recs[j]["ch"] == Cout:
            w, b = fold_bn(w, b, Cout, recs[j]["stats"])
            j += 1
        elif relu:
            j = i + 2          # the ReLU stays; no BN was consumed after it
        else:
            j = i + 1
        ws, wq = quantize_weights(np.ascontiguousarray(w.reshape(-1, Cout), np.float32))
        am = 0.0 if act_max is None else float(act_max[k])
        Wr.c = r["Cin"]
        Wr.records = []
        Wr.conv_int8(wq, ws, b, r["KH"], r["KW"], Cout, r["st"], r["pd"], am)
        out.append(Wr.records[0])
        if relu:
            out.append(struct.pack("<I", 3))
        k += 1
        i = j
    return MAGIC + struct.pack("<5I", 1, inC, inH, inW, len(out)) + b"".join(out)
