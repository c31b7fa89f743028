"""TEST INFRASTRUCTURE ONLY: CPU restatement of the ACFUN0 loader, fuser and executor.

Follows hit-droid/Acfun src/model.cpp:
  * parse           model.cpp:106-196 (magic, version, inC/inH/inW, layer records)
  * fuse            model.cpp:198-247 — for Conv/FC/ConvGrouped: an optional ReLU, then an
                    optional BN with ch == Cout folded into the weights (fold_bn_into,
                    :69-95); a ReLU followed by MaxPool is DROPPED (:220-224, :232); a
                    MaxPool followed by ReLU gets post_relu (:241)
  * execute         model.cpp:274-349 — batch 1, ping-pong buffers, Softmax over the whole
                    current tensor (:335), FC flattens NHWC
Layer math uses the C oracle (acfun_oracle.c).
"""
from __future__ import annotations

import struct

import numpy as np

from . import pyoracle as P


class OracleModel:
    def __init__(self, blob: bytes):
        if len(blob) < 6 + 16 or blob[:6] != b"ACFUN0":
            raise ValueError("bad ACFUN0 magic/size")
        u32 = lambda o: struct.unpack_from("<I", blob, o)[0]
        off = 10
        self.inC, self.inH, self.inW, num = (u32(off), u32(off + 4), u32(off + 8), u32(off + 12))
        off += 16
        raw = []
        prevC = self.inC
        for _ in range(num):
            t = u32(off)
            off += 4
            L = {"type": t}
            if t in (1, 7):
                KH, KW, Cout, st, pd = (u32(off + 4 * k) for k in range(5))
                off += 20
                groups = 1
                if t == 7:
                    groups = u32(off)
                    off += 4
                wn = KH * KW * prevC * Cout // groups
                L.update(KH=KH, KW=KW, Cout=Cout, st=st, pd=pd, groups=groups, wn=wn)
                L["w"] = np.frombuffer(blob, "<f4", wn, off).copy()
                off += 4 * wn
                L["b"] = np.frombuffer(blob, "<f4", Cout, off).copy()
                off += 4 * Cout
                prevC = Cout
            elif t == 2:
                Cout, inDim = u32(off), u32(off + 4)
                off += 8
                L.update(Cout=Cout, inDim=inDim, wn=inDim * Cout, groups=0)
                L["w"] = np.frombuffer(blob, "<f4", inDim * Cout, off).copy()
                off += 4 * inDim * Cout
                L["b"] = np.frombuffer(blob, "<f4", Cout, off).copy()
                off += 4 * Cout
                prevC = Cout
            elif t == 4:
                L.update(pool=u32(off), st=u32(off + 4), pd=u32(off + 8))
                off += 12
            elif t == 6:
                ch = u32(off)
                off += 4
                L["ch"] = ch
                L["stats"] = np.frombuffer(blob, "<f4", 4 * ch, off).copy().reshape(4, ch)
                off += 16 * ch
            elif t in (3, 5):
                pass
            else:
                raise ValueError(f"unknown layer type {t}")
            raw.append(L)
        self.layers = self._fuse(raw)

    @staticmethod
    def _fuse(raw):
        out = []
        consumed = [False] * len(raw)
        n = len(raw)
        for i, L in enumerate(raw):
            if consumed[i]:
                continue
            t = L["type"]
            if t in (1, 2, 7):
                F = dict(L)
                F["act"] = 0
                Cout = L["Cout"]
                j = i + 1
                relu_idx = -1
                if j < n and raw[j]["type"] == 3:
                    relu_idx = j
                    j += 1
                if j < n and raw[j]["type"] == 6 and raw[j]["ch"] == Cout:
                    w = F["w"].copy()
                    b = F["b"].copy()
                    mean, var, gamma, beta = (np.ascontiguousarray(s) for s in raw[j]["stats"])
                    P.oracle().orc_fold_bn(w, b, w.size, Cout, F["groups"] if t == 7 else 0,
                                           mean, var, gamma, beta)
                    F["w"], F["b"] = w, b
                    consumed[j] = True
                if relu_idx >= 0:
                    consumed[relu_idx] = True
                    F["act"] = 0 if (j < n and raw[j]["type"] == 4) else 1
                out.append(F)
            elif t == 3:
                if i + 1 < n and raw[i + 1]["type"] == 4:
                    consumed[i] = True
                    continue
                out.append({"type": 3})
            elif t == 6:
                out.append(dict(L))
            elif t == 4:
                F = dict(L)
                F["post_relu"] = 0
                if i + 1 < n and raw[i + 1]["type"] == 3:
                    F["post_relu"] = 1
                    consumed[i + 1] = True
                out.append(F)
            else:
                out.append(dict(L))
        return out

    def infer(self, x: np.ndarray, int8: bool = False) -> np.ndarray:
        """One image.  int8=True runs every dense conv as the reference's int8 harness does:
        acfun_quantize_weights of the folded weights, then acfun_conv2d_int8 on this image
        (conv_int8.cpp:24-37, :63-148); everything else stays fp32."""
        O = P.oracle()
        H, W, C = self.inH, self.inW, self.inC
        cur = np.ascontiguousarray(x, np.float32).reshape(-1).copy()
        for L in self.layers:
            t = L["type"]
            if t == 1 and int8:
                KH, KW, Cout, st, pd = L["KH"], L["KW"], L["Cout"], L["st"], L["pd"]
                if "wq" not in L:
                    K = KH * KW * C
                    L["ws"] = np.empty(Cout, np.float32)
                    L["wq"] = np.empty((K, Cout), np.int8)
                    O.orc_quantize_weights(np.ascontiguousarray(L["w"], np.float32), K, Cout, L["ws"], L["wq"])
                out = P.orc_conv2d_int8(cur, L["wq"], L["ws"], L["b"], 1, H, W, C, KH, KW, Cout, st, pd,
                                        L["act"])
                OH, OW = P.conv_out_hw(H, W, KH, KW, st, pd)
                cur, H, W, C = out.reshape(-1), OH, OW, Cout
            elif t in (1, 7):
                KH, KW, Cout, st, pd = L["KH"], L["KW"], L["Cout"], L["st"], L["pd"]
                groups = L.get("groups", 1) if t == 7 else 1
                OH, OW = P.conv_out_hw(H, W, KH, KW, st, pd)
                out = np.empty(OH * OW * Cout, np.float32)
                O.orc_conv2d(cur, 1, H, W, C, L["w"], L["b"].ctypes.data, KH, KW, Cout, st, pd,
                             groups if groups > 1 else 1, out, L["act"])
                cur, H, W, C = out, OH, OW, Cout
            elif t == 2:
                out = np.empty(L["Cout"], np.float32)
                O.orc_fc(cur, 1, H * W * C, L["w"], L["b"].ctypes.data, L["Cout"], out, L["act"])
                cur, H, W, C = out, 1, 1, L["Cout"]
            elif t == 3:
                O.orc_relu(cur, cur.size)
            elif t == 4:
                OH, OW = P.conv_out_hw(H, W, L["pool"], L["pool"], L["st"], L["pd"])
                out = np.empty(OH * OW * C, np.float32)
                O.orc_maxpool(cur, 1, H, W, C, L["pool"], L["st"], L["pd"], out, L["post_relu"])
                cur, H, W = out, OH, OW
            elif t == 5:
                out = np.empty_like(cur)
                O.orc_softmax(cur, 1, cur.size, out)
                cur = out
            elif t == 6:
                ch = L["ch"]
                mean, var, gamma, beta = (np.ascontiguousarray(s) for s in L["stats"])
                O.orc_batchnorm(cur, cur.size, ch, mean, var, gamma.ctypes.data, beta.ctypes.data,
                                np.float32(1e-5))
        return cur

    def ref_infer(self, R, x: np.ndarray, int8: bool = False) -> np.ndarray:
        """One image through the reference library itself (R = pyoracle.ref()), layer by layer
        over this fused list: the harness composition the reference needs for an int8 model
        (it has no int8 model format), or its fp32 layer API.  CPU-baseline timing only."""
        H, W, C = self.inH, self.inW, self.inC
        cur = np.ascontiguousarray(x, np.float32).reshape(-1).copy()
        for L in self.layers:
            t = L["type"]
            if t in (1, 7):
                KH, KW, Cout, st, pd = L["KH"], L["KW"], L["Cout"], L["st"], L["pd"]
                OH, OW = P.conv_out_hw(H, W, KH, KW, st, pd)
                out = np.empty(OH * OW * Cout, np.float32)
                b = L["b"].ctypes.data
                if t == 1 and int8:
                    if "ref_wq" not in L:
                        K = KH * KW * C
                        L["ref_ws"] = np.empty(Cout, np.float32)
                        L["ref_wq"] = np.empty((K, Cout), np.int8)
                        R.acfun_quantize_weights(np.ascontiguousarray(L["w"], np.float32), K, Cout,
                                                 L["ref_ws"], L["ref_wq"])
                    R.acfun_conv2d_int8(cur, 1, H, W, C, L["ref_wq"], L["ref_ws"], b, KH, KW, Cout, st, pd,
                                        0.0, out, L["act"])
                else:
                    groups = L.get("groups", 1) if t == 7 else 1
                    R.acfun_conv2d_g(cur, 1, H, W, C, np.ascontiguousarray(L["w"], np.float32), b, KH, KW,
                                     Cout, st, pd, groups, out, L["act"])
                cur, H, W, C = out, OH, OW, Cout
            elif t == 2:
                out = np.empty(L["Cout"], np.float32)
                fn = R.acfun_fc_relu if L["act"] else R.acfun_fc
                fn(cur, 1, H * W * C, np.ascontiguousarray(L["w"], np.float32), L["b"].ctypes.data, L["Cout"], out)
                cur, H, W, C = out, 1, 1, L["Cout"]
            elif t == 3:
                R.acfun_relu(cur, cur.size)
            elif t == 4:
                OH, OW = P.conv_out_hw(H, W, L["pool"], L["pool"], L["st"], L["pd"])
                out = np.empty(OH * OW * C, np.float32)
                fn = R.acfun_maxpool_relu if L["post_relu"] else R.acfun_maxpool
                fn(cur, 1, H, W, C, L["pool"], L["st"], L["pd"], out)
                cur, H, W = out, OH, OW
            elif t == 5:
                out = np.empty_like(cur)
                R.acfun_softmax(cur, 1, cur.size, out)
                cur = out
            elif t == 6:
                ch = L["ch"]
                mean, var, gamma, beta = (np.ascontiguousarray(s) for s in L["stats"])
                R.acfun_batchnorm(cur, cur.size, ch, mean, var, gamma.ctypes.data, beta.ctypes.data,
                                  np.float32(1e-5))
        return cur
