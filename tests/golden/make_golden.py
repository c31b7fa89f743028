"""Generate the golden parity fixtures in tests/golden/ by running the REFERENCE library.

The reference (hit-droid/Acfun) is compiled from its own sources into
oracle/_ref/libacfun_ref.so by ``make -C oracle ref`` (needs the reference source tree, so
run this where it is present).  Every fixture stores seeded inputs and the reference's own
outputs on this host (AVX-512F/BW/DQ/VNNI/BF16 routing, recorded in meta.json).  The CPU
tests pin the oracle against these files and the GPU tests check the CUDA library against
them, so neither needs the reference tree at run time.

    python tests/golden/make_golden.py
"""
import json
import os
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from acfun_b200 import acfun0  # noqa: E402
from oracle import pyoracle as P  # noqa: E402


def nul(a):
    return None if a is None else a.ctypes.data


def save(name, **arrays):
    np.savez_compressed(os.path.join(HERE, name + ".npz"), **arrays)


def main():
    R = P.ref()
    P.ref_set_threads(4)
    g = np.random.default_rng(20241201)
    meta = {"backend": R.acfun_backend_name().decode(), "cases": []}

    # ---- int8 GEMM (u8 x s8 -> s32) and its fused epilogue
    for (M, N, K) in [(63, 100, 37), (128, 256, 512), (255, 17, 1000)]:
        A = g.integers(0, 256, (M, K), dtype=np.uint8)
        B = g.integers(-128, 128, (K, N), dtype=np.int8)
        C = np.empty((M, N), np.int32)
        R.acfun_gemm_int8(M, N, K, A, B, C)
        save(f"gemm_int8_{M}x{N}x{K}", A=A, B=B, C=C)
        meta["cases"].append(f"gemm_int8_{M}x{N}x{K}")
    for (M, N, K, act) in [(100, 100, 100, 1), (127, 129, 63, 0), (1023, 4, 7, 1), (512, 17, 64, 1)]:
        A = g.integers(0, 256, (M, K), dtype=np.uint8)
        B = g.integers(-128, 128, (K, N), dtype=np.int8)
        al = g.uniform(1e-4, 1e-2, N).astype(np.float32)
        be = g.uniform(-20, 20, N).astype(np.float32)
        C = np.empty((M, N), np.float32)
        R.acfun_gemm_int8_epi(M, N, K, A, B, C, al, be, act)
        save(f"gemm_int8_epi_{M}x{N}x{K}_a{act}", A=A, B=B, alpha=al, beta=be, C=C, act=np.int32(act))
        meta["cases"].append(f"gemm_int8_epi_{M}x{N}x{K}_a{act}")

    # ---- s8 x s8 requant: the reference expresses it as u8 GEMM on A+128, then the exact
    # correction -128*colsum(B); the requant expression is applied to that int32 result.
    M, N, K = 96, 160, 320
    A = g.integers(-127, 128, (M, K), dtype=np.int8)
    B = g.integers(-127, 128, (K, N), dtype=np.int8)
    bias = g.integers(-1000, 1001, N, dtype=np.int32)
    scale = g.uniform(1e-3, 1e-2, N).astype(np.float32)
    Cu = np.empty((M, N), np.int32)
    R.acfun_gemm_int8(M, N, K, (A.astype(np.int16) + 128).astype(np.uint8), B, Cu)
    acc = (Cu.astype(np.int64) - 128 * B.astype(np.int64).sum(0)).astype(np.int32)
    for act in (0, 1):
        s = (acc.astype(np.int64) + bias).astype(np.int32)
        v = s.astype(np.float32) * scale
        if act:
            v = np.where(v > 0, v, np.float32(0))
        q = np.clip(np.rint(v), -128, 127).astype(np.int8)
        save(f"gemm_s8_requant_a{act}", A=A, B=B, bias=bias, scale=scale, acc=acc, C=q, act=np.int32(act))
        meta["cases"].append(f"gemm_s8_requant_a{act}")

    # ---- activation quantisation (AVX-512 path: round half to even)
    x = g.uniform(-3, 3, 4099).astype(np.float32)
    x[:12] = [0.5, -0.5, 1.5, 2.5, -2.5, 0.0, -0.0, 127.5, -127.5, 0.49999997, 3e9, -3e9]
    q = np.empty(x.size, np.uint8)
    R.acfun_quantize_u8(x, q, x.size, np.float32(1.0), 128)
    save("quantize_u8", x=x, q=q)
    meta["cases"].append("quantize_u8")

    # ---- weight quantisation + int8 conv, one case per route of conv_int8.cpp:63-148
    int8_cases = [
        ("wino", 2, 9, 11, 8, 3, 3, 16, 1, 1),
        ("wino_tailc", 1, 6, 6, 20, 3, 3, 21, 1, 1),
        ("direct_s2", 2, 10, 9, 3, 3, 3, 16, 2, 1),
        ("conv1x1", 1, 8, 8, 32, 1, 1, 24, 1, 0),
        ("im2col", 1, 9, 9, 40, 3, 3, 8, 2, 1),
        ("direct_1x1s2", 2, 7, 7, 20, 1, 1, 9, 2, 0),
    ]
    for (tag, N, H, W, Cin, KH, KW, Cout, st, pd) in int8_cases:
        x = g.uniform(-1, 1, (N, H, W, Cin)).astype(np.float32)
        w = g.uniform(-0.2, 0.2, (KH * KW * Cin, Cout)).astype(np.float32)
        ws = np.empty(Cout, np.float32)
        wq = np.empty((KH * KW * Cin, Cout), np.int8)
        R.acfun_quantize_weights(w, KH * KW * Cin, Cout, ws, wq)
        b = g.uniform(-0.5, 0.5, Cout).astype(np.float32)
        for act in (0, 1):
            out = P.ref_conv2d_int8(x, wq, ws, b, N, H, W, Cin, KH, KW, Cout, st, pd, act)
            save(f"conv_int8_{tag}_a{act}", x=x, w=w, wq=wq, ws=ws, b=b, out=out,
                 shape=np.array([N, H, W, Cin, KH, KW, Cout, st, pd, act], np.int32))
            meta["cases"].append(f"conv_int8_{tag}_a{act}")

    # ---- fp32 GEMM (+epi) and bf16 GEMM
    for (M, N, K) in [(64, 64, 64), (100, 100, 100), (33, 47, 129)]:
        A = g.uniform(-1, 1, (M, K)).astype(np.float32)
        B = g.uniform(-1, 1, (K, N)).astype(np.float32)
        bias = g.uniform(-1, 1, N).astype(np.float32)
        C = np.empty((M, N), np.float32)
        R.acfun_gemm_epi(M, N, K, A, B, C, nul(bias), 1)
        Cb = np.empty((M, N), np.float32)
        R.acfun_gemm_bf16(M, N, K, A, B, Cb)
        save(f"gemm_f32_{M}x{N}x{K}", A=A, B=B, bias=bias, C_epi_relu=C, C_bf16=Cb)
        meta["cases"].append(f"gemm_f32_{M}x{N}x{K}")

    # ---- float conv routes of layers.cpp:106-195
    f32_cases = [
        ("wino23", 2, 10, 9, 8, 3, 3, 8, 1, 1, 1),
        ("im2col_s2", 1, 11, 10, 5, 3, 3, 7, 2, 1, 1),
        ("k5", 1, 9, 9, 6, 5, 5, 4, 1, 2, 0),
        ("pw_s1", 2, 6, 7, 12, 1, 1, 10, 1, 0, 1),
        ("pw_s2", 1, 9, 9, 8, 1, 1, 16, 2, 0, 0),
    ]
    for (tag, N, H, W, Cin, KH, KW, Cout, st, pd, act) in f32_cases:
        x = g.uniform(0, 1, (N, H, W, Cin)).astype(np.float32)
        w = acfun0.he_uniform(g, (KH * KW * Cin, Cout), KH * KW * Cin)
        b = g.uniform(-0.1, 0.1, Cout).astype(np.float32)
        OH, OW = P.conv_out_hw(H, W, KH, KW, st, pd)
        out = np.empty((N, OH, OW, Cout), np.float32)
        fn = R.acfun_conv2d_relu if act else R.acfun_conv2d
        fn(x, N, H, W, Cin, w, nul(b), KH, KW, Cout, st, pd, out)
        save(f"conv_f32_{tag}", x=x, w=w, b=b, out=out,
             shape=np.array([N, H, W, Cin, KH, KW, Cout, st, pd, act, 1], np.int32))
        meta["cases"].append(f"conv_f32_{tag}")
    # F(4,3) through the internal entry point on a small map (the router needs >=112^2)
    x = g.uniform(0, 1, (1, 13, 11, 8)).astype(np.float32)
    w = acfun0.he_uniform(g, (72, 8), 72)
    b = g.uniform(-0.1, 0.1, 8).astype(np.float32)
    out = np.empty((1, 13, 11, 8), np.float32)
    fn = R.acfun_winograd43_conv3x3
    fn.argtypes = None
    fn(x.ctypes.data_as(P.C.c_void_p), 1, 13, 11, 8, w.ctypes.data_as(P.C.c_void_p),
       b.ctypes.data_as(P.C.c_void_p), 8, out.ctypes.data_as(P.C.c_void_p), 1)
    save("conv_f32_wino43", x=x, w=w, b=b, out=out,
         shape=np.array([1, 13, 11, 8, 3, 3, 8, 1, 1, 1, 1], np.int32))
    meta["cases"].append("conv_f32_wino43")

    # ---- depthwise and grouped
    for (tag, N, H, W, C, K, st, pd) in [("dw_s1", 2, 9, 8, 20, 3, 1, 1), ("dw_s2", 1, 10, 10, 16, 3, 2, 1)]:
        x = g.uniform(0, 1, (N, H, W, C)).astype(np.float32)
        w = acfun0.he_uniform(g, (C, K, K), K * K)
        b = g.uniform(-0.1, 0.1, C).astype(np.float32)
        OH, OW = P.conv_out_hw(H, W, K, K, st, pd)
        out = np.empty((N, OH, OW, C), np.float32)
        R.acfun_conv2d_dw(x, N, H, W, C, w, nul(b), K, K, st, pd, out, 1)
        save(f"conv_{tag}", x=x, w=w, b=b, out=out, shape=np.array([N, H, W, C, K, K, C, st, pd, 1, C], np.int32))
        meta["cases"].append(f"conv_{tag}")
    for (tag, N, H, W, Cin, Cout, gr, st) in [("grp_s1", 2, 7, 7, 24, 48, 6, 1), ("grp_s2", 1, 9, 9, 24, 48, 6, 2),
                                              ("grp_narrow", 1, 6, 6, 16, 16, 4, 1),
                                              ("grp_split", 1, 5, 5, 160, 16, 2, 1)]:
        x = g.uniform(0, 1, (N, H, W, Cin)).astype(np.float32)
        w = acfun0.he_uniform(g, (gr, 9 * (Cin // gr), Cout // gr), 9 * (Cin // gr))
        b = g.uniform(-0.1, 0.1, Cout).astype(np.float32)
        OH, OW = P.conv_out_hw(H, W, 3, 3, st, 1)
        out = np.empty((N, OH, OW, Cout), np.float32)
        R.acfun_conv2d_g(x, N, H, W, Cin, w, nul(b), 3, 3, Cout, st, 1, gr, out, 1)
        save(f"conv_{tag}", x=x, w=w, b=b, out=out, shape=np.array([N, H, W, Cin, 3, 3, Cout, st, 1, 1, gr], np.int32))
        meta["cases"].append(f"conv_{tag}")

    # ---- max pool, softmax, batch norm, FC
    for (tag, N, H, W, C, pool, st, pd, post) in [("mp2", 2, 9, 9, 20, 2, 2, 0, 0), ("mp3", 1, 7, 7, 5, 3, 2, 1, 1),
                                                   ("mp2_c64", 1, 8, 8, 64, 2, 2, 0, 1)]:
        x = g.uniform(-1, 1, (N, H, W, C)).astype(np.float32)
        OH, OW = P.conv_out_hw(H, W, pool, pool, st, pd)
        out = np.empty((N, OH, OW, C), np.float32)
        (R.acfun_maxpool_relu if post else R.acfun_maxpool)(x, N, H, W, C, pool, st, pd, out)
        save(f"maxpool_{tag}", x=x, out=out, shape=np.array([N, H, W, C, pool, st, pd, post], np.int32))
        meta["cases"].append(f"maxpool_{tag}")
    x = g.uniform(-5, 5, (3, 1000)).astype(np.float32)
    out = np.empty_like(x)
    R.acfun_softmax(x, 3, 1000, out)
    save("softmax", x=x, out=out)
    d = g.uniform(-1, 1, (4, 5, 5, 12)).astype(np.float32)
    mean, var, gamma, beta = acfun0.bn_params(g, 12)
    d2 = d.copy()
    R.acfun_batchnorm(d2, d2.size, 12, mean, var, nul(gamma), nul(beta), np.float32(1e-5))
    save("batchnorm", x=d, mean=mean, var=var, gamma=gamma, beta=beta, out=d2)
    x = g.uniform(-1, 1, (5, 300)).astype(np.float32)
    w = g.uniform(-0.1, 0.1, (300, 70)).astype(np.float32)
    b = g.uniform(-0.1, 0.1, 70).astype(np.float32)
    o1 = np.empty((5, 70), np.float32)
    o2 = np.empty((5, 70), np.float32)
    R.acfun_fc(x, 5, 300, w, nul(b), 70, o1)
    R.acfun_fc_relu(x, 5, 300, w, nul(b), 70, o2)
    save("fc", x=x, w=w, b=b, out=o1, out_relu=o2)
    meta["cases"] += ["softmax", "batchnorm", "fc"]

    # ---- end-to-end ACFUN0 (every layer type, loader fusion quirks included)
    blob = acfun0.demo_net(seed=7).tobytes()
    with tempfile.NamedTemporaryFile(suffix=".acfun", delete=False) as fh:
        fh.write(blob)
        path = fh.name
    m = R.acfun_model_load(path.encode())
    assert m
    xs = g.uniform(0, 1, (2, 32, 32, 3)).astype(np.float32)
    outs = []
    for k in range(2):
        o = np.empty(4096, np.float32)
        n = R.acfun_model_infer(m, np.ascontiguousarray(xs[k]), o)
        outs.append(o[:n].copy())
    R.acfun_model_destroy(m)
    os.unlink(path)
    save("model_demo", blob=np.frombuffer(blob, np.uint8), x=xs, out=np.stack(outs))
    meta["cases"].append("model_demo")

    with open(os.path.join(HERE, "meta.json"), "w") as fh:
        json.dump(meta, fh, indent=1)
    total = sum(os.path.getsize(os.path.join(HERE, f)) for f in os.listdir(HERE) if f.endswith(".npz"))
    print(f"{len(meta['cases'])} fixtures, {total / 1024:.0f} KiB")


if __name__ == "__main__":
    main()
