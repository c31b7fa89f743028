"""TEST INFRASTRUCTURE ONLY: ctypes access to the CPU oracle and to the reference library.

* ``liboracle.so`` — the plain-C restatement in ``oracle/acfun_oracle.c`` (built by
  ``make -C oracle`` with the system gcc; built on demand here when missing).
* ``libacfun_ref.so`` — the hit-droid/Acfun reference compiled from its own sources by
  ``make -C oracle ref`` (optional: present only where the reference tree was available at
  build time, or where the prebuilt file travelled with the repository snapshot).

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / reference legs
import this module.  The product library never does.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
import threading

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "_build", "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "libacfun_ref.so")

_lock = threading.Lock()
_oracle = None
_ref = None

f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
u8p = np.ctypeslib.ndpointer(np.uint8, flags="C_CONTIGUOUS")
s8p = np.ctypeslib.ndpointer(np.int8, flags="C_CONTIGUOUS")
s32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")
i, f, sz = C.c_int, C.c_float, C.c_size_t


def _null_or(arr):
    return None if arr is None else arr.ctypes.data_as(C.c_void_p)


def build_oracle(force: bool = False) -> str:
    src = os.path.join(HERE, "acfun_oracle.c")
    if force or not os.path.exists(ORACLE_SO) or os.path.getmtime(ORACLE_SO) < os.path.getmtime(src):
        subprocess.run(["make", "-s", "-C", HERE], check=True)
    return ORACLE_SO


def oracle() -> C.CDLL:
    global _oracle
    with _lock:
        if _oracle is None:
            lib = C.CDLL(build_oracle())
            vp = C.c_void_p
            sig = {
                "orc_gemm_f32": [i, i, i, f32p, f32p, f32p, vp, i],
                "orc_gemm_bf16": [i, i, i, f32p, f32p, f32p],
                "orc_gemm_int8": [i, i, i, u8p, s8p, s32p],
                "orc_gemm_int8_epi": [i, i, i, u8p, s8p, f32p, f32p, f32p, i],
                "orc_gemm_s8_requant": [i, i, i, s8p, s8p, vp, f32p, s8p, i],
                "orc_quantize_u8": [f32p, u8p, sz, f, i, i],
                "orc_quantize_weights": [f32p, i, i, f32p, s8p],
                "orc_conv2d_int8": [f32p, i, i, i, i, s8p, f32p, vp, i, i, i, i, i, f, f32p, i],
                "orc_conv2d_int8_route": [f32p, i, i, i, i, i, i, i, i, i],
                "orc_winograd_int8": [f32p, i, i, i, i, s8p, f32p, vp, i, f, f, f32p, i],
                "orc_conv2d_int8_direct": [u8p, i, i, i, i, s8p, f32p, f32p, i, i, i, i, i, i, i, f32p, i],
                "orc_conv2d": [f32p, i, i, i, i, f32p, vp, i, i, i, i, i, i, f32p, i],
                "orc_conv2d_route": [i] * 10,
                "orc_winograd23": [f32p, i, i, i, i, f32p, vp, i, f32p, i],
                "orc_winograd43": [f32p, i, i, i, i, f32p, vp, i, f32p, i],
                "orc_fc": [f32p, i, i, f32p, vp, i, f32p, i],
                "orc_relu": [f32p, sz],
                "orc_relu6": [f32p, sz],
                "orc_maxpool": [f32p, i, i, i, i, i, i, i, f32p, i],
                "orc_softmax": [f32p, i, i, f32p],
                "orc_batchnorm": [f32p, i, i, f32p, f32p, vp, vp, f],
                "orc_fold_bn": [f32p, f32p, sz, i, i, f32p, f32p, f32p, f32p],
            }
            for name, args in sig.items():
                fn = getattr(lib, name)
                fn.argtypes = args
                fn.restype = i if name.endswith("_route") else None
            _oracle = lib
        return _oracle


def ref_available() -> bool:
    return os.path.exists(REF_SO)


def ref() -> C.CDLL:
    """The reference library (raises FileNotFoundError when it was never built)."""
    global _ref
    with _lock:
        if _ref is None:
            if not os.path.exists(REF_SO):
                raise FileNotFoundError(REF_SO)
            lib = C.CDLL(REF_SO)
            vp = C.c_void_p
            sig = {
                "acfun_set_threads": [i],
                "acfun_set_num_threads_runtime": [i],
                "acfun_effective_cores": [],
                "acfun_backend_name": [],
                "acfun_gemm": [i, i, i, f32p, f32p, f32p],
                "acfun_gemm_epi": [i, i, i, f32p, f32p, f32p, vp, i],
                "acfun_gemm_bf16": [i, i, i, f32p, f32p, f32p],
                "acfun_gemm_int8": [i, i, i, u8p, s8p, s32p],
                "acfun_gemm_int8_epi": [i, i, i, u8p, s8p, f32p, f32p, f32p, i],
                "acfun_quantize_u8": [f32p, u8p, sz, f, i],
                "acfun_quantize_weights": [f32p, i, i, f32p, s8p],
                "acfun_conv2d_int8": [f32p, i, i, i, i, s8p, f32p, vp, i, i, i, i, i, f, f32p, i],
                "acfun_conv2d_int8_direct": [u8p, i, i, i, i, s8p, f32p, f32p, i, i, i, i, i, i, i, f32p, i],
                "acfun_conv1x1_int8": [u8p, i, i, i, s8p, f32p, f32p, f32p, i],
                "acfun_conv2d": [f32p, i, i, i, i, f32p, vp, i, i, i, i, i, f32p],
                "acfun_conv2d_relu": [f32p, i, i, i, i, f32p, vp, i, i, i, i, i, f32p],
                "acfun_conv2d_dw": [f32p, i, i, i, i, f32p, vp, i, i, i, i, f32p, i],
                "acfun_conv2d_g": [f32p, i, i, i, i, f32p, vp, i, i, i, i, i, i, f32p, i],
                "acfun_fc": [f32p, i, i, f32p, vp, i, f32p],
                "acfun_fc_relu": [f32p, i, i, f32p, vp, i, f32p],
                "acfun_relu": [f32p, sz],
                "acfun_relu6": [f32p, sz],
                "acfun_maxpool": [f32p, i, i, i, i, i, i, i, f32p],
                "acfun_maxpool_relu": [f32p, i, i, i, i, i, i, i, f32p],
                "acfun_softmax": [f32p, i, i, f32p],
                "acfun_batchnorm": [f32p, i, i, f32p, f32p, vp, vp, f],
                "acfun_model_load": [C.c_char_p],
                "acfun_model_destroy": [vp],
                "acfun_model_infer": [vp, f32p, f32p],
                "acfun_model_output_size": [vp],
            }
            for name, args in sig.items():
                fn = getattr(lib, name)
                fn.argtypes = args
                fn.restype = None
            lib.acfun_effective_cores.restype = i
            lib.acfun_backend_name.restype = C.c_char_p
            lib.acfun_model_load.restype = vp
            lib.acfun_model_infer.restype = i
            lib.acfun_model_output_size.restype = i
            _ref = lib
        return _ref


def ref_set_threads(n: int) -> None:
    lib = ref()
    lib.acfun_set_threads(n)
    lib.acfun_set_num_threads_runtime(n)


# ------------------------------------------------------------------ numpy conveniences
def conv_out_hw(H, W, KH, KW, stride, pad):
    return (H + 2 * pad - KH) // stride + 1, (W + 2 * pad - KW) // stride + 1


def orc_conv2d_int8(x, wq, ws, bias, N, H, W, Cin, KH, KW, Cout, stride, pad, act):
    OH, OW = conv_out_hw(H, W, KH, KW, stride, pad)
    out = np.empty((N, OH, OW, Cout), np.float32)
    oracle().orc_conv2d_int8(x, N, H, W, Cin, wq, ws, _null_or(bias), KH, KW, Cout, stride, pad,
                             0.0, out, act)
    return out


def ref_conv2d_int8(x, wq, ws, bias, N, H, W, Cin, KH, KW, Cout, stride, pad, act):
    OH, OW = conv_out_hw(H, W, KH, KW, stride, pad)
    out = np.empty((N, OH, OW, Cout), np.float32)
    ref().acfun_conv2d_int8(x, N, H, W, Cin, wq, ws, _null_or(bias), KH, KW, Cout, stride, pad,
                            0.0, out, act)
    return out
