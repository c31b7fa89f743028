"""acfun_b200 — Python host mirror of the Acfun C API, backed by libacfun_b200.so.

The shared library (hand-written sm_100a CUDA behind an ``extern "C"`` boundary declared in
``include/acfun/*.h``) is the product; this module only binds it with ctypes and offers
numpy / torch conveniences with the reference's names and argument meaning.  There is no
CPU fallback: if the library is missing or no GPU is present, calls raise.

Tensor arguments may be numpy arrays (host memory, synchronous calls) or CUDA torch tensors
(device memory, stream-ordered calls; use ``synchronize()`` before reading on the host).
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
import threading

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libacfun_b200.so")

_lock = threading.Lock()
_lib = None

vp, i, f, sz = C.c_void_p, C.c_int, C.c_float, C.c_size_t

# every exported entry point with its ctypes signature (restype, argtypes)
SIGNATURES = {
    # acfun.h
    "acfun_set_threads": (None, [i]),
    "acfun_backend": (i, []),
    "acfun_backend_name": (C.c_char_p, []),
    "acfun_autotune": (None, []),
    "acfun_tune_status": (C.c_char_p, []),
    "acfun_gemm": (None, [i, i, i, vp, vp, vp]),
    "acfun_gemm_epi": (None, [i, i, i, vp, vp, vp, vp, i]),
    "acfun_gemm_bf16": (None, [i, i, i, vp, vp, vp]),
    "acfun_conv2d": (None, [vp, i, i, i, i, vp, vp, i, i, i, i, i, vp]),
    "acfun_conv2d_relu": (None, [vp, i, i, i, i, vp, vp, i, i, i, i, i, vp]),
    "acfun_conv2d_dw": (None, [vp, i, i, i, i, vp, vp, i, i, i, i, vp, i]),
    "acfun_conv2d_g": (None, [vp, i, i, i, i, vp, vp, i, i, i, i, i, i, vp, i]),
    "acfun_fc": (None, [vp, i, i, vp, vp, i, vp]),
    "acfun_fc_relu": (None, [vp, i, i, vp, vp, i, vp]),
    "acfun_relu": (None, [vp, sz]),
    "acfun_relu6": (None, [vp, sz]),
    "acfun_maxpool": (None, [vp, i, i, i, i, i, i, i, vp]),
    "acfun_maxpool_relu": (None, [vp, i, i, i, i, i, i, i, vp]),
    "acfun_softmax": (None, [vp, i, i, vp]),
    "acfun_batchnorm": (None, [vp, i, i, vp, vp, vp, vp, f]),
    "acfun_quantize_weights": (None, [vp, i, i, vp, vp]),
    "acfun_conv2d_int8": (None, [vp, i, i, i, i, vp, vp, vp, i, i, i, i, i, f, vp, i]),
    "acfun_model_load": (vp, [C.c_char_p]),
    "acfun_model_destroy": (None, [vp]),
    "acfun_model_infer": (i, [vp, vp, vp]),
    "acfun_model_output_size": (i, [vp]),
    "acfun_model_input_dims": (None, [vp, vp, vp, vp]),
    "acfun_model_infer_batch": (i, [vp, i, vp, vp]),
    "acfun_model_set_int8": (i, [vp, i]),
    "acfun_gemm_s8_requant": (None, [i, i, i, vp, vp, vp, vp, vp, i]),
    "acfun_gemm_epi_noalloc": (i, [i, i, i, vp, vp, vp, vp, i]),
    "acfun_set_fp32_math": (i, [i]),
    "acfun_set_stream": (None, [vp]),
    "acfun_get_stream": (vp, []),
    "acfun_set_device": (i, [i]),
    "acfun_synchronize": (i, []),
    "acfun_last_error_code": (i, []),
    "acfun_last_error": (C.c_char_p, []),
    "acfun_clear_error": (None, []),
    # acfun_internal.h
    "acfun_set_num_threads_runtime": (None, [i]),
    "acfun_get_num_threads_runtime": (i, []),
    "acfun_pick_threads": (i, [i, i, i]),
    "acfun_effective_cores": (i, []),
    "acfun_gemm_int8": (None, [i, i, i, vp, vp, vp]),
    "acfun_gemm_int8_epi": (None, [i, i, i, vp, vp, vp, vp, vp, i]),
    "acfun_quantize_u8": (None, [vp, vp, sz, f, i]),
    "acfun_conv2d_int8_direct": (None, [vp, i, i, i, i, vp, vp, vp, i, i, i, i, i, i, i, vp, i]),
    "acfun_conv1x1_int8": (None, [vp, i, i, i, vp, vp, vp, vp, i]),
    "acfun_winograd_conv3x3_int8": (None, [vp, i, i, i, i, vp, vp, vp, i, f, f, vp, i]),
    "acfun_winograd_conv3x3": (None, [vp, i, i, i, i, vp, vp, i, vp, i]),
    "acfun_winograd43_conv3x3": (None, [vp, i, i, i, i, vp, vp, i, vp, i]),
    "acfun_conv2d_grouped": (None, [vp, i, i, i, i, vp, vp, i, i, i, i, i, i, vp, i]),
}


class AcfunError(RuntimeError):
    """Raised when the library reports an error through acfun_last_error()."""


def build(jobs: int = 8) -> str:
    """Compile libacfun_b200.so for sm_100a (nvcc; works without a GPU)."""
    subprocess.run(["make", "-s", "-C", HERE, f"-j{jobs}"], check=True)
    return LIB_PATH


def lib() -> C.CDLL:
    """The loaded library; raises if it has not been built (there is no fallback)."""
    global _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise FileNotFoundError(f"{LIB_PATH} is missing: run acfun_b200.build()")
            L = C.CDLL(LIB_PATH)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(L, name, None)
                if fn is None:
                    continue
                fn.restype = res
                fn.argtypes = args
            _lib = L
        return _lib


def ptr(x):
    """Raw address of a numpy array / torch tensor (None -> NULL)."""
    if x is None:
        return None
    if isinstance(x, np.ndarray):
        if not x.flags["C_CONTIGUOUS"]:
            raise ValueError("arrays must be C-contiguous")
        return x.ctypes.data
    if hasattr(x, "data_ptr"):
        if not x.is_contiguous():
            raise ValueError("tensors must be contiguous")
        return x.data_ptr()
    if isinstance(x, int):
        return x
    raise TypeError(f"unsupported tensor type {type(x)!r}")


def check() -> None:
    """Raise AcfunError if the last call of this thread failed (and clear the error)."""
    L = lib()
    code = L.acfun_last_error_code()
    if code:
        msg = L.acfun_last_error().decode(errors="replace")
        L.acfun_clear_error()
        raise AcfunError(f"acfun error {code}: {msg}")


def synchronize() -> None:
    L = lib()
    if L.acfun_synchronize():
        check()


def _call(name, *args):
    getattr(lib(), name)(*[ptr(a) if isinstance(a, np.ndarray) or hasattr(a, "data_ptr") else a
                           for a in args])
    check()


def _empty_like_kind(x, shape, dtype):
    if isinstance(x, np.ndarray):
        return np.empty(shape, dtype=dtype)
    import torch  # device tensors
    tmap = {np.float32: torch.float32, np.int32: torch.int32, np.int8: torch.int8, np.uint8: torch.uint8}
    return torch.empty(shape, dtype=tmap[dtype], device=x.device)


def conv_out_hw(H, W, KH, KW, stride, pad):
    return (H + 2 * pad - KH) // stride + 1, (W + 2 * pad - KW) // stride + 1


# ------------------------------------------------------------------ GEMM family
def gemm(A, B, bias=None, act=0):
    M, K = A.shape
    N = B.shape[1]
    Cm = _empty_like_kind(A, (M, N), np.float32)
    _call("acfun_gemm_epi", M, N, K, A, B, Cm, bias, act)
    return Cm


def gemm_bf16(A, B):
    M, K = A.shape
    N = B.shape[1]
    Cm = _empty_like_kind(A, (M, N), np.float32)
    _call("acfun_gemm_bf16", M, N, K, A, B, Cm)
    return Cm


def gemm_int8(A, B):
    M, K = A.shape
    N = B.shape[1]
    Cm = _empty_like_kind(A, (M, N), np.int32)
    _call("acfun_gemm_int8", M, N, K, A, B, Cm)
    return Cm


def gemm_int8_epi(A, B, alpha, beta, act=0):
    M, K = A.shape
    N = B.shape[1]
    Cm = _empty_like_kind(A, (M, N), np.float32)
    _call("acfun_gemm_int8_epi", M, N, K, A, B, Cm, alpha, beta, act)
    return Cm


def gemm_s8_requant(A, B, bias, scale, act=1):
    M, K = A.shape
    N = B.shape[1]
    Cm = _empty_like_kind(A, (M, N), np.int8)
    _call("acfun_gemm_s8_requant", M, N, K, A, B, bias, scale, Cm, act)
    return Cm


# ------------------------------------------------------------------ conv family
def conv2d(x, w, bias, KH, KW, Cout, stride, pad, act=0, groups=1):
    N, H, W, Cin = x.shape
    OH, OW = conv_out_hw(H, W, KH, KW, stride, pad)
    out = _empty_like_kind(x, (N, OH, OW, Cout), np.float32)
    if groups > 1:
        _call("acfun_conv2d_g", x, N, H, W, Cin, w, bias, KH, KW, Cout, stride, pad, groups, out, act)
    elif act:
        _call("acfun_conv2d_relu", x, N, H, W, Cin, w, bias, KH, KW, Cout, stride, pad, out)
    else:
        _call("acfun_conv2d", x, N, H, W, Cin, w, bias, KH, KW, Cout, stride, pad, out)
    return out


def conv2d_dw(x, w, bias, KH, KW, stride, pad, act=0):
    N, H, W, Cc = x.shape
    OH, OW = conv_out_hw(H, W, KH, KW, stride, pad)
    out = _empty_like_kind(x, (N, OH, OW, Cc), np.float32)
    _call("acfun_conv2d_dw", x, N, H, W, Cc, w, bias, KH, KW, stride, pad, out, act)
    return out


def conv2d_int8(x, wq, wscale, bias, KH, KW, Cout, stride, pad, act=0):
    N, H, W, Cin = x.shape
    OH, OW = conv_out_hw(H, W, KH, KW, stride, pad)
    out = _empty_like_kind(x, (N, OH, OW, Cout), np.float32)
    _call("acfun_conv2d_int8", x, N, H, W, Cin, wq, wscale, bias, KH, KW, Cout, stride, pad,
          0.0, out, act)
    return out


def quantize_weights(w):
    K, N = w.shape
    scales = np.empty(N, np.float32)
    wq = np.empty((K, N), np.int8)
    _call("acfun_quantize_weights", w, K, N, scales, wq)
    return scales, wq


def fc(x, w, bias, act=0):
    N, Cin = x.shape
    Cout = w.shape[1]
    out = _empty_like_kind(x, (N, Cout), np.float32)
    _call("acfun_fc_relu" if act else "acfun_fc", x, N, Cin, w, bias, Cout, out)
    return out


def maxpool(x, pool, stride, pad, post_relu=0):
    N, H, W, Cc = x.shape
    OH, OW = conv_out_hw(H, W, pool, pool, stride, pad)
    out = _empty_like_kind(x, (N, OH, OW, Cc), np.float32)
    _call("acfun_maxpool_relu" if post_relu else "acfun_maxpool", x, N, H, W, Cc, pool, stride, pad, out)
    return out


def softmax(x):
    rows, cols = x.shape
    out = _empty_like_kind(x, (rows, cols), np.float32)
    _call("acfun_softmax", x, rows, cols, out)
    return out


# ------------------------------------------------------------------ model
class Model:
    """ACFUN0 model loaded by acfun_model_load (weights resident on the GPU)."""

    def __init__(self, path: str):
        self.h = lib().acfun_model_load(os.fsencode(path))
        if not self.h:
            code = lib().acfun_last_error_code()
            msg = lib().acfun_last_error().decode(errors="replace")
            lib().acfun_clear_error()
            raise AcfunError(f"acfun_model_load failed ({code}): {msg}")
        c_, h_, w_ = C.c_int(), C.c_int(), C.c_int()
        lib().acfun_model_input_dims(self.h, C.byref(c_), C.byref(h_), C.byref(w_))
        self.in_dims = (h_.value, w_.value, c_.value)

    def infer(self, x):
        out = _empty_like_kind(x, (max(self.output_size(), 1) if self.output_size() else 1 << 20,), np.float32)
        n = lib().acfun_model_infer(self.h, ptr(x), ptr(out))
        check()
        return out[:n]

    def infer_batch(self, x, out=None):
        n = x.shape[0]
        if out is None:
            size = self.output_size()
            if size <= 0:  # unknown until the first inference
                self.infer(x[0])
                size = self.output_size()
            out = _empty_like_kind(x, (n, size), np.float32)
        r = lib().acfun_model_infer_batch(self.h, n, ptr(x), ptr(out))
        check()
        if r <= 0:
            raise AcfunError("acfun_model_infer_batch returned 0")
        return out

    def set_int8(self, enable: bool = True) -> None:
        """Dense convolutions through the int8 router, one activation scale per image
        (acfun_model_set_int8; FC / pooling / softmax stay fp32)."""
        rc = lib().acfun_model_set_int8(self.h, 1 if enable else 0)
        check()
        if rc != 0:
            raise AcfunError(f"acfun_model_set_int8 failed ({rc})")

    def output_size(self) -> int:
        return lib().acfun_model_output_size(self.h)

    def close(self):
        if self.h:
            lib().acfun_model_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
