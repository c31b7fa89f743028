"""CPU: the C-ABI library loads without a GPU and exports every symbol include/*.h declares."""
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    names = set()
    for h in ("acfun.h", "acfun_internal.h"):
        txt = open(os.path.join(ROOT, "include", "acfun", h)).read()
        txt = re.sub(r"/\*.*?\*/", "", txt, flags=re.S)
        for m in re.finditer(r"\b(acfun_[a-z0-9_]+)\s*\(", txt):
            names.add(m.group(1))
    return names


def test_headers_declare_the_reference_surface():
    names = declared_symbols()
    # the reference's public API (include/acfun/acfun.h:19-144) is fully present
    for n in ["acfun_set_threads", "acfun_backend", "acfun_backend_name", "acfun_autotune",
              "acfun_tune_status", "acfun_gemm", "acfun_gemm_epi", "acfun_gemm_bf16",
              "acfun_conv2d", "acfun_conv2d_relu", "acfun_conv2d_dw", "acfun_conv2d_g",
              "acfun_fc", "acfun_fc_relu", "acfun_relu", "acfun_relu6", "acfun_maxpool",
              "acfun_maxpool_relu", "acfun_softmax", "acfun_batchnorm",
              "acfun_quantize_weights", "acfun_conv2d_int8", "acfun_model_load",
              "acfun_model_destroy", "acfun_model_infer", "acfun_model_output_size",
              "acfun_model_input_dims", "acfun_gemm_int8", "acfun_gemm_int8_epi",
              "acfun_quantize_u8", "acfun_conv2d_int8_direct", "acfun_conv1x1_int8",
              "acfun_set_num_threads_runtime"]:
        assert n in names, n


def test_library_exports_every_declared_symbol():
    import acfun_b200
    if not os.path.exists(acfun_b200.LIB_PATH):
        acfun_b200.build()
    L = acfun_b200.lib()
    missing = [n for n in sorted(declared_symbols()) if not hasattr(L, n)]
    assert not missing, missing
    # every exported symbol has a ctypes signature in the host mirror
    assert not [n for n in declared_symbols() if n not in acfun_b200.SIGNATURES]


def test_host_mirror_fails_loudly_without_library(tmp_path, monkeypatch):
    import acfun_b200
    monkeypatch.setattr(acfun_b200, "_lib", None)
    monkeypatch.setattr(acfun_b200, "LIB_PATH", str(tmp_path / "missing.so"))
    with pytest.raises(FileNotFoundError):
        acfun_b200.lib()
