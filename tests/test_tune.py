"""The tile table behind acfun_autotune / acfun_tune_status (tune.cu): the cache format is
read without a GPU; the GPU test measures a table and checks results through it."""
import os
import subprocess
import sys

import numpy as np
import pytest

from helpers import TOL_F32, assert_bits_equal, max_rel

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def status_in_fresh_process(env):
    code = ("import acfun_b200 as a; import sys; "
            "sys.stdout.write(a.lib().acfun_tune_status().decode())")
    r = subprocess.run([sys.executable, "-c", code], cwd=ROOT, env=env, capture_output=True,
                       text=True, timeout=300)
    assert r.returncode == 0, r.stderr
    return r.stdout


def test_tile_table_file_is_loaded(tmp_path):
    p = tmp_path / "table.txt"
    p.write_text("# acfun tile table v1 (family lgM lgN lgK variant us)\n"
                 "0 10 10 10 3 21.5\n"
                 "2 12 12 12 1 57.0\n"
                 "1 12 12 12 9 1.0\n"        # variant out of range: ignored
                 "garbage line\n")
    env = dict(os.environ, ACFUN_TUNE_CACHE=str(p))
    s = status_in_fresh_process(env)
    assert s.startswith("tuned: 2 shape classes from "), s


def test_missing_or_headerless_table_means_heuristics(tmp_path):
    p = tmp_path / "none.txt"
    env = dict(os.environ, ACFUN_TUNE_CACHE=str(p))
    assert status_in_fresh_process(env).startswith("static heuristics"), "no file"
    p.write_text("0 10 10 10 3 21.5\n")
    assert status_in_fresh_process(env).startswith("static heuristics"), "no header"


@pytest.mark.gpu
def test_autotune_measures_a_table_and_results_hold(acf, orc, tmp_path, monkeypatch):
    path = tmp_path / "tt.txt"
    monkeypatch.setenv("ACFUN_TUNE_CACHE", str(path))
    L = acf.lib()
    L.acfun_autotune()
    acf.check()
    s = L.acfun_tune_status().decode()
    assert s.startswith("tuned: ") and str(path) in s, s
    lines = path.read_text().splitlines()
    assert lines[0].startswith("# acfun tile table v1") and len(lines) > 10
    for ln in lines[1:]:
        fam, lm, lnn, lk, v, us = ln.split()
        assert 0 <= int(fam) <= 2 and int(v) >= 0 and float(us) > 0
    g = np.random.default_rng(5)
    for (M, N, K) in [(1024, 1024, 1024), (256, 4096, 4096)]:   # tuned fp32 classes
        A = g.uniform(-1, 1, (M, K)).astype(np.float32)
        B = g.uniform(-1, 1, (K, N)).astype(np.float32)
        bias = g.uniform(-1, 1, N).astype(np.float32)
        ref = np.empty((M, N), np.float32)
        orc.oracle().orc_gemm_f32(M, N, K, A, B, ref, bias.ctypes.data, 1)
        assert max_rel(acf.gemm(A, B, bias, 1), ref) < TOL_F32, (M, N, K)
    M = N = K = 1024                                               # tuned int8 class
    A = g.integers(0, 256, (M, K), dtype=np.uint8)
    Bq = g.integers(-128, 128, (K, N), dtype=np.int8)
    ref = np.empty((M, N), np.int32)
    orc.oracle().orc_gemm_int8(M, N, K, A, Bq, ref)
    assert_bits_equal(acf.gemm_int8(A, Bq), ref, "int8 through the tile table")
