"""GPU parity: the tcgen05 GEMM family through the C ABI against the oracle and the golden
vectors (bit-exact for int8, max-rel tolerance for float)."""
import glob
import os

import numpy as np
import pytest

from helpers import TOL_BF16, TOL_F32, assert_bits_equal, max_rel

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def load(name):
    return dict(np.load(os.path.join(GOLD, name + ".npz")))


def torch_dev(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


# the reference's own gates (benchmark.cpp:53-77, :930-962) plus tcgen05 tile edges
INT8_SHAPES = [(63, 63, 63), (100, 100, 100), (255, 255, 255), (512, 512, 512), (1023, 1023, 1023),
               (64, 64, 64), (512, 17, 64), (63, 512, 33), (127, 129, 63), (1023, 4, 7),
               (128, 256, 128), (129, 257, 129), (1, 1, 1), (300, 640, 2000), (2048, 384, 4096),
               (2560, 2048, 640), (2600, 2000, 200)]   # > 148 tiles: more than one wave, ragged


def rand_u8s8(g, M, N, K):
    return (g.integers(0, 256, (M, K), dtype=np.uint8), g.integers(-128, 128, (K, N), dtype=np.int8))


@pytest.mark.parametrize("M,N,K", INT8_SHAPES)
def test_gemm_int8_exact(acf, orc, M, N, K):
    g = np.random.default_rng(M * 7919 + N * 31 + K)
    A, B = rand_u8s8(g, M, N, K)
    ref = np.empty((M, N), np.int32)
    orc.oracle().orc_gemm_int8(M, N, K, A, B, ref)
    assert_bits_equal(acf.gemm_int8(A, B), ref, f"gemm_int8 {M}x{N}x{K} host")


@pytest.mark.parametrize("M,N,K,act", [(64, 64, 64, 1), (100, 100, 100, 1), (255, 255, 255, 0),
                                       (512, 17, 64, 1), (63, 512, 33, 1), (127, 129, 63, 0),
                                       (1023, 4, 7, 1), (700, 300, 1111, 1), (2560, 2048, 384, 1)])
def test_gemm_int8_epi_exact(acf, orc, M, N, K, act):
    g = np.random.default_rng(K)
    A, B = rand_u8s8(g, M, N, K)
    al = g.uniform(1e-4, 1e-2, N).astype(np.float32)
    be = g.uniform(-20, 20, N).astype(np.float32)
    ref = np.empty((M, N), np.float32)
    orc.oracle().orc_gemm_int8_epi(M, N, K, A, B, ref, al, be, act)
    assert_bits_equal(acf.gemm_int8_epi(A, B, al, be, act), ref, f"epi {M}x{N}x{K}")


def test_gemm_int8_device_pointers(acf, orc):
    M, N, K = 384, 512, 640
    g = np.random.default_rng(5)
    A, B = rand_u8s8(g, M, N, K)
    ref = np.empty((M, N), np.int32)
    orc.oracle().orc_gemm_int8(M, N, K, A, B, ref)
    out = acf.gemm_int8(torch_dev(A), torch_dev(B))
    acf.synchronize()
    assert_bits_equal(out.cpu().numpy(), ref, "device pointers")


@pytest.mark.parametrize("name", sorted(os.path.basename(p)[:-4] for p in glob.glob(os.path.join(GOLD, "gemm_int8_*.npz"))))
def test_gemm_int8_golden(acf, name):
    d = load(name)
    if "_epi_" in name:
        got = acf.gemm_int8_epi(d["A"], d["B"], d["alpha"], d["beta"], int(d["act"]))
    else:
        got = acf.gemm_int8(d["A"], d["B"])
    assert_bits_equal(got, d["C"], name)


@pytest.mark.parametrize("act", [0, 1])
def test_gemm_s8_requant_golden(acf, act):
    d = load(f"gemm_s8_requant_a{act}")
    got = acf.gemm_s8_requant(d["A"], d["B"], d["bias"], d["scale"], act)
    assert_bits_equal(got, d["C"], "s8 requant")


@pytest.mark.parametrize("M,N,K", [(4096, 4096, 4096)])
def test_gemm_s8_requant_full_size_sampled(acf, orc, M, N, K):
    """BASELINE cfg2 at full size: every sampled row is bit-exact against the oracle."""
    g = np.random.default_rng(2)
    A = g.integers(-127, 128, (M, K), dtype=np.int8)
    B = g.integers(-127, 128, (K, N), dtype=np.int8)
    bias = g.integers(-1000, 1001, N, dtype=np.int32)
    scale = g.uniform(1e-3, 1e-2, N).astype(np.float32)
    got = acf.gemm_s8_requant(A, B, bias, scale, 1)
    rows = np.sort(g.choice(M, 24, replace=False))
    rows = np.concatenate([[0, 127, 128, M - 1], rows])
    ref = np.empty((rows.size, N), np.int8)
    orc.oracle().orc_gemm_s8_requant(rows.size, N, K, np.ascontiguousarray(A[rows]), B,
                                     bias.ctypes.data, scale, ref, 1)
    assert_bits_equal(got[rows], ref, "requant 4096^3 sampled rows")


@pytest.mark.parametrize("M,N,K", [(64, 64, 64), (100, 100, 100), (255, 255, 255), (1024, 1024, 1024),
                                   (33, 47, 129), (300, 24, 144), (1, 1000, 4096), (512, 17, 64),
                                   (10240, 300, 200),    # 256-column tiles, ragged N and K
                                   (40000, 100, 136),    # two 128-row sub-tiles per CTA, N 128
                                   (37856, 40, 72),      # the same at N 64; last sub-tile empty
                                   (300, 520, 5000),     # split-K over 14 K ranges, K tail
                                   (256, 4096, 25088)])  # VGG FC1 shape (split-K)
def test_gemm_f32_tolerance(acf, orc, M, N, K):
    g = np.random.default_rng(M + N + K)
    A = g.uniform(-1, 1, (M, K)).astype(np.float32)
    B = g.uniform(-1, 1, (K, N)).astype(np.float32)
    bias = g.uniform(-1, 1, N).astype(np.float32)
    ref = np.empty((M, N), np.float32)
    orc.oracle().orc_gemm_f32(M, N, K, A, B, ref, bias.ctypes.data, 1)
    got = acf.gemm(A, B, bias, 1)
    assert max_rel(got, ref) < TOL_F32, max_rel(got, ref)


@pytest.mark.parametrize("M,N,K", [(64, 64, 64), (33, 47, 129), (1024, 1024, 1024), (200, 520, 300),
                                   (2560, 2048, 256),    # 160 tiles: a second, partial wave
                                   (2200, 2450, 333)])   # ragged M / N / K
def test_gemm_bf16_tolerance(acf, orc, M, N, K):
    g = np.random.default_rng(M * N + K)
    A = g.uniform(-1, 1, (M, K)).astype(np.float32)
    B = g.uniform(-1, 1, (K, N)).astype(np.float32)
    ref = np.empty((M, N), np.float32)
    orc.oracle().orc_gemm_bf16(M, N, K, A, B, ref)
    got = acf.gemm_bf16(A, B)
    # same bf16 operands, fp32 accumulation: only the summation order differs
    assert max_rel(got, ref) < 1e-4
    exact = A.astype(np.float64) @ B.astype(np.float64)
    assert max_rel(got, exact) < TOL_BF16


@pytest.mark.parametrize("M,N,K", [(4096, 4096, 4096),   # BASELINE cfg2 bf16 shape
                                   (3100, 3300, 1100)])  # ragged M / N / K
def test_gemm_bf16_2sm_sampled(acf, orc, M, N, K):
    """bf16 GEMMs with two or more waves of 256 x 256 tiles and K >= 1024 run on the 2-SM kernel:
    sampled rows (the first / last of a 256-row pair tile and the last row among them) against
    the oracle's bf16 GEMM."""
    g = np.random.default_rng(M + N + K)
    A = g.uniform(-1, 1, (M, K)).astype(np.float32)
    B = g.uniform(-1, 1, (K, N)).astype(np.float32)
    got = acf.gemm_bf16(A, B)
    rows = np.unique(np.concatenate([[0, 127, 128, 255, 256, M - 1], g.choice(M, 10, replace=False)]))
    ref = np.empty((rows.size, N), np.float32)
    orc.oracle().orc_gemm_bf16(rows.size, N, K, np.ascontiguousarray(A[rows]), B, ref)
    assert max_rel(got[rows], ref) < 1e-4


@pytest.mark.parametrize("name", sorted(os.path.basename(p)[:-4] for p in glob.glob(os.path.join(GOLD, "gemm_f32_*.npz"))))
def test_gemm_float_golden(acf, name):
    d = load(name)
    assert max_rel(acf.gemm(d["A"], d["B"], d["bias"], 1), d["C_epi_relu"]) < TOL_F32
    assert max_rel(acf.gemm_bf16(d["A"], d["B"]), d["C_bf16"]) < TOL_BF16


def test_gemm_empty_and_bad_shapes_are_silent(acf):
    L = acf.lib()
    C = np.full((2, 2), 7, np.int32)
    L.acfun_gemm_int8(0, 2, 2, None, None, acf.ptr(C))       # M<=0: returns, output untouched
    L.acfun_gemm_int8(2, 2, -1, None, None, acf.ptr(C))
    acf.check()
    assert (C == 7).all()


@pytest.mark.parametrize("M,N,K", [(1100, 96, 4100), (2047, 200, 2304)])
def test_host_buffer_row_pipeline_exact(acf, orc, M, N, K):
    """Host A and C of >= 4 MB take the row-chunked path (H2D / GEMM / D2H overlapped on
    three streams; ragged last chunk, A pitch not a multiple of 16): bit-identical to the
    oracle and to the device-pointer call."""
    g = np.random.default_rng(M + K)
    A, B = rand_u8s8(g, M, N, K)
    ref = np.empty((M, N), np.int32)
    orc.oracle().orc_gemm_int8(M, N, K, A, B, ref)
    assert_bits_equal(acf.gemm_int8(A, B), ref, f"gemm_int8 pipelined {M}x{N}x{K}")
    al = g.uniform(1e-4, 1e-2, N).astype(np.float32)
    be = g.uniform(-20, 20, N).astype(np.float32)
    ref_e = np.empty((M, N), np.float32)
    orc.oracle().orc_gemm_int8_epi(M, N, K, A, B, ref_e, al, be, 1)
    assert_bits_equal(acf.gemm_int8_epi(A, B, al, be, 1), ref_e, "epi pipelined")
    As = (A.astype(np.int16) - 128).astype(np.int8)
    bias = g.integers(-1000, 1001, N, dtype=np.int32)
    scale = g.uniform(1e-4, 1e-3, N).astype(np.float32)
    ref_q = np.empty((M, N), np.int8)
    orc.oracle().orc_gemm_s8_requant(M, N, K, As, B, bias.ctypes.data, scale, ref_q, 0)
    got_host = acf.gemm_s8_requant(As, B, bias, scale, 0)
    assert_bits_equal(got_host, ref_q, "s8 requant pipelined")
    got_dev = acf.gemm_s8_requant(torch_dev(As), torch_dev(B), torch_dev(bias), torch_dev(scale), 0)
    acf.synchronize()
    assert_bits_equal(got_dev.cpu().numpy(), got_host, "s8 requant device vs host path")
    # mixed: host A, device C -> single-launch path
    import torch
    Cd = torch.empty((M, N), dtype=torch.int8, device="cuda")
    Bd = torch_dev(B)
    acf.lib().acfun_gemm_s8_requant(M, N, K, acf.ptr(As), Bd.data_ptr(), acf.ptr(bias), acf.ptr(scale),
                                    Cd.data_ptr(), 0)
    acf.synchronize()
    acf.check()
    assert_bits_equal(Cd.cpu().numpy(), ref_q, "s8 requant host A / device C")


def test_s8_requant_two_waves_device(acf, orc):
    """160 tiles of 128x256 on 148 persistent CTAs (a second, partial wave) through the
    device-pointer path; every row of the last 3 row blocks is compared."""
    M, N, K = 2560, 2048, 1000
    g = np.random.default_rng(31)
    A = g.integers(-127, 128, (M, K), dtype=np.int8)
    B = g.integers(-127, 128, (K, N), dtype=np.int8)
    bias = g.integers(-1000, 1001, N, dtype=np.int32)
    scale = g.uniform(1e-4, 1e-3, N).astype(np.float32)
    got = acf.gemm_s8_requant(torch_dev(A), torch_dev(B), torch_dev(bias), torch_dev(scale), 1)
    acf.synchronize()
    got = got.cpu().numpy()
    rows = np.arange(M - 384, M)            # the second wave's tiles cover rows 2304..2559
    rows = np.concatenate([[0, 1, 1000], rows])
    ref = np.empty((rows.size, N), np.int8)
    orc.oracle().orc_gemm_s8_requant(rows.size, N, K, np.ascontiguousarray(A[rows]), B, bias.ctypes.data,
                                     scale, ref, 1)
    assert_bits_equal(got[rows], ref, "requant two waves")


@pytest.mark.parametrize("M,N,K", [(2432, 2000, 700),     # 152 tiles: 4 left, in two halves
                                   (2560, 2048, 1000)])  # 160 tiles: 12 left, in two halves
def test_int8_last_wave_column_parts_exact(acf, orc, M, N, K):
    """The persistent walk's last, partial wave of 128x256 tiles runs as 128-column parts on
    more SMs (ragged N in the last part): bit-exact against the oracle on the last row
    blocks, through host and device pointers."""
    g = np.random.default_rng(M + N + K)
    A, B = rand_u8s8(g, M, N, K)
    rows = np.arange(M - 256, M)
    ref = np.empty((rows.size, N), np.int32)
    orc.oracle().orc_gemm_int8(rows.size, N, K, np.ascontiguousarray(A[rows]), B, ref)
    assert_bits_equal(acf.gemm_int8(A, B)[rows], ref, f"last wave {M}x{N}x{K} host")
    out = acf.gemm_int8(torch_dev(A), torch_dev(B))
    acf.synchronize()
    assert_bits_equal(out.cpu().numpy()[rows], ref, f"last wave {M}x{N}x{K} device")


@pytest.mark.parametrize("M,N,K", [(2560, 2048, 512), (4096, 4096, 1024)])
def test_float_last_wave_column_parts(acf, orc, M, N, K):
    """bf16 and fp32 (3xBF16) GEMMs whose last wave is cut into 64- or 128-column parts:
    within tolerance of the oracle on the last row blocks."""
    g = np.random.default_rng(M + K)
    A = g.uniform(-1, 1, (M, K)).astype(np.float32)
    B = g.uniform(-1, 1, (K, N)).astype(np.float32)
    bias = g.uniform(-1, 1, N).astype(np.float32)
    rows = np.arange(M - 256, M)
    Ar = np.ascontiguousarray(A[rows])
    ref = np.empty((rows.size, N), np.float32)
    orc.oracle().orc_gemm_f32(rows.size, N, K, Ar, B, ref, bias.ctypes.data, 1)
    got = acf.gemm(A, B, bias, 1)[rows]
    assert max_rel(got, ref) < TOL_F32, f"fp32 last wave {M}x{N}x{K}: {max_rel(got, ref)}"
    ref16 = np.empty((rows.size, N), np.float32)
    orc.oracle().orc_gemm_bf16(rows.size, N, K, Ar, B, ref16)
    got16 = acf.gemm_bf16(A, B)[rows]
    assert max_rel(got16, ref16) < 1e-4, f"bf16 last wave {M}x{N}x{K}: {max_rel(got16, ref16)}"


def test_int8_full_size_all_elements_vs_fp64(acf):
    """BASELINE cfg2 shape, u8 x s8 -> s32: every element (444 whole 128x256 tiles, then the
    68 tiles of the last wave as 136 column halves) equals torch's float64 product on the
    GPU, exact here because every partial sum is an integer below 2^53."""
    import torch
    M = N = K = 4096
    gen = torch.Generator(device="cuda").manual_seed(7)
    A = torch.randint(0, 256, (M, K), dtype=torch.uint8, device="cuda", generator=gen)
    B = torch.randint(-128, 128, (K, N), dtype=torch.int8, device="cuda", generator=gen)
    out = acf.gemm_int8(A, B)
    acf.synchronize()
    ref = (A.double() @ B.double()).to(torch.int32)
    bad = int((out != ref).sum().item())
    assert bad == 0, f"{bad} of {M * N} elements differ"


_SPLIT_OFF_CHILD = r"""
import sys, numpy as np
import acfun_b200 as acf
M, N, K = 2560, 2048, 512
g = np.random.default_rng(11)
A = g.uniform(-1, 1, (M, K)).astype(np.float32)
B = g.uniform(-1, 1, (K, N)).astype(np.float32)
Ai, Bi = g.integers(0, 256, (M, K), dtype=np.uint8), g.integers(-128, 128, (K, N), dtype=np.int8)
np.savez(sys.argv[1], f32=acf.gemm(A, B), bf16=acf.gemm_bf16(A, B), i8=acf.gemm_int8(Ai, Bi))
"""


def test_last_wave_column_parts_same_bits_as_whole_tiles(acf, tmp_path):
    """160 tiles on 148 SMs: the 12 last-wave tiles run as column parts by default and as
    whole tiles with ACFUN_TAIL_SPLIT=0 (a child process); fp32 (3xBF16), bf16 and int8
    results are bit-identical, because each output column keeps its whole K loop."""
    import subprocess
    import sys
    out = tmp_path / "whole.npz"
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    env = dict(os.environ, ACFUN_TAIL_SPLIT="0", PYTHONPATH=root)
    subprocess.run([sys.executable, "-c", _SPLIT_OFF_CHILD, str(out)], env=env, cwd=root,
                   check=True, timeout=300)
    whole = np.load(out)
    M, N, K = 2560, 2048, 512
    g = np.random.default_rng(11)
    A = g.uniform(-1, 1, (M, K)).astype(np.float32)
    B = g.uniform(-1, 1, (K, N)).astype(np.float32)
    Ai, Bi = g.integers(0, 256, (M, K), dtype=np.uint8), g.integers(-128, 128, (K, N), dtype=np.int8)
    assert_bits_equal(acf.gemm(A, B), whole["f32"], "fp32 column parts vs whole tiles")
    assert_bits_equal(acf.gemm_bf16(A, B), whole["bf16"], "bf16 column parts vs whole tiles")
    assert_bits_equal(acf.gemm_int8(Ai, Bi), whole["i8"], "int8 column parts vs whole tiles")


def _requant_ref_torch(A, B, bias, scale, act):
    """sat_s8(rne(relu((float)(acc + bias) * scale))) for every element, on the GPU: the integer
    product in float64 (exact: every partial sum is an integer below 2^53), then the fp32
    multiply and round-half-even the kernel's epilogue performs."""
    import torch
    acc = (A.double() @ B.double()).to(torch.int64) + bias.to(torch.int64)
    v = acc.to(torch.int32).to(torch.float32) * scale
    if act:
        v = torch.clamp(v, min=0.0)
    return torch.clamp(torch.round(v), -128, 127).to(torch.int8)


@pytest.mark.parametrize("M,N,K,act", [(2304, 2304, 256, 1), (2200, 2450, 333, 0), (4096, 4096, 4096, 1)])
def test_s8_requant_2sm_every_element(acf, M, N, K, act):
    """The 2-SM path (tcgen05.mma.cta_group::2, 256 x 256 tiles on CTA pairs; taken when the
    GEMM has enough such tiles) against an every-element reference: exact multiples, ragged M /
    N / K (TMA zero fill past the edges, padded operand copies), and the BASELINE cfg2 shape."""
    import torch
    gen = torch.Generator(device="cuda").manual_seed(M + N + K)
    A = torch.randint(-127, 128, (M, K), dtype=torch.int8, device="cuda", generator=gen)
    B = torch.randint(-127, 128, (K, N), dtype=torch.int8, device="cuda", generator=gen)
    bias = torch.randint(-1000, 1001, (N,), dtype=torch.int32, device="cuda", generator=gen)
    scale = (torch.rand(N, device="cuda", generator=gen) * 9e-3 + 1e-3).to(torch.float32)
    out = acf.gemm_s8_requant(A, B, bias, scale, act)
    acf.synchronize()
    ref = _requant_ref_torch(A, B, bias, scale, act)
    bad = int((out != ref).sum().item())
    assert bad == 0, f"{bad} of {M * N} elements differ"
