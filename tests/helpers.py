"""Shared helpers for the parity tests (seeded inputs and comparisons)."""
import numpy as np


def rng(seed):
    return np.random.default_rng(seed)


def uni(g, shape, lo, hi):
    return g.uniform(lo, hi, size=shape).astype(np.float32)


def max_rel(got, ref):
    """max|got-ref| / max|ref| (the reference gates scale by the output magnitude)."""
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    den = max(np.abs(ref).max(), 1e-30)
    return float(np.abs(got - ref).max() / den)


def assert_bits_equal(got, ref, what=""):
    got = np.ascontiguousarray(got)
    ref = np.ascontiguousarray(ref)
    assert got.shape == ref.shape, (what, got.shape, ref.shape)
    if got.dtype == np.float32:
        g, r = got.view(np.int32), ref.view(np.int32)
    else:
        g, r = got, ref
    bad = np.flatnonzero(g.ravel() != r.ravel())
    if bad.size:
        k = bad[0]
        raise AssertionError(f"{what}: {bad.size} of {g.size} elements differ; first at flat "
                             f"{k}: got {got.ravel()[k]!r} ref {ref.ravel()[k]!r}")


# tolerances written down once (north star: <=1e-4 max-rel fp32, <=1e-2 bf16)
TOL_F32 = 1e-4
TOL_BF16 = 1e-2
