"""Shared helpers of the test suite: seeded inputs in the reference layouts and the error metrics."""
import numpy as np

F32_TOL = 1e-4   # max|got-ref| / max|ref|, f32 I/O
HALF_TOL = 3e-3  # max|got-ref| / max|ref|, f16/bf16 I/O against the f32 oracle on the same rounded inputs


def make_inputs(h, w, bh, hd, seed, table_std=1.0):
    """q [bh,n,hd], kt [bh,hd,n], v [bh,n,hd] ~ N(0,1); table [(2h-1)+(2w-1), hd] ~ N(0, table_std)."""
    n = h * w
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((bh, n, hd), dtype=np.float32)
    kt = rng.standard_normal((bh, hd, n), dtype=np.float32)
    v = rng.standard_normal((bh, n, hd), dtype=np.float32)
    table = (rng.standard_normal(((2 * h - 1) + (2 * w - 1), hd), dtype=np.float32) * table_std).astype(np.float32)
    return q, kt, v, table


def rel_max_err(got, ref):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    return float(np.abs(got - ref).max() / max(np.abs(ref).max(), 1e-30))


def mean_rel_err(got, ref):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    return float(np.abs(got - ref).mean() / max(np.abs(ref).mean(), 1e-30))
