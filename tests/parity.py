"""Parity helpers shared by the GPU tests.

The CUDA path and the oracle implement the same exact-reduction semantics
(see oracle/bmo_oracle.c): fp32 operations in the reference's order,
reductions carried in double and rounded once, transcendentals evaluated in
double and rounded once.  Two double sums of the same terms in different
orders can still round to adjacent floats when they straddle a rounding
boundary (about 2^-21 per output for 256-term sums), so "near exact" allows
a rare 1-2 ULP difference.
"""
import numpy as np


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def ulp_diff(a, b):
    """Distance in units in the last place between float32 arrays."""
    a = np.ascontiguousarray(a, np.float32).view(np.int32).astype(np.int64)
    b = np.ascontiguousarray(b, np.float32).view(np.int32).astype(np.int64)
    a = np.where(a < 0, -(a & 0x7FFFFFFF), a)
    b = np.where(b < 0, -(b & 0x7FFFFFFF), b)
    return np.abs(a - b)


def assert_near_exact(got, want, max_ulp=2, max_frac=1e-3, what=""):
    got = np.asarray(got, np.float32).ravel()
    want = np.asarray(want, np.float32).ravel()
    assert got.shape == want.shape, (what, got.shape, want.shape)
    d = ulp_diff(got, want)
    frac = float((d > 0).mean()) if d.size else 0.0
    assert int(d.max(initial=0)) <= max_ulp and frac <= max_frac, \
        f"{what}: max ulp {int(d.max(initial=0))}, differing fraction {frac:.2e}, rel_l2 {rel_l2(got, want):.2e}"
