"""Parity metrics and tolerances shared by the tests.

The BASELINE contract: attention outputs within rel-L2 <= 1e-2 and
max-abs <= 2e-2 of the reference's fp32-accumulating path; Q8 dequantisation
(and the integer/byte helpers) bit-exact.
"""
from __future__ import annotations

import numpy as np

REL_L2 = 1e-2
MAX_ABS = 2e-2


def rel_l2(got, ref) -> float:
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    return float(np.linalg.norm(got - ref) / max(np.linalg.norm(ref), 1e-30))


def max_abs(got, ref) -> float:
    return float(np.max(np.abs(np.asarray(got, np.float64) - np.asarray(ref, np.float64))))


def assert_close(got, ref, rel=REL_L2, mabs=MAX_ABS, what=""):
    r, m = rel_l2(got, ref), max_abs(got, ref)
    assert np.all(np.isfinite(got)), f"{what}: non-finite output"
    assert r <= rel and m <= mabs, f"{what}: rel_l2={r:.3e} (<= {rel}) max_abs={m:.3e} (<= {mabs})"
    return r, m
