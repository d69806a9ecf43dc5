"""Shared comparison helpers for the parity tests."""
import numpy as np


def rel_err(actual, expected):
    """max |actual - expected| / max |expected| (normwise max relative error)."""
    a = np.asarray(actual, dtype=np.float64)
    e = np.asarray(expected, dtype=np.float64)
    denom = max(float(np.abs(e).max()), 1e-30)
    return float(np.abs(a - e).max()) / denom


def rel_l2(actual, expected):
    a = np.asarray(actual, dtype=np.float64).ravel()
    e = np.asarray(expected, dtype=np.float64).ravel()
    return float(np.linalg.norm(a - e) / max(np.linalg.norm(e), 1e-30))
