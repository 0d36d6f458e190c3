"""Shared helpers for the parity tests."""
import numpy as np


def rel_err(a, ref):
    """Normwise max relative error max|a - ref| / max|ref| (the metric the
    tolerances below are stated in: 1e-2 for BF16/F16/Q8, 1e-4 for F32)."""
    a = np.asarray(a, np.float64)
    ref = np.asarray(ref, np.float64)
    den = np.abs(ref).max()
    return float(np.abs(a - ref).max() / (den if den > 0 else 1.0))


def to_np(t):
    return t.detach().float().cpu().numpy()
