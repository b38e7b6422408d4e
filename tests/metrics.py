"""Accuracy metrics of the reference's test suite (``mamba3_pallas/tests.py:60-96``)."""

import math

import numpy as np


def _np(x):
    if hasattr(x, "detach"):
        x = x.detach().float().cpu().double().numpy() if x.dtype.is_floating_point else x.cpu().numpy()
    return np.asarray(x, np.float64)


def rel_error(got, ref, *, mag_floor=1e-2, pct=95.0, angle=False):
    """95th-percentile elementwise relative error over entries with ``|ref| >= mag_floor``;
    circular absolute error in radians when ``angle`` (``tests.py:60-88``)."""
    g, r = _np(got), _np(ref)
    if g.shape != r.shape:
        raise AssertionError(f"shape mismatch: {g.shape} vs {r.shape}")
    if angle:
        d = np.abs((g - r + math.pi) % (2 * math.pi) - math.pi)
        return float(np.percentile(d, pct))
    mask = np.abs(r) >= mag_floor
    if not mask.any():
        return 0.0
    return float(np.percentile(np.abs(g - r)[mask] / np.abs(r)[mask], pct))


def max_rel(got, ref):
    """Max abs error normalised by the reference's largest magnitude (``tests.py:91-96``)."""
    g, r = _np(got), _np(ref)
    return float(np.max(np.abs(g - r)) / max(float(np.max(np.abs(r))), 1e-30))
