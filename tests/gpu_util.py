"""Shared helpers for the -m gpu parity tests."""
import numpy as np


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def n_mismatch(a, b) -> int:
    return int(np.count_nonzero(bits(a) != bits(b)))


def abs_err_scaled(a, b, scale=None) -> float:
    """kernels/ops_ref.ts:206 absErrScaled (scale defaults to amax(b))."""
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    s = float(np.abs(b).max()) if scale is None else scale
    return float(np.abs(a - b).max() / s) if a.size else 0.0


def rel_err(a, b, floor=1e-6) -> float:
    """kernels/ops_ref.ts:185 relErr."""
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.max(np.abs(a - b) / np.maximum(floor, np.abs(b)))) if a.size else 0.0
