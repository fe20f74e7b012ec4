"""Shared helpers for the parity tests."""
import numpy as np


def rel_err(y, r) -> float:
    """max_i |y_i - r_i| / max(|r_i|, 1e-3 * ||r||_inf): elementwise relative error with a
    floor, so outputs near zero are judged against the vector's scale."""
    y = np.asarray(y, dtype=np.float64)
    r = np.asarray(r, dtype=np.float64)
    if r.size == 0:
        return 0.0
    floor = max(1e-3 * np.max(np.abs(r)), 1e-30)
    return float(np.max(np.abs(y - r) / np.maximum(np.abs(r), floor)))


def normwise(y, r) -> float:
    y = np.asarray(y, dtype=np.float64)
    r = np.asarray(r, dtype=np.float64)
    return float(np.max(np.abs(y - r)) / max(np.max(np.abs(r)), 1e-30))


def gpu_available() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


def parity(y, r, exact, tol=1e-3) -> bool:
    """GPU result y vs oracle r at rel_err <= tol; where the oracle's own fp32 rounding
    (long sequential sums) is what exceeds tol, an fp64 result arbitrates: y passes if
    it is no further from `exact` than the oracle is."""
    if rel_err(y, r) <= tol:
        return True
    return rel_err(y, exact) <= max(rel_err(r, exact), tol)
