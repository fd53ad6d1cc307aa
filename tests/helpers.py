"""Shared helpers of the GPU parity tests (device buffers via torch, comparisons)."""
from __future__ import annotations

import numpy as np


def dev(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def rel_rms(a, b) -> float:
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.sqrt(((a - b) ** 2).mean() / max((b ** 2).mean(), 1e-30)))


def max_abs(a, b) -> float:
    return float(np.abs(np.asarray(a, np.float64) - np.asarray(b, np.float64)).max())


# The decoder-level tolerance: attention outputs and logits within 2e-2 max-abs and
# 1e-3 relative RMS of the oracle run with the same arithmetic (exact GEMM mode).
TOL_MAX_ABS = 2e-2
TOL_REL_RMS = 1e-3


def assert_close(a, b, max_abs_tol=TOL_MAX_ABS, rel_rms_tol=TOL_REL_RMS, what=""):
    ma, rr = max_abs(a, b), rel_rms(a, b)
    assert ma <= max_abs_tol and rr <= rel_rms_tol, f"{what}: max-abs {ma:.3g} (tol {max_abs_tol}), rel-rms {rr:.3g} (tol {rel_rms_tol})"
