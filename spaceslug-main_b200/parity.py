"""Parity metrics for the int4 path.

``compare_float_arrays`` keeps the reference's definition and report shape
(python/spaceslug/parity.py:6-16; the same criterion as
vulkan-runtime/tests/test_q4gemm.cpp:376-390): per element
rel = |actual - expected| / max(1, |expected|), pass when max rel <= tolerance.

``gemm_error_report`` adds the tolerances this build is held to:
  * max-abs error <= 1e-3 * ||x||_inf * ||W||_inf * sqrt(K) (16-bit tensor-core
    prefill path),
  * normwise relative error ||Y - Yref||_F / ||Yref||_F <= 2e-3 (prefill path),
  * elementwise relative error (the reference criterion) <= 1e-4 for the fp32
    GEMV path.
"""
from __future__ import annotations

import math

import numpy as np


def compare_float_arrays(actual, expected, *, tolerance: float = 1e-3) -> dict:
    a = np.asarray(actual, np.float64).reshape(-1)
    e = np.asarray(expected, np.float64).reshape(-1)
    if a.shape != e.shape:
        raise ValueError("parity arrays must have equal length")
    err = np.abs(a - e) / np.maximum(1.0, np.abs(e))
    bad = np.flatnonzero(~(err <= tolerance))
    return {
        "status": "pass" if bad.size == 0 else "fail",
        "tolerance": tolerance,
        "max_relative_error": float(np.nanmax(err)) if err.size else 0.0,
        "first_bad_index": int(bad[0]) if bad.size else None,
        "count": int(a.size),
    }


GEMV_REL_TOL = 1e-4
GEMM_ABS_FACTOR = 1e-3
GEMM_NORM_REL_TOL = 2e-3


def gemm_error_report(y, y_ref, x, w_absmax: float, k: int) -> dict:
    """Error metrics of an int4 GEMM output against the double oracle."""
    x_inf = float(np.max(np.abs(x))) if np.size(x) else 0.0
    return gemm_error_report_bound(y, y_ref, x_inf, w_absmax, k)


def gemm_error_report_bound(y, y_ref, x_inf: float, w_absmax: float, k: int) -> dict:
    """gemm_error_report with ||x||_inf given (y may hold sampled rows of Y)."""
    y = np.asarray(y, np.float64)
    r = np.asarray(y_ref, np.float64)
    diff = y - r
    max_abs = float(np.max(np.abs(diff))) if diff.size else 0.0
    abs_bound = GEMM_ABS_FACTOR * x_inf * w_absmax * math.sqrt(k)
    ref_norm = float(np.linalg.norm(r))
    norm_rel = float(np.linalg.norm(diff)) / ref_norm if ref_norm > 0 else float(np.linalg.norm(diff))
    elem_rel = float(np.max(np.abs(diff) / np.maximum(1.0, np.abs(r)))) if diff.size else 0.0
    return {
        "max_abs": max_abs,
        "abs_bound": abs_bound,
        "norm_rel": norm_rel,
        "elem_rel": elem_rel,
        "finite": bool(np.all(np.isfinite(y))),
    }


def gemm_passes(rep: dict) -> bool:
    """The tensor-core GEMM bars: finite, max-abs within the bound, normwise <= 2e-3."""
    return bool(rep["finite"] and rep["max_abs"] <= rep["abs_bound"] and rep["norm_rel"] <= GEMM_NORM_REL_TOL)
