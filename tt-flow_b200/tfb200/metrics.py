"""Parity metrics for the fused path.

``compute_metrics`` mirrors the reference harness's metric set
(tensixflow ``python/tensixflow/harness.py:164-181``: PCC, cosine, max/mean
absolute and relative error, accumulated in float64). ``parity`` applies this
backend's bar: after dividing both outputs by the RMS of the fp32 golden, the
maximum absolute difference is at most 2e-2, and the PCC is at least 0.9999.
"""

from __future__ import annotations

import numpy as np

MAX_ABS_UNIT_RMS = 2e-2
PCC_MIN = 0.9999

__all__ = ["compute_metrics", "parity", "MAX_ABS_UNIT_RMS", "PCC_MIN"]


def compute_metrics(got, golden) -> dict:
    s = np.asarray(got, dtype=np.float64).ravel()
    g = np.asarray(golden, dtype=np.float64).ravel()
    d = np.abs(s - g)
    rel = d / np.maximum(np.abs(g), 1e-6)
    denom = np.linalg.norm(s) * np.linalg.norm(g)
    return {
        "pcc": float(np.corrcoef(s, g)[0, 1]) if s.size > 1 else float("nan"),
        "cosine": float(np.dot(s, g) / denom) if denom > 0 else float("nan"),
        "max_abs_diff": float(d.max()) if d.size else 0.0,
        "mean_abs_err": float(d.mean()) if d.size else 0.0,
        "mean_rel_err": float(rel.mean()) if rel.size else 0.0,
        "max_rel_err": float(rel.max()) if rel.size else 0.0,
    }


def parity(got, golden, max_abs: float = MAX_ABS_UNIT_RMS, pcc_min: float = PCC_MIN) -> dict:
    """Metrics plus the pass/fail verdict of the parity bar."""
    m = compute_metrics(got, golden)
    g = np.asarray(golden, dtype=np.float64)
    rms = float(np.sqrt(np.mean(g * g))) if g.size else 0.0
    m["golden_rms"] = rms
    m["max_abs_unit_rms"] = m["max_abs_diff"] / rms if rms > 0 else float("inf")
    m["finite"] = bool(np.all(np.isfinite(np.asarray(got, dtype=np.float64))))
    m["ok"] = bool(m["finite"] and m["max_abs_unit_rms"] <= max_abs and m["pcc"] >= pcc_min)
    return m
