"""Robust summaries of right-skewed timing samples.

Follows decodebench/stats.py:7-57: median with the 25th/75th percentiles, and a
percentile bootstrap of the difference of medians (seeded, chunked so that long
sample vectors never allocate n_resamples x n indices at once).
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Sequence as _Seq

import numpy as np


@dataclass(frozen=True)
class Summary:
    median: float
    p25: float
    p75: float
    n: int

    @property
    def iqr(self) -> float:
        return self.p75 - self.p25


def _as_samples(x, what: str) -> np.ndarray:
    a = np.asarray(x, dtype=np.float64)
    if a.ndim != 1:
        raise ValueError(f"{what} samples must be one-dimensional")
    if a.size and not np.isfinite(a).all():
        raise ValueError(f"{what} samples must all be finite")
    return a


def summarize(samples: _Seq[float]) -> Summary:
    a = np.asarray(samples, dtype=np.float64)
    if a.size == 0:
        raise ValueError("summarize() requires at least one sample")
    a = _as_samples(a, "summarize()")
    p25, med, p75 = np.percentile(a, [25.0, 50.0, 75.0])
    return Summary(median=float(med), p25=float(p25), p75=float(p75), n=int(a.size))


def bootstrap_diff_ci(a, b, n_resamples: int = 10000, ci: float = 0.95,
                      seed: int = 42) -> tuple[float, float, float]:
    """Percentile-bootstrap CI of median(a) - median(b): returns (lo, hi, point)."""
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    if a.size == 0 or b.size == 0:
        raise ValueError("bootstrap_diff_ci() requires non-empty samples")
    a = _as_samples(a, "bootstrap_diff_ci()")
    b = _as_samples(b, "bootstrap_diff_ci()")
    if n_resamples <= 0:
        raise ValueError("n_resamples must be positive")
    if not (0.0 < ci < 1.0):
        raise ValueError("ci must be between 0 and 1")
    rng = np.random.default_rng(seed)
    diffs = np.empty(n_resamples)
    rows = max(1, 1_000_000 // max(a.size, b.size))
    done = 0
    while done < n_resamples:
        m = min(rows, n_resamples - done)
        ia = rng.integers(0, a.size, size=(m, a.size))
        ib = rng.integers(0, b.size, size=(m, b.size))
        diffs[done:done + m] = np.median(a[ia], axis=1) - np.median(b[ib], axis=1)
        done += m
    tail = 0.5 * (1.0 - ci)
    lo, hi = np.quantile(diffs, [tail, 1.0 - tail])
    return float(lo), float(hi), float(np.median(a) - np.median(b))
