"""Sample qualification and α/β fitting of measured components.

Qualification keeps only samples produced by the native executor (never a
simulation or a unit fixture), drops launches before the first stable round
(coefficient of variation below ``max_cv``), and requires the probe's
numerical check to have passed.  ``fit_curve`` fits ``t = α + β·bytes`` by
least squares; if the relative error exceeds the limit it splits the size
range into piecewise segments, each of which needs at least two payloads of
its own (reference: vericcl/verification/online/component_fitting.py:26-82,
cost_fitting.py:58).
"""
from __future__ import annotations

import statistics
from dataclasses import dataclass

import numpy as np

from vericcl_b200.errors import RuntimeFailure

NATIVE_SOURCES = frozenset({"native_interpreter"})


@dataclass(frozen=True)
class Sample:
    component: str
    bytes: int
    time_us: float
    source: str
    launch: int = 0
    correct: bool = True


@dataclass(frozen=True)
class Segment:
    alpha_us: float
    beta_us_per_byte: float
    min_bytes: int
    max_bytes: int | None
    relative_error: float


def cv(values) -> float:
    if len(values) < 2:
        return 0.0
    mean = statistics.fmean(values)
    return statistics.pstdev(values) / mean if mean else float("inf")


def qualify(samples, *, max_cv: float):
    """Return (qualified samples, reasons for rejected ones)."""
    reasons = []
    good = [s for s in samples if s.source in NATIVE_SOURCES]
    if len(good) != len(samples):
        reasons.append("non-native samples rejected")
    bad = [s for s in good if not s.correct]
    if bad:
        reasons.append("%d samples failed their numerical check" % len(bad))
        good = [s for s in good if s.correct]
    by_size = {}
    for s in good:
        by_size.setdefault(s.bytes, []).append(s)
    out = []
    for size, items in sorted(by_size.items()):
        launches = sorted({s.launch for s in items})
        stable = None
        for first in launches:
            values = [s.time_us for s in items if s.launch >= first]
            if len(values) >= 3 and cv(values) <= max_cv:
                stable = first
                break
        if stable is None:
            reasons.append("size %d never stabilised (cv > %.3f)" % (size, max_cv))
            continue
        out.extend(s for s in items if s.launch >= stable)
    return out, reasons


def _lsq(points):
    x = np.array([p[0] for p in points], dtype=float)
    y = np.array([p[1] for p in points], dtype=float)
    if len(set(x)) < 2:
        raise RuntimeFailure("need at least two payload sizes to fit alpha and beta")
    a = np.vstack([np.ones_like(x), x]).T
    (alpha, beta), *_ = np.linalg.lstsq(a, y, rcond=None)
    alpha = max(0.0, float(alpha))
    beta = float(beta)
    if beta <= 0:
        beta = float(np.max(y / x))
    pred = alpha + beta * x
    err = float(np.max(np.abs(pred - y) / np.maximum(y, 1e-12)))
    return alpha, beta, err


def fit_curve(samples, *, max_relative_error: float):
    """Segments covering the sampled sizes; medians per size are fitted."""
    by_size = {}
    for s in samples:
        by_size.setdefault(s.bytes, []).append(s.time_us)
    points = sorted((size, statistics.median(v)) for size, v in by_size.items())
    if len(points) < 2:
        raise RuntimeFailure("not enough payload sizes to fit")
    alpha, beta, err = _lsq(points)
    if err <= max_relative_error or len(points) < 4:
        return [Segment(alpha, beta, 1, None, err)]
    mid = len(points) // 2
    left, right = points[:mid + 1], points[mid:]
    a1, b1, e1 = _lsq(left)
    a2, b2, e2 = _lsq(right)
    boundary = left[-1][0]
    return [Segment(a1, b1, 1, boundary, e1), Segment(a2, b2, boundary + 1, None, e2)]
