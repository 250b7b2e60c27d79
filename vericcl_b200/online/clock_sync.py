"""Alignment of per-GPU %globaltimer clocks to one host clock.

Before and after a traced invocation every rank takes bracketing samples:
host time before (``L``), a GPU timer read (``g``), host time after (``U``).
If the GPU clock maps to host time as ``host = offset + g·(1 + drift)``, every
sample says ``L <= offset + g·(1 + drift) <= U``: the true (offset, drift)
lies in the intersection of these strips, a convex polygon.

:func:`fit_transform` picks the point of that polygon that is deepest inside
all brackets — it maximises the margin ``m`` in
``L + m <= offset + g·(1 + drift) <= U - m`` (a two-variable linear
program) — and reports as uncertainty the widest half-bracket less that
margin (never below zero).  Brackets that contradict
each other (a clock step, a sample delayed between its reads) make the
program infeasible; then the samples whose brackets are widest are dropped
one at a time until the rest agree, and as a last resort a least-squares fit
of the bracket midpoints is used, with the widest half-bracket as its
uncertainty.  Two events on different GPUs are "ordered" only when their
aligned intervals do not overlap (reference behaviour:
vericcl/verification/online/clock_sync.py:236-370; the feasibility-polygon
fit is this project's own).
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np


@dataclass(frozen=True)
class ClockMap:
    offset_ns: float      # host = gpu * (1 + drift) + offset
    drift: float
    uncertainty_ns: float
    method: str = "bracket-lp"
    samples_used: int = 0

    def to_host(self, gpu_ns: float) -> float:
        return gpu_ns * (1.0 + self.drift) + self.offset_ns


def _deepest_point(samples):
    """(offset, drift, margin) maximising the margin inside every bracket, or None when they disagree."""
    from scipy.optimize import linprog
    g0 = float(samples[0][1])
    # variables: offset' (host at g0), drift, margin; host(g) = offset' + (g - g0) * (1 + drift)
    # lower: offset' + dg*drift - m >= L - dg   ->  -offset' - dg*drift + m <= dg - L
    # upper: offset' + dg*drift + m <= U - dg
    a, b = [], []
    for lo, g, hi in samples:
        dg = float(g) - g0
        a.append([-1.0, -dg, 1.0])
        b.append(dg - float(lo))
        a.append([1.0, dg, 1.0])
        b.append(float(hi) - dg)
    span = max(float(s[2]) for s in samples) - min(float(s[0]) for s in samples) + 1.0
    res = linprog(c=[0.0, 0.0, -1.0], A_ub=np.array(a), b_ub=np.array(b),
                  bounds=[(None, None), (-0.01, 0.01), (None, span)], method="highs")
    if res.status != 0 or res.x is None or res.x[2] < -1e-9:
        return None
    off_at_g0, drift, margin = (float(v) for v in res.x)
    return off_at_g0 - g0 * (1.0 + drift), drift, max(0.0, margin)


def fit_transform(samples, *, keep_fraction: float = 1.0) -> ClockMap:
    """``samples``: [(host_before_ns, gpu_ns, host_after_ns)] for one rank.

    ``keep_fraction`` < 1 first keeps only that fraction of the narrowest brackets.
    """
    if not samples:
        raise ValueError("no clock samples")
    for lo, _g, hi in samples:
        if hi < lo:
            raise ValueError("a clock sample's host reads are out of order")
    ordered_samples = sorted(samples, key=lambda s: s[2] - s[0])
    keep = max(1, int(round(len(ordered_samples) * keep_fraction)))
    kept = ordered_samples[:keep]
    while len(kept) >= 1:
        found = _deepest_point(kept) if len(kept) >= 2 else None
        if found is not None:
            offset, drift, margin = found
            half = max((s[2] - s[0]) / 2.0 for s in kept)
            return ClockMap(offset, drift, max(0.0, half - margin), "bracket-lp", len(kept))
        if len(kept) <= 2:
            break
        kept = kept[:-1]          # drop the widest bracket and try again
    mid = np.array([(s[0] + s[2]) / 2.0 for s in ordered_samples], dtype=float)
    gpu = np.array([s[1] for s in ordered_samples], dtype=float)
    if len(ordered_samples) >= 2 and np.ptp(gpu) > 0:
        slope, intercept = np.polyfit(gpu - gpu[0], mid, 1)
        drift = float(slope - 1.0)
        offset = float(intercept - gpu[0] * (1.0 + drift))
    else:
        drift, offset = 0.0, float(np.mean(mid - gpu))
    half = float(max(s[2] - s[0] for s in ordered_samples) / 2.0)
    return ClockMap(offset, drift, half, "least-squares", len(ordered_samples))


def align_bracketed_globaltimers(per_rank_samples) -> dict:
    return {rank: fit_transform(samples) for rank, samples in per_rank_samples.items()}


def ordered(a_interval, b_interval) -> str:
    """'before', 'after' or 'uncertain' for two (start, end) host-time intervals."""
    if a_interval[1] < b_interval[0]:
        return "before"
    if b_interval[1] < a_interval[0]:
        return "after"
    return "uncertain"
