"""Alignment of per-GPU %globaltimer clocks to one host clock.

Before and after a traced invocation every rank takes bracketing samples:
host time before, a GPU timer read, host time after.  The GPU reading is
mapped to the bracket's midpoint with an uncertainty of half the bracket
width; offset and drift per rank come from a least-squares fit over all
samples, keeping the narrowest brackets.  Two events on different GPUs are
"ordered" only when their aligned intervals do not overlap (reference:
vericcl/verification/online/clock_sync.py:236-370).
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np


@dataclass(frozen=True)
class ClockMap:
    offset_ns: float      # host = gpu * (1 + drift) + offset
    drift: float
    uncertainty_ns: float

    def to_host(self, gpu_ns: float) -> float:
        return gpu_ns * (1.0 + self.drift) + self.offset_ns


def fit_transform(samples, *, keep_fraction: float = 0.5) -> ClockMap:
    """``samples``: [(host_before_ns, gpu_ns, host_after_ns)] for one rank."""
    if not samples:
        raise ValueError("no clock samples")
    widths = sorted(s[2] - s[0] for s in samples)
    limit = widths[max(0, int(len(widths) * keep_fraction) - 1)]
    kept = [s for s in samples if s[2] - s[0] <= limit] or list(samples)
    gpu = np.array([s[1] for s in kept], dtype=float)
    host = np.array([(s[0] + s[2]) / 2.0 for s in kept], dtype=float)
    if len(kept) >= 2 and np.ptp(gpu) > 0:
        slope, intercept = np.polyfit(gpu - gpu[0], host, 1)
        drift = float(slope - 1.0)
        offset = float(intercept - gpu[0] * (1.0 + drift))
    else:
        drift = 0.0
        offset = float(np.mean(host - gpu))
    unc = float(max(s[2] - s[0] for s in kept) / 2.0)
    return ClockMap(offset, drift, unc)


def align_bracketed_globaltimers(per_rank_samples) -> dict:
    return {rank: fit_transform(samples) for rank, samples in per_rank_samples.items()}


def ordered(a_interval, b_interval) -> str:
    """'before', 'after' or 'uncertain' for two (start, end) host-time intervals."""
    if a_interval[1] < b_interval[0]:
        return "before"
    if b_interval[1] < a_interval[0]:
        return "after"
    return "uncertain"
