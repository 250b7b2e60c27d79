"""Paired measured acceptance of a candidate against the incumbent.

The launch order of AB/BA pairs is fixed in advance from a seed; each pair
measures both schedules back to back (device time, max over ranks).  Rounds
whose coefficient of variation exceeds ``max_cv`` are repeated up to
``max_rounds``.  The decision is a one-sided exact binomial sign test of
"candidate faster" at a significance level drawn from the task's statistical
ledger, plus the requirement that the median relative gain exceeds
``min_relative_gain`` (reference: vericcl/verification/online/acceptance.py:21-168).
Measurements labelled as simulations or fixtures are never accepted.
"""
from __future__ import annotations

import random
import statistics
from dataclasses import dataclass
from math import comb

from vericcl_b200.online.fitting import cv

NATIVE = frozenset({"native_interpreter"})


def one_sided_binomial(successes: int, trials: int) -> float:
    """P(X >= successes) for X ~ Binomial(trials, 1/2)."""
    return sum(comb(trials, k) for k in range(successes, trials + 1)) / 2 ** trials


def pair_order(pairs: int, seed: int):
    rng = random.Random(seed)
    order = []
    for _ in range(pairs // 2):
        first = rng.choice(("AB", "BA"))
        order += [first, "BA" if first == "AB" else "AB"]
    return order


@dataclass
class MeasuredComparison:
    accepted: bool
    p_value: float | None
    alpha: float
    median_gain: float | None
    pairs: int
    reason: str
    rounds: int = 1


def compare_measured(measure, *, pairs: int, seed: int, alpha: float, max_cv: float, max_rounds: int,
                     min_relative_gain: float, source: str = "native_interpreter") -> MeasuredComparison:
    """``measure(label) -> time_us`` runs schedule ``label`` ('A' incumbent, 'B' candidate) once."""
    if source not in NATIVE:
        return MeasuredComparison(False, None, alpha, None, 0, "measurement source %r is not native" % source)
    for round_index in range(1, max_rounds + 1):
        a_times, b_times = [], []
        for order in pair_order(pairs, seed + round_index):
            first, second = order[0], order[1]
            t1 = measure(first)
            t2 = measure(second)
            (a_times if first == "A" else b_times).append(t1)
            (a_times if second == "A" else b_times).append(t2)
        if cv(a_times) <= max_cv and cv(b_times) <= max_cv:
            break
    else:
        return MeasuredComparison(False, None, alpha, None, pairs, "measurements never stabilised", max_rounds)
    wins = sum(1 for a, b in zip(a_times, b_times) if b < a)
    p = one_sided_binomial(wins, len(a_times))
    gains = [(a - b) / a for a, b in zip(a_times, b_times) if a > 0]
    median_gain = statistics.median(gains) if gains else None
    accepted = p <= alpha and median_gain is not None and median_gain > min_relative_gain
    reason = "accepted" if accepted else ("sign test p=%.4g > alpha=%.4g" % (p, alpha) if p > alpha
                                          else "median gain %.4g not above %.4g" % (median_gain or 0,
                                                                                  min_relative_gain))
    return MeasuredComparison(accepted, p, alpha, median_gain, len(a_times), reason, round_index)
