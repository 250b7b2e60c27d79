"""Stage budgets and leases.

Stages (initial synthesis, online validation, offline validation, repair)
each have a per-round and a total limit; the run may have a wall limit and a
cleanup reserve.  A :class:`BudgetLease` is a deadline-carrying token handed
to solvers and workers; ``check()`` raises :class:`BudgetExhausted` once the
lease expired or was cancelled.  CPU slots come from the cgroup quota when
one is set (reference: vericcl/execution/budget.py:34-220).
"""
from __future__ import annotations

import os
import threading
import time
from dataclasses import dataclass, field

from vericcl_b200.errors import BudgetExhausted

STAGES = ("initial", "online", "offline", "repair")


def available_cpu_slots() -> int:
    try:
        quota, period = open("/sys/fs/cgroup/cpu.max").read().split()[:2]
        if quota != "max":
            return max(1, int(int(quota) / int(period)))
    except (OSError, ValueError):
        pass
    try:
        return max(1, len(os.sched_getaffinity(0)))
    except AttributeError:  # pragma: no cover
        return max(1, os.cpu_count() or 1)


class StandaloneLease:
    """A lease with only a deadline (tests and one-off tools)."""

    def __init__(self, seconds: float, clock=time.monotonic):
        self.clock = clock
        self.deadline = clock() + seconds
        self.cancelled = False

    @classmethod
    def after(cls, seconds, clock=time.monotonic):
        return cls(seconds, clock)

    def remaining(self) -> float:
        return max(0.0, self.deadline - self.clock())

    def check(self) -> None:
        if self.cancelled or self.clock() >= self.deadline:
            raise BudgetExhausted("lease expired")


@dataclass
class BudgetLease:
    stage: str
    seconds: float
    threads: int = 1
    clock: object = time.monotonic
    started: float = field(default=0.0)
    manager: object = None
    released: bool = False

    def __post_init__(self):
        self.started = self.clock()

    @property
    def deadline(self) -> float:
        return self.started + self.seconds

    def remaining(self) -> float:
        return max(0.0, self.deadline - self.clock())

    def check(self) -> None:
        if self.manager is not None and self.manager.cancelled:
            raise BudgetExhausted("run cancelled")
        if self.clock() >= self.deadline:
            raise BudgetExhausted("%s lease of %.1fs expired" % (self.stage, self.seconds))

    def release(self) -> float:
        if self.released:
            return 0.0
        self.released = True
        used = min(self.seconds, self.clock() - self.started)
        if self.manager is not None:
            self.manager._charge(self.stage, used, self.threads)
        return used

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.release()


class BudgetManager:
    def __init__(self, budgets: dict, *, cpu_budget: int | None = None, clock=time.monotonic, consumed=None,
                 round_consumed=None):
        self.budgets = dict(budgets)
        self.clock = clock
        self.started = clock()
        self.cpu_budget = min(cpu_budget or available_cpu_slots(), available_cpu_slots())
        self.consumed = dict(consumed or {s: 0.0 for s in STAGES})
        self.round_consumed = dict(round_consumed or {s: 0.0 for s in STAGES})
        self.threads_in_use = 0
        self.cancelled = False
        self._lock = threading.Lock()

    def _limits(self, stage):
        if stage == "initial":
            return None, self.budgets.get("max_initial_synthesis_s")
        key = {"online": "online_validation", "offline": "offline_validation", "repair": "repair"}[stage]
        return self.budgets.get("max_%s_per_round_s" % key), self.budgets.get("max_%s_total_s" % key)

    def remaining(self, stage: str) -> float:
        per_round, total = self._limits(stage)
        left = []
        if per_round is not None:
            left.append(per_round - self.round_consumed.get(stage, 0.0))
        if total is not None:
            left.append(total - self.consumed.get(stage, 0.0))
        wall = self.budgets.get("max_run_wall_s")
        if wall is not None:
            left.append(wall - (self.clock() - self.started) - self.budgets.get("cleanup_reserve_s", 0.0))
        return max(0.0, min(left)) if left else float("inf")

    def acquire(self, stage: str, seconds: float | None = None, threads: int = 1) -> BudgetLease:
        if stage not in STAGES:
            raise ValueError("unknown stage " + stage)
        with self._lock:
            if self.cancelled:
                raise BudgetExhausted("run cancelled")
            left = self.remaining(stage)
            if left <= 0:
                raise BudgetExhausted("%s budget exhausted" % stage)
            threads = max(1, min(threads, self.cpu_budget - self.threads_in_use))
            self.threads_in_use += threads
            return BudgetLease(stage, min(left, seconds if seconds is not None else left), threads, self.clock,
                               manager=self)

    def _charge(self, stage, used, threads):
        with self._lock:
            self.consumed[stage] = self.consumed.get(stage, 0.0) + used
            self.round_consumed[stage] = self.round_consumed.get(stage, 0.0) + used
            self.threads_in_use = max(0, self.threads_in_use - threads)

    def new_round(self) -> None:
        self.round_consumed = {s: 0.0 for s in STAGES}

    def add_downtime(self, seconds: float, stages=()) -> None:
        """Resume: downtime counts against the wall limit and against every stage active at the crash."""
        seconds = max(0.0, float(seconds))
        self.started -= seconds
        for stage in stages:
            self.consumed[stage] = self.consumed.get(stage, 0.0) + seconds
            self.round_consumed[stage] = self.round_consumed.get(stage, 0.0) + seconds

    def restore_elapsed(self, elapsed_s: float) -> None:
        self.started = self.clock() - max(0.0, float(elapsed_s))

    def cancel(self) -> None:
        self.cancelled = True

    def snapshot(self) -> dict:
        return {"consumed": dict(self.consumed), "round_consumed": dict(self.round_consumed),
                "elapsed_s": self.clock() - self.started, "budgets": dict(self.budgets)}
