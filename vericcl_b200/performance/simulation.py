"""Discrete-event replay of an executable under a cost model (T_pred).

Each operation pays its α once when it starts, then moves its remaining bytes
at a rate set by the *current* concurrency mode: a measured
:class:`RateProfile` when one matches the set of active flows sharing
resources, otherwise min(link rate, fair share of every shared resource).
Rates are re-evaluated whenever an operation starts or finishes; progress is
never restarted.  ``exact=True`` performs all arithmetic on rationals
(``fractions.Fraction`` built from the decimal text of each parameter), so the
event order and the completion time are exact for the model
(reference: vericcl/performance/simulation.py:97-279).
"""
from __future__ import annotations

import heapq
from collections import deque
from dataclasses import dataclass
from fractions import Fraction
from functools import lru_cache
from types import MappingProxyType

from vericcl_b200.errors import SemanticError
from vericcl_b200.performance.events import COMM_KINDS, Executable
from vericcl_b200.performance.model import CostModel


@dataclass(frozen=True)
class Prediction:
    model_version: str
    t_pred_us: float | None
    output_ready_us: float | None
    start_times: dict
    end_times: dict
    segments: tuple
    used_components: frozenset
    missing_components: frozenset
    unavailable_operations: tuple
    model_coverage: str
    exact_completion_ratio: tuple | None = None
    unmeasured_modes: tuple = ()

    def critical_path(self, executable: Executable) -> list:
        """Operation ids on one longest dependency chain ending at T_pred."""
        if self.t_pred_us is None:
            return []
        ops = {op.operation_id: op for op in executable.operations}
        end = max(self.end_times, key=lambda k: (self.end_times[k], k))
        chain = [end]
        while True:
            op = ops[chain[-1]]
            if not op.dependencies:
                break
            chain.append(max(op.dependencies, key=lambda k: (self.end_times.get(k, 0), k)))
        return list(reversed(chain))


def _exact(value):
    return Fraction(value) if isinstance(value, int) else Fraction(str(value))


def _to_float(value):
    return value.numerator / value.denominator if isinstance(value, Fraction) else float(value)


def _acyclic(operations):
    degrees = {op.operation_id: len(op.dependencies) for op in operations}
    successors = {key: [] for key in degrees}
    for op in operations:
        for dep in op.dependencies:
            successors[dep].append(op.operation_id)
    remaining, ready, done = dict(degrees), deque(k for k, d in degrees.items() if d == 0), 0
    while ready:
        key = ready.popleft()
        done += 1
        for nxt in successors[key]:
            remaining[nxt] -= 1
            if remaining[nxt] == 0:
                ready.append(nxt)
    if done != len(degrees):
        raise SemanticError("executable dependency cycle")
    return degrees, successors


def _components(ops):
    """Connected components of communication operations by shared resources."""
    parent = {}

    def find(x):
        while parent[x] != x:
            parent[x] = parent[parent[x]]
            x = parent[x]
        return x

    owner = {}
    for op in ops:
        parent[op.operation_id] = op.operation_id
        for res in op.resources:
            if res in owner:
                a, b = find(owner[res]), find(op.operation_id)
                if a != b:
                    parent[a] = b
            else:
                owner[res] = op.operation_id
    groups = {}
    for op in ops:
        groups.setdefault(find(op.operation_id), []).append(op)
    return list(groups.values())


def _profile(group, model):
    matches = [p for p in model.profiles if p.applies(group)]
    if len(matches) > 1:
        raise SemanticError("multiple profiles apply to one concurrency mode")
    return matches[0] if matches else None


def predict(executable: Executable, model: CostModel, *, exact: bool = False) -> Prediction:
    num = lru_cache(maxsize=None)(_exact) if exact else float
    if dict(executable.context) != dict(model.context):
        raise SemanticError("cost model context differs from the executable")
    ops = {op.operation_id: op for op in executable.operations}
    degrees, successors = _acyclic(executable.operations)
    costs, unavailable, missing, used = {}, set(), set(), set()
    for key, op in ops.items():
        if op.kind == "nop":
            continue
        cost = model.service_for(op.cost_key, op.payload_bytes)
        if cost is None:
            unavailable.add(key)
            missing.add("service:" + op.cost_key)
        else:
            costs[key] = cost
        for res in op.resources:
            if res not in model.resources:
                unavailable.add(key)
                missing.add("resource:" + res)
    changed = True
    while changed:
        changed = False
        bad_res = {r for k in unavailable for r in ops[k].resources}
        for key, op in ops.items():
            if key not in unavailable and (set(op.dependencies) & unavailable or set(op.resources) & bad_res):
                unavailable.add(key)
                changed = True
    pending = set(ops) - unavailable
    releases = [(num(ops[k].not_before_us), k) for k in pending if degrees[k] == 0]
    heapq.heapify(releases)
    starts, ends, segments = {}, {}, []
    startup, active, remaining = {}, set(), {}
    sources_used, unmeasured = set(), set()
    now = num(0)

    def complete(key, time):
        ends[key] = time
        for nxt in successors[key]:
            if nxt in pending:
                degrees[nxt] -= 1
                if degrees[nxt] == 0:
                    heapq.heappush(releases, (max(time, num(ops[nxt].not_before_us)), nxt))

    def rates_for(active_ops):
        rates, srcs = {}, {}
        comm = []
        for op in active_ops:
            if op.kind in COMM_KINDS:
                comm.append(op)
            else:
                rates[op.operation_id] = 1 / num(costs[op.operation_id].beta_us_per_byte)
                srcs[op.operation_id] = (op.source_override or costs[op.operation_id].source)
        for group in _components(comm):
            if len({op.flow_id for op in group}) != len(group):
                raise SemanticError("concurrent operations share a flow identity")
            profile = _profile(group, model)
            resources = {r for op in group for r in op.resources}
            used.update("resource:" + r for r in resources)
            if profile is not None:
                used.add("profile:" + profile.profile_id)
                for op in group:
                    rates[op.operation_id] = num(profile.rates[op.flow_id])
                    srcs[op.operation_id] = profile.source
                continue
            if len(group) > 1:
                unmeasured.add(tuple(sorted(op.flow_id for op in group)))
            for op in group:
                own = 1 / num(costs[op.operation_id].beta_us_per_byte)
                limits = [own]
                for res in op.resources:
                    count = sum(res in other.resources for other in group)
                    limits.append(num(model.resources[res]) / count)
                rate = min(limits)
                rates[op.operation_id] = rate
                srcs[op.operation_id] = ("initial_sharing_estimate" if rate < own or len(group) > 1
                                         else (op.source_override or costs[op.operation_id].source))
        return rates, srcs

    while pending or startup or active:
        for key in sorted(startup):
            if startup[key] <= now:
                del startup[key]
                active.add(key)
        ready = []
        while releases and releases[0][0] <= now:
            ready.append(heapq.heappop(releases)[1])
        ready.sort()
        for key in ready:
            op = ops[key]
            pending.discard(key)
            starts[key] = now
            if op.kind == "nop":
                complete(key, now)
                continue
            cost = costs[key]
            used.add("service:" + op.cost_key)
            sources_used.add(op.source_override or cost.source)
            remaining[key] = num(op.payload_bytes)
            startup[key] = now + num(cost.alpha_us)
        if any(t <= now for t in startup.values()) or (releases and releases[0][0] <= now):
            continue
        rates, rate_sources = rates_for([ops[k] for k in sorted(active)])
        sources_used.update(rate_sources.values())
        finish = {k: now + remaining[k] / rates[k] for k in active}
        future = list(finish.values()) + list(startup.values())
        if releases:
            future.append(releases[0][0])
        if not future:
            if pending:
                raise SemanticError("executable stalls with unresolved work")
            break
        nxt = min(future)
        if nxt <= now:
            raise SemanticError("model precision cannot represent positive progress")
        delta = nxt - now
        for key in sorted(active):
            segments.append((key, _to_float(now), _to_float(nxt), _to_float(rates[key]), rate_sources[key]))
            remaining[key] = max(num(0), remaining[key] - rates[key] * delta)
        now = nxt
        for key in sorted(active):
            if finish[key] == nxt or remaining[key] == 0:
                active.discard(key)
                complete(key, now)
    t_pred = None if unavailable else max(ends.values(), default=num(0))
    out_ready = None if set(executable.output_operations) & unavailable else \
        max((ends[k] for k in executable.output_operations if k in ends), default=num(0))
    measured = {"measured", "history"}
    if unavailable:
        coverage = "unavailable"
    elif not sources_used:
        coverage = "not_required"
    elif sources_used <= measured:
        coverage = "measured"
    elif sources_used & measured:
        coverage = "partial"
    else:
        coverage = "initial"
    ratio = (t_pred.numerator, t_pred.denominator) if exact and t_pred is not None else None
    return Prediction(model.version, None if t_pred is None else _to_float(t_pred),
                      None if out_ready is None else _to_float(out_ready),
                      MappingProxyType({k: _to_float(v) for k, v in starts.items()}),
                      MappingProxyType({k: _to_float(v) for k, v in ends.items()}),
                      tuple(segments), frozenset(used), frozenset(missing), tuple(sorted(unavailable)),
                      coverage, ratio, tuple(sorted(unmeasured)))
