"""T_pred: an exact fluid replay of a work graph under a cost model.

The rules (the behaviour the reference specifies for its predictor,
vericcl/performance/simulation.py:136; the algorithm below is this project's):

* An operation is *released* once all its dependencies have completed and its
  ``release_us`` has passed.  A dependency-only operation completes there.
* A released data operation first spends its segment's α moving nothing,
  then drains its payload as a fluid whose rate is constant between two
  consecutive events (a release, the end of an α, a completion).
* Local work (copy, reduce) drains at its segment's rate 1/β.
* Network operations that cross a common shared resource, directly or
  through others, form a *sharing group*.  A group whose flows are exactly
  those of a measured sharing mode runs at the measured rates.  Otherwise
  rates are max-min fair (progressive filling, Bertsekas & Gallager, *Data
  Networks*, §6.5.2): every flow is capped by its own 1/β, all unfrozen flows
  rise together, a flow freezes when it reaches its cap or when a resource it
  crosses is full, and capacity a frozen flow leaves unused goes to the
  others.  On an NVSwitch this is what a GPU's NVLink port does when one of
  its transfers is held back elsewhere.
* ``exact=True`` runs the whole replay on rationals built from the decimal
  text of every parameter, so event order and completion time are exact
  for the model; the completion time is then also returned as a ratio.

The result records every operation's start and end, the rate segments, which
components were used or missing, and which multi-flow sharing modes had no
measurement.
"""
from __future__ import annotations

import heapq
from dataclasses import dataclass, field
from fractions import Fraction
from types import MappingProxyType

from vericcl_b200.errors import SemanticError
from vericcl_b200.performance.events import COMM_KINDS, Executable
from vericcl_b200.performance.model import CostModel

_MEASURED = frozenset({"measured", "history"})
SHARED_ESTIMATE = "initial_sharing_estimate"
ESTIMATED = "estimated"             # the source label of work marked estimated (priced, not measured)


@dataclass(frozen=True)
class Prediction:
    model_version: str
    t_pred_us: float | None
    output_ready_us: float | None
    start_times: dict
    end_times: dict
    segments: tuple                     # (operation, t0, t1, rate bytes/µs, rate source)
    used_components: frozenset
    missing_components: frozenset
    unavailable_operations: tuple
    model_coverage: str                 # incomplete | no_data | measured | mixed | initial
    exact_completion_ratio: tuple | None = None
    unmeasured_modes: tuple = ()
    source_time_us: dict = field(default_factory=dict)   # busy µs of priced work per rate source

    def critical_path(self, executable: Executable) -> list:
        """One dependency chain that ends at T_pred: from the last operation, follow the latest dependency."""
        if self.t_pred_us is None or not self.end_times:
            return []
        ops = executable.by_id()
        node = max(self.end_times, key=lambda k: (self.end_times[k], k))
        chain = [node]
        while ops[node].after:
            node = max(ops[node].after, key=lambda k: (self.end_times.get(k, 0.0), k))
            chain.append(node)
        chain.reverse()
        return chain


class _Numbers:
    """Float or exact rational arithmetic for one replay."""

    def __init__(self, exact: bool):
        self.exact = exact
        self._memo: dict = {}

    def __call__(self, value):
        if not self.exact:
            return float(value)
        hit = self._memo.get(value)
        if hit is None:
            hit = Fraction(value) if isinstance(value, int) else Fraction(repr(float(value)))
            self._memo[value] = hit
        return hit

    @staticmethod
    def out(value) -> float:
        return float(value)


def _successors_in_order(executable: Executable):
    """Successor lists, and a check that the dependency graph has no cycle (iterative depth-first search)."""
    succ = {op.operation_id: [] for op in executable.operations}
    deps = {op.operation_id: op.after for op in executable.operations}
    for op in executable.operations:
        for d in op.after:
            succ[d].append(op.operation_id)
    state = dict.fromkeys(deps, 0)          # 0 unseen, 1 on the stack, 2 finished
    for root in deps:
        if state[root]:
            continue
        stack = [(root, iter(deps[root]))]
        state[root] = 1
        while stack:
            node, it = stack[-1]
            nxt = next(it, None)
            if nxt is None:
                state[node] = 2
                stack.pop()
            elif state[nxt] == 1:
                raise SemanticError("the work graph has a dependency cycle through %s" % nxt)
            elif state[nxt] == 0:
                state[nxt] = 1
                stack.append((nxt, iter(deps[nxt])))
    return succ


def _sharing_groups(active_ops):
    """Partition network operations into groups connected through common resources (breadth-first search)."""
    users: dict = {}
    for op in active_ops:
        for r in op.crosses:
            users.setdefault(r, []).append(op)
    seen, groups = set(), []
    for op in active_ops:
        if op.operation_id in seen:
            continue
        group, frontier = [], [op]
        seen.add(op.operation_id)
        while frontier:
            cur = frontier.pop()
            group.append(cur)
            for r in cur.crosses:
                for other in users[r]:
                    if other.operation_id not in seen:
                        seen.add(other.operation_id)
                        frontier.append(other)
        groups.append(sorted(group, key=lambda o: o.operation_id))
    return groups


def max_min_rates(caps: dict, crossings: dict, capacity: dict, zero):
    """Max-min fair rates by progressive filling.

    ``caps``: flow → its own rate limit; ``crossings``: flow → resources it uses;
    ``capacity``: resource → capacity.  Every flow ends at its cap or crosses a
    saturated resource on which no other flow has a higher rate.
    """
    rate = dict.fromkeys(caps, zero)
    left = dict(capacity)
    live = set(caps)
    while live:
        users = {}
        for f in live:
            for r in crossings[f]:
                users[r] = users.get(r, 0) + 1
        step = min(caps[f] - rate[f] for f in live)
        for r, n in users.items():
            share = left[r] / n
            if share < step:
                step = share
        if step < zero:
            step = zero
        for f in live:
            rate[f] += step
        for r, n in users.items():
            left[r] -= step * n
        full = {r for r, n in users.items() if left[r] <= zero}
        done = {f for f in live if rate[f] >= caps[f] or any(r in full for r in crossings[f])}
        if not done:          # floating-point rounding left every margin a hair above zero
            done = {min(live, key=lambda f: min([caps[f] - rate[f]] + [left[r] for r in crossings[f]]))}
        live -= done
    return rate


class _Replay:
    def __init__(self, executable: Executable, model: CostModel, exact: bool):
        self.ex, self.model = executable, model
        self.num = _Numbers(exact)
        self.ops = executable.by_id()
        self.succ = _successors_in_order(executable)
        self.used, self.missing = set(), set()
        self.seg = {}
        self.blocked = self._price()

    def _price(self) -> set:
        """Look up every operation's segment; return the operations that cannot be timed."""
        blocked = set()
        for key, op in self.ops.items():
            if op.kind == "nop":
                continue
            seg = self.model.service_for(op.component, op.nbytes)
            if seg is None:
                self.missing.add("service:" + op.component)
                blocked.add(key)
            else:
                self.seg[key] = seg
            for r in op.crosses:
                if self.model.capacity(r) is None:
                    self.missing.add("resource:" + r)
                    blocked.add(key)
        # whatever waits for, or shares a resource with, untimeable work cannot be timed either
        by_res: dict = {}
        for op in self.ops.values():
            for r in op.crosses:
                by_res.setdefault(r, []).append(op.operation_id)
        todo = list(blocked)
        while todo:
            key = todo.pop()
            spread = list(self.succ[key])
            for r in self.ops[key].crosses:
                spread.extend(by_res[r])
            for other in spread:
                if other not in blocked:
                    blocked.add(other)
                    todo.append(other)
        return blocked

    def _rates(self, flowing: list):
        """Rate and rate source of every draining operation for the current interval."""
        num, rates, src, modes = self.num, {}, {}, set()
        network = []
        for op in flowing:
            if op.kind in COMM_KINDS:
                network.append(op)
            else:
                seg = self.seg[op.operation_id]
                rates[op.operation_id] = 1 / num(seg.beta_us_per_byte)
                src[op.operation_id] = ESTIMATED if op.estimated else seg.source
        for group in _sharing_groups(network):
            flows = [op.flow_id for op in group]
            if len(set(flows)) < len(flows):
                raise SemanticError("two concurrent operations claim one flow id in %s" % sorted(flows))
            self.used.update("resource:" + r for op in group for r in op.crosses)
            mode = self.model.measured_mode(group)
            if mode is not None:
                self.used.add("profile:" + mode.profile_id)
                for op in group:
                    rates[op.operation_id] = num(mode.rates[op.flow_id])
                    src[op.operation_id] = mode.source
                continue
            if len(group) > 1:
                modes.add(tuple(sorted(flows)))
            caps = {op.operation_id: 1 / num(self.seg[op.operation_id].beta_us_per_byte) for op in group}
            cross = {op.operation_id: op.crosses for op in group}
            capacity = {r: num(self.model.capacity(r)) for op in group for r in op.crosses}
            fair = max_min_rates(caps, cross, capacity, num(0))
            for op in group:
                k = op.operation_id
                rates[k] = fair[k]
                shared = len(group) > 1 or fair[k] < caps[k]
                src[k] = SHARED_ESTIMATE if shared else (ESTIMATED if op.estimated else self.seg[k].source)
        return rates, src, modes

    def run(self) -> Prediction:
        num, ops = self.num, self.ops
        zero = num(0)
        waiting = {k: len(op.after) for k, op in ops.items() if k not in self.blocked}
        calendar: list = []      # (time, phase, operation): phase 0 release, 1 end of alpha
        for k, n in waiting.items():
            if n == 0:
                heapq.heappush(calendar, (num(ops[k].release_us), 0, k))
        start, end, segments = {}, {}, []
        left, drain = {}, {}     # bytes still to move; operations draining now
        source_time: dict = {}
        sources, unmeasured = set(), set()
        now = zero

        def finish(key, t):
            end[key] = t
            for s in self.succ[key]:
                if s in waiting:
                    waiting[s] -= 1
                    if waiting[s] == 0:
                        heapq.heappush(calendar, (max(t, num(ops[s].release_us)), 0, s))

        while calendar or drain:
            # everything that happens at `now`: releases, ends of α (in that order, each by id)
            while calendar and calendar[0][0] <= now:
                _, phase, key = heapq.heappop(calendar)
                op = ops[key]
                if phase == 0:
                    start[key] = now
                    if op.kind == "nop":
                        finish(key, now)
                        continue
                    seg = self.seg[key]
                    self.used.add("service:" + op.component)
                    sources.add(ESTIMATED if op.estimated else seg.source)
                    left[key] = num(op.nbytes)
                    heapq.heappush(calendar, (now + num(seg.alpha_us), 1, key))
                else:
                    drain[key] = op
            if not drain:
                if not calendar:
                    break
                now = calendar[0][0]
                continue
            rates, rsrc, modes = self._rates([drain[k] for k in sorted(drain)])
            unmeasured |= modes
            sources.update(rsrc.values())
            done_at = {k: now + left[k] / rates[k] for k in drain}
            horizon = min(done_at.values())
            if calendar and calendar[0][0] < horizon:
                horizon = calendar[0][0]
            if horizon <= now:
                raise SemanticError("no progress at t=%r: the model's numbers are too small to represent" % now)
            dt = horizon - now
            for k in sorted(drain):
                segments.append((k, num.out(now), num.out(horizon), num.out(rates[k]), rsrc[k]))
                source_time[rsrc[k]] = source_time.get(rsrc[k], 0.0) + num.out(dt)
                left[k] = left[k] - rates[k] * dt
            now = horizon
            for k in sorted(drain):
                if done_at[k] <= horizon or left[k] <= zero or \
                        (not num.exact and left[k] <= 1e-9 * ops[k].nbytes):
                    del drain[k]
                    finish(k, now)
        if any(n > 0 for n in waiting.values()):
            raise SemanticError("work never became ready: %s" % sorted(k for k, n in waiting.items() if n)[:5])
        blocked = self.blocked
        t_pred = None if blocked else max(end.values(), default=zero)
        outs = self.ex.output_operations
        ready = None if set(outs) & blocked else max((end[k] for k in outs if k in end), default=zero)
        if blocked:
            label = "incomplete"
        elif not sources:
            label = "no_data"
        elif sources <= _MEASURED:
            label = "measured"
        elif sources & _MEASURED:
            label = "mixed"
        else:
            label = "initial"
        ratio = None
        if self.num.exact and t_pred is not None:
            ratio = (t_pred.numerator, t_pred.denominator)
        return Prediction(self.model.version, None if t_pred is None else num.out(t_pred),
                          None if ready is None else num.out(ready),
                          MappingProxyType({k: num.out(v) for k, v in start.items()}),
                          MappingProxyType({k: num.out(v) for k, v in end.items()}),
                          tuple(segments), frozenset(self.used), frozenset(self.missing), tuple(sorted(blocked)),
                          label, ratio, tuple(sorted(unmeasured)), source_time)


def predict(executable: Executable, model: CostModel, *, exact: bool = False) -> Prediction:
    """Replay ``executable`` under ``model`` and return the prediction (see the module docstring)."""
    if dict(executable.context) != dict(model.context):
        raise SemanticError("the executable was lowered for %r but the model describes %r"
                            % (dict(executable.context), dict(model.context)))
    return _Replay(executable, model, exact).run()
