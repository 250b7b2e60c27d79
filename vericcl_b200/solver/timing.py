"""Fixed-route timing MILP: start times and connection order once routes are chosen.

With routes fixed, every transfer has a duration (α + β·S on its link) and
precedences (its data dependencies).  Transfers that share a connection
(same sender, receiver and channel — one thread-block pair) cannot overlap;
each such pair gets a big-M disjunction with an order binary.  The MILP
minimises the makespan; its start times become the operations' priorities,
which the storage plan and the lowering turn into thread-block order
(reference: vericcl/solver/trees/timing.py:218-345, where a native-checked
seed is improved by a full channel/order MILP).

Shared resources are part of the model.  On an NVSwitch every GPU's NVLink
transmit and receive ports are shared by all its transfers; the MILP treats
each shared resource as a unary machine that a transfer holds for
``bytes / capacity`` (the same total busy time the fluid sharing of the event
simulator gives), with one order binary per pair of transfers on it.  This is
what makes the timing matter on a switch, where every pairwise link is
uncontended and only the ports are.

Large schedules (an 8-GPU AllReduce has hundreds of transfers) are solved by
a rolling horizon: the operations, in list-schedule order, are cut into
windows that are closed under dependencies; each window is one MILP whose
earlier windows are fixed (their end times are release times, their last use
of a connection blocks it), and whose objective is the window's makespan
plus a small weight on the sum of its completion times.  Every schedule is
therefore solver-timed; a window whose MILP gives no solution keeps the
list-schedule times of its operations.
"""
from __future__ import annotations

from dataclasses import replace
from itertools import combinations

from vericcl_b200.solver.milp import Model
from vericcl_b200.topology.model import LinkKey

WINDOW = 20


def _durations(ops, topology, size):
    return {op.operation_id: topology.link(LinkKey(op.src_rank, op.dst_rank)).time_us(size) for op in ops}


def _holds(ops, topology, size):
    """Per operation: {shared resource: µs it keeps the resource busy} (bytes over the resource's capacity)."""
    out = {}
    for op in ops:
        link = topology.link(LinkKey(op.src_rank, op.dst_rank))
        out[op.operation_id] = {r: size / topology.resources[r].capacity_bytes_per_us
                                for r in link.resource_ids if r in topology.resources}
    return out


def _solve_window(window, dur, hold, release, conn_free, res_free, time_limit):
    """Start times of ``window`` (dict) or None.

    ``release``: per operation, the end of its dependencies in earlier windows;
    ``conn_free`` / ``res_free``: when earlier windows stop using a connection / a resource.
    """
    ids = {op.operation_id for op in window}
    lower = {op.operation_id: max([release.get(op.operation_id, 0.0),
                                   conn_free.get((op.src_rank, op.dst_rank, op.channel), 0.0)] +
                                  [res_free.get(r, 0.0) for r in hold[op.operation_id]]) for op in window}
    # running the window's operations one after another from its latest lower bound is always feasible
    horizon = max(lower.values()) + sum(dur[k] for k in ids) + 1.0
    m = Model("fixed-route-timing-window")
    start = {op.operation_id: m.continuous("s:" + op.operation_id, lower[op.operation_id], horizon)
             for op in window}
    z = m.continuous("makespan", 0, horizon + max(dur.values()))
    for op in window:
        k = op.operation_id
        m.add_le([(1, start[k]), (-1, z)], -dur[k])
        for dep in op.dependencies:
            if dep in ids:
                m.add_ge([(1, start[k]), (-1, start[dep])], dur[dep])
    by_conn = {}
    for op in window:
        by_conn.setdefault((op.src_rank, op.dst_rank, op.channel), []).append(op)
    big = horizon + max(dur.values())
    for members in by_conn.values():
        for a, b in combinations(members, 2):
            order = m.binary("o:%s:%s" % (a.operation_id, b.operation_id))
            sa, sb = start[a.operation_id], start[b.operation_id]
            m.add_le([(1, sa), (-1, sb), (big, order)], big - dur[a.operation_id])
            m.add_le([(1, sb), (-1, sa), (-big, order)], -dur[b.operation_id])
    users = {}
    for op in window:
        for r in hold[op.operation_id]:
            users.setdefault(r, []).append(op)
    for r, members in users.items():
        for a, b in combinations(members, 2):
            if (a.src_rank, a.dst_rank, a.channel) == (b.src_rank, b.dst_rank, b.channel):
                continue        # already ordered by their connection
            order = m.binary("r:%s:%s:%s" % (r, a.operation_id, b.operation_id))
            sa, sb = start[a.operation_id], start[b.operation_id]
            m.add_le([(1, sa), (-1, sb), (big, order)], big - hold[a.operation_id][r])
            m.add_le([(1, sb), (-1, sa), (-big, order)], -hold[b.operation_id][r])
    weight = 1.0 / (4 * len(window))
    m.minimize([(1, z)] + [(weight, start[op.operation_id]) for op in window],
               constant=weight * sum(dur[op.operation_id] for op in window))
    sol = m.solve(time_limit=time_limit)
    if not sol.usable:
        return None
    return {k: sol.values[v.name] for k, v in start.items()}


def _topological(ops):
    """Operations in list-schedule order, with every operation after its dependencies."""
    pos = {op.operation_id: i for i, op in enumerate(sorted(ops, key=lambda o: (o.priority_time, o.operation_id)))}
    by_id = {op.operation_id: op for op in ops}
    out, placed = [], set()

    def place(op):
        stack = [op]
        while stack:
            cur = stack[-1]
            pending = [by_id[d] for d in sorted(cur.dependencies, key=lambda d: pos[d]) if d not in placed]
            if pending:
                stack.append(pending[0])
                continue
            stack.pop()
            if cur.operation_id not in placed:
                placed.add(cur.operation_id)
                out.append(cur)

    for op in sorted(ops, key=lambda o: pos[o.operation_id]):
        place(op)
    return out


def optimize_fixed_routes(candidate, topology, *, window: int = WINDOW, time_limit: float = 6.0):
    """Solver-timed priorities for every operation of ``candidate`` (see the module docstring)."""
    ops = list(candidate.operations)
    if not ops:
        return candidate
    dur = _durations(ops, topology, candidate.slice_size_bytes)
    hold = _holds(ops, topology, candidate.slice_size_bytes)
    order = _topological(ops)
    chunks = [order[i:i + window] for i in range(0, len(order), window)]
    per_window = max(0.1, time_limit / len(chunks))
    start, end, conn_free, res_free = {}, {}, {}, {}
    solved = 0
    for chunk in chunks:
        release = {op.operation_id: max([end[d] for d in op.dependencies if d in end], default=0.0)
                   for op in chunk}
        times = _solve_window(chunk, dur, hold, release, conn_free, res_free, per_window)
        if times is None:
            # list-schedule the window: earliest start after dependencies and the connection
            times = {}
            local_free, local_res = dict(conn_free), dict(res_free)
            for op in chunk:
                k = op.operation_id
                conn = (op.src_rank, op.dst_rank, op.channel)
                t = max([release[k], local_free.get(conn, 0.0)] + [times[d] + dur[d] for d in op.dependencies
                                                                   if d in times] +
                        [local_res.get(r, 0.0) for r in hold[k]])
                times[k] = t
                local_free[conn] = t + dur[k]
                for r, busy in hold[k].items():
                    local_res[r] = t + busy
        else:
            solved += 1
        for op in chunk:
            k = op.operation_id
            start[k] = times[k]
            end[k] = times[k] + dur[k]
            conn = (op.src_rank, op.dst_rank, op.channel)
            conn_free[conn] = max(conn_free.get(conn, 0.0), end[k])
            for r, busy in hold[k].items():
                res_free[r] = max(res_free.get(r, 0.0), times[k] + busy)
    if not solved:
        return candidate
    timed = [replace(op, priority_time=round(start[op.operation_id], 6)) for op in ops]
    tag = "+timing" if solved == len(chunks) else "+timing(%d/%d windows)" % (solved, len(chunks))
    return replace(candidate, operations=tuple(timed), origin=candidate.origin + tag)


def makespan(candidate, topology) -> float:
    """The schedule length the priorities imply on the link model (start + duration, maximised)."""
    dur = _durations(candidate.operations, topology, candidate.slice_size_bytes)
    return max((op.priority_time + dur[op.operation_id] for op in candidate.operations), default=0.0)


def keep_better(seed_bundle, timed_bundle):
    """The lowered candidate with the smaller exact T_pred (the seed on a tie or when one is unavailable)."""
    a, b = seed_bundle.t_pred_us, timed_bundle.t_pred_us
    if b is not None and (a is None or b < a) and timed_bundle.can_execute:
        return timed_bundle
    return seed_bundle
