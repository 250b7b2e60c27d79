"""Fixed-route timing MILP: start times and connection order for small schedules.

With routes fixed, every transfer has a duration (α + β·S on its link) and
precedences (its data dependencies).  Transfers that share a connection
(same sender, receiver and channel — one thread block pair) cannot overlap;
each such pair gets a big-M disjunction with an order binary.  The MILP
minimises the makespan; its start times become the operations' priorities,
which the storage plan and the lowering turn into TB order (reference:
vericcl/solver/trees/timing.py:218-345, where a native-checked seed is
improved by a full channel/order MILP).  Instances above ``max_ops`` keep the
list-schedule seed.
"""
from __future__ import annotations

from dataclasses import replace
from itertools import combinations

from vericcl_b200.solver.milp import Model
from vericcl_b200.topology.model import LinkKey


def optimize_fixed_routes(candidate, topology, *, max_ops: int = 48, time_limit: float = 20.0):
    ops = list(candidate.operations)
    if not ops or len(ops) > max_ops:
        return candidate
    dur = {op.operation_id: topology.link(LinkKey(op.src_rank, op.dst_rank)).time_us(candidate.slice_size_bytes)
           for op in ops}
    horizon = sum(dur.values()) + 1.0
    m = Model("fixed-route-timing")
    start = {op.operation_id: m.continuous("s:" + op.operation_id, 0, horizon) for op in ops}
    z = m.continuous("makespan", 0, horizon)
    for op in ops:
        m.add_le([(1, start[op.operation_id]), (-1, z)], -dur[op.operation_id])
        for dep in op.dependencies:
            m.add_ge([(1, start[op.operation_id]), (-1, start[dep])], dur[dep])
    by_conn = {}
    for op in ops:
        by_conn.setdefault((op.src_rank, op.dst_rank, op.channel), []).append(op)
    for members in by_conn.values():
        for a, b in combinations(members, 2):
            order = m.binary("o:%s:%s" % (a.operation_id, b.operation_id))
            sa, sb = start[a.operation_id], start[b.operation_id]
            # order=1: a before b; order=0: b before a
            m.add_le([(1, sa), (-1, sb), (horizon, order)], horizon - dur[a.operation_id])
            m.add_le([(1, sb), (-1, sa), (-horizon, order)], -dur[b.operation_id])
    m.minimize([(1, z)])
    sol = m.solve(time_limit=time_limit)
    if not sol.usable:
        return candidate
    timed = [replace(op, priority_time=round(sol.values[start[op.operation_id].name], 6)) for op in ops]
    return replace(candidate, operations=tuple(timed), origin=candidate.origin + "+timing")
