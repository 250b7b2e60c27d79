"""Compose chosen route trees into a timed network schedule.

Every tree edge becomes one :class:`NetworkOperation` moving one logical slice
over one directed link: ``send`` for broadcast trees, ``rrc``
(receive-reduce-copy) for reduction trees.  Dependencies follow data
availability: a relay forwards only after it received, a reduction edge
leaves a child only after all of the child's subtree arrived, successive
reductions into one parent are chained through its accumulator, and a plan
node's first transfers wait for the producer nodes' deliveries at their
source rank.  Channels are assigned round-robin per directed link, and start
times come from a list schedule that serialises work on each
(src, dst, channel) connection (reference: vericcl/composer/compose.py:617,
vericcl/composer/timing.py:401).
"""
from __future__ import annotations

import heapq
from dataclasses import dataclass

from vericcl_b200.errors import SemanticError
from vericcl_b200.topology.model import LinkKey


@dataclass(frozen=True)
class NetworkOperation:
    operation_id: str
    kind: str                   # send | rrc
    src_rank: int
    dst_rank: int
    channel: int
    stage_id: int
    contributors: frozenset     # contributors of the value that crosses the link
    target_contributors: frozenset
    dependencies: frozenset
    priority_time: float
    index: int = -1             # logical slice position


@dataclass(frozen=True)
class NetworkCandidate:
    rank_count: int
    slice_count: int
    slice_size_bytes: int
    operations: tuple
    origin: str
    channels: int = 1
    metadata: tuple = ()


def compose_routes(plan, demands, trees, topology, slice_bytes: int, *, channels: int = 1, origin: str = "direct"):
    """Return a :class:`NetworkCandidate` for the chosen trees."""
    n, p = plan.slice_count, plan.rank_count
    ops = []
    # (rank, index, contributors) -> op id that made the value available there (None = original input)
    ready = {}
    for rank in range(p):
        for index in range(n):
            ready[(rank, index, frozenset({rank * n + index}))] = None
    by_node = {d.node_id: d for d in demands}
    link_count = {}

    def channel_for(a, b):
        key = (a, b)
        c = link_count.get(key, 0)
        link_count[key] = c + 1
        limit = min(channels, topology.link(LinkKey(a, b)).max_channels)
        return c % limit

    def lookup(rank, index, contributors):
        key = (rank, index, frozenset(contributors))
        if key not in ready:
            raise SemanticError("value %s is not available at rank %d before it is used" % (sorted(contributors), rank))
        return ready[key]

    for node in plan.nodes:
        d = by_node[node.node_id]
        tree = trees.get(d.demand_id)
        if d.kind == "broadcast":
            (value,) = d.contributors.values()
            src_dep = lookup(d.root, d.index, value)
            if tree is None:
                continue
            arrival = {d.root: src_dep}
            for a, b in _from_root(tree.edges, d.root):
                if a not in arrival:
                    raise SemanticError("broadcast tree edge leaves a rank that has not received the value")
                op_id = "%s:%d>%d" % (d.demand_id, a, b)
                deps = frozenset({arrival[a]} - {None})
                ops.append(NetworkOperation(op_id, "send", a, b, channel_for(a, b), d.stage_id, frozenset(value),
                                            frozenset(value), deps, 0.0, d.index))
                arrival[b] = op_id
                ready[(b, d.index, frozenset(value))] = op_id
        else:
            if tree is None:
                continue
            children = {}
            for a, b in tree.edges:
                children.setdefault(b, []).append(a)
            subtree = {}

            def value_of(rank):
                if rank in subtree:
                    return subtree[rank]
                own = frozenset(d.contributors.get(rank, frozenset()))
                total = own
                for child in children.get(rank, ()):
                    total = total | value_of(child)
                subtree[rank] = total
                return total

            value_of(d.root)
            accumulator = {}
            # post-order: a child's edge is emitted after all its own inbound edges
            emitted = set()

            def emit(rank):
                for child in sorted(children.get(rank, ())):
                    emit(child)
                    carried = subtree[child]
                    deps = set()
                    if child in accumulator:
                        deps.add(accumulator[child][0])
                    else:
                        dep = lookup(child, d.index, d.contributors[child])
                        if dep:
                            deps.add(dep)
                    if rank in accumulator:
                        deps.add(accumulator[rank][0])
                        base = accumulator[rank][1]
                    else:
                        base = frozenset(d.contributors.get(rank, frozenset()))
                        dep = lookup(rank, d.index, base) if base else None
                        if dep:
                            deps.add(dep)
                    op_id = "%s:%d>%d" % (d.demand_id, child, rank)
                    combined = base | carried
                    if base & carried:
                        raise SemanticError("reduction tree combines overlapping contributors")
                    ops.append(NetworkOperation(op_id, "rrc", child, rank, channel_for(child, rank), d.stage_id,
                                                carried, combined, frozenset(deps), 0.0, d.index))
                    accumulator[rank] = (op_id, combined)
                    ready[(rank, d.index, combined)] = op_id
                    emitted.add(op_id)

            emit(d.root)
            if subtree[d.root] != d.target:
                raise SemanticError("reduction tree does not deliver the node's target contributors")
    timed = list_schedule(ops, topology, slice_bytes)
    return NetworkCandidate(p, n, slice_bytes, tuple(timed), origin, channels)


def _from_root(edges, root):
    """Broadcast tree edges ordered so that every edge leaves an already-reached rank."""
    children = {}
    for a, b in edges:
        children.setdefault(a, []).append(b)
    out, frontier = [], [root]
    while frontier:
        nxt = []
        for a in frontier:
            for b in children.get(a, ()):
                out.append((a, b))
                nxt.append(b)
        frontier = nxt
    if len(out) != len(edges):
        raise SemanticError("broadcast tree is not an arborescence rooted at %d" % root)
    return out


def list_schedule(ops, topology, slice_bytes: int):
    """Assign priority times: earliest start with per-connection serialisation."""
    by_id = {op.operation_id: op for op in ops}
    indeg = {op.operation_id: len(op.dependencies) for op in ops}
    succ = {op.operation_id: [] for op in ops}
    for op in ops:
        for dep in op.dependencies:
            if dep not in by_id:
                raise SemanticError("unknown network dependency " + dep)
            succ[dep].append(op.operation_id)
    earliest = {key: 0.0 for key in by_id}
    conn_free = {}
    heap = [(0.0, i, op.operation_id) for i, op in enumerate(ops) if not op.dependencies]
    heapq.heapify(heap)
    order = {op.operation_id: i for i, op in enumerate(ops)}
    start, out = {}, []
    while heap:
        t, _, key = heapq.heappop(heap)
        op = by_id[key]
        conn = (op.src_rank, op.dst_rank, op.channel)
        s = max(t, conn_free.get(conn, 0.0))
        duration = topology.link(LinkKey(op.src_rank, op.dst_rank)).time_us(slice_bytes)
        conn_free[conn] = s + duration
        start[key] = s
        for nxt in succ[key]:
            indeg[nxt] -= 1
            earliest[nxt] = max(earliest[nxt], s + duration)
            if indeg[nxt] == 0:
                heapq.heappush(heap, (earliest[nxt], order[nxt], nxt))
    if len(start) != len(ops):
        raise SemanticError("network dependencies contain a cycle")
    for op in ops:
        out.append(NetworkOperation(op.operation_id, op.kind, op.src_rank, op.dst_rank, op.channel, op.stage_id,
                                    op.contributors, op.target_contributors, op.dependencies,
                                    round(start[op.operation_id], 6), op.index))
    return out
