"""AllGather ↔ ReduceScatter duality: each schedule reversed into the other.

An AllGather moves every slice ``sid = s·q + j`` from its owner ``s`` to all
ranks along a broadcast tree.  Reversing every edge of that tree gives a
reduction tree into ``s`` — exactly what a ReduceScatter needs for its output
``sid`` (owned by rank ``s``), over the same links and channels.  Each AG
``send a→b`` becomes an ``rrc b→a`` carrying the sum of ``b``'s subtree;
a rank forwards only after all of its subtree arrived, and reductions into
one rank chain through its accumulator, children taken in reverse AG time
order (the branch the AllGather served last is reduced first).  Start times
come from the same list schedule as composed candidates (reference:
vericcl/composer/dual.py:412, ``reverse_allgather_schedule``).

The AllGather candidate has ``q`` slices per rank; the ReduceScatter
candidate has ``p·q`` slices per rank of the same slice size, so its request
is the AllGather's with ``p`` times the bytes per rank.
"""
from __future__ import annotations

from collections import defaultdict

from vericcl_b200.composer.compose import NetworkCandidate, NetworkOperation, list_schedule
from vericcl_b200.errors import SemanticError


def reverse_allgather(ag: NetworkCandidate, topology, *, origin: str = "dual") -> NetworkCandidate:
    p, q = ag.rank_count, ag.slice_count
    n = p * q
    trees = defaultdict(list)
    for op in ag.operations:
        if op.kind != "send" or len(op.contributors) != 1:
            raise SemanticError("only broadcast-tree AllGather schedules can be reversed")
        trees[next(iter(op.contributors))].append(op)
    if set(trees) != set(range(n)):
        raise SemanticError("the AllGather schedule does not move every slice")
    ops = []
    for sid in sorted(trees):
        root = sid // q
        children = defaultdict(list)
        seen = set()
        for op in trees[sid]:
            if op.dst_rank in seen or op.dst_rank == root:
                raise SemanticError("slice %d reaches a rank twice; not a tree" % sid)
            seen.add(op.dst_rank)
            children[op.src_rank].append(op)
        if seen != set(range(p)) - {root}:
            raise SemanticError("slice %d does not reach every rank" % sid)
        subtree = {}

        def value_of(rank):
            if rank not in subtree:
                total = frozenset({rank * n + sid})
                for child_op in children.get(rank, ()):
                    total |= value_of(child_op.dst_rank)
                subtree[rank] = total
            return subtree[rank]

        if value_of(root) != frozenset(r * n + sid for r in range(p)):
            raise SemanticError("slice %d's tree is not connected to its owner" % sid)
        accumulator = {}

        def emit(rank):
            # the branch the AllGather served last is reduced first
            for child_op in sorted(children.get(rank, ()), key=lambda o: (-o.priority_time, o.operation_id)):
                child = child_op.dst_rank
                emit(child)
                deps = set()
                if child in accumulator:
                    deps.add(accumulator[child][0])
                if rank in accumulator:
                    deps.add(accumulator[rank][0])
                    base = accumulator[rank][1]
                else:
                    base = frozenset({rank * n + sid})
                carried = subtree[child]
                op_id = "dual:" + child_op.operation_id
                ops.append(NetworkOperation(op_id, "rrc", child, rank, child_op.channel, child_op.stage_id, carried,
                                            base | carried, frozenset(deps), 0.0, sid))
                accumulator[rank] = (op_id, base | carried)

        emit(root)
    timed = list_schedule(ops, topology, ag.slice_size_bytes)
    return NetworkCandidate(p, n, ag.slice_size_bytes, tuple(timed), origin, ag.channels)


def allreduce_from_allgather(ag: NetworkCandidate, topology, *, origin: str = "rs_ag") -> NetworkCandidate:
    """An AllReduce as the reversed AllGather (a ReduceScatter) followed by the AllGather itself.

    Slice ``sid`` is reduced into its owner along the reversed tree, then
    broadcast from the owner along the original tree; the broadcast of a slice
    waits only for that slice's reduction, so the two phases overlap slice by
    slice.  The AllReduce request has ``p·q`` slices per rank.
    """
    rs = reverse_allgather(ag, topology, origin=origin)
    p, q = ag.rank_count, ag.slice_count
    n = p * q
    final = {}
    for op in rs.operations:
        if op.dst_rank == op.index // q and len(op.target_contributors) == p:
            final[op.index] = op.operation_id
    ops = list(rs.operations)
    for op in ag.operations:
        sid = next(iter(op.contributors))
        full = frozenset(r * n + sid for r in range(p))
        deps = {"bcast:" + d for d in op.dependencies}
        if op.src_rank == sid // q:
            if p > 1 and sid not in final:
                raise SemanticError("slice %d has no completed reduction at its owner" % sid)
            if sid in final:
                deps.add(final[sid])
        ops.append(NetworkOperation("bcast:" + op.operation_id, "send", op.src_rank, op.dst_rank, op.channel,
                                    op.stage_id + 1, full, full, frozenset(deps), 0.0, sid))
    timed = list_schedule(ops, topology, ag.slice_size_bytes)
    return NetworkCandidate(p, n, ag.slice_size_bytes, tuple(timed), origin, ag.channels)


def reverse_reduce_scatter(rs: NetworkCandidate, topology, *, origin: str = "dual") -> NetworkCandidate:
    """The other direction: every reduction tree of a ReduceScatter reversed into a broadcast tree.

    The ReduceScatter has ``p·q`` slices per rank; output ``idx`` is reduced
    into rank ``idx // q``.  Reversed, that rank broadcasts its slice ``idx``
    (``q`` slices per rank) to every rank over the same links and channels, a
    relay forwarding only after it received.
    """
    p, n = rs.rank_count, rs.slice_count
    if n % p:
        raise SemanticError("the ReduceScatter slice count must be a multiple of the rank count")
    q = n // p
    parent_of = defaultdict(dict)        # idx -> child -> op
    for op in rs.operations:
        if op.kind != "rrc":
            raise SemanticError("only reduction-tree ReduceScatter schedules can be reversed")
        if op.src_rank in parent_of[op.index]:
            raise SemanticError("slice %d leaves rank %d twice; not a tree" % (op.index, op.src_rank))
        parent_of[op.index][op.src_rank] = op
    ops = []
    for idx in range(n):
        owner = idx // q
        edges = parent_of.get(idx, {})
        if set(edges) != set(range(p)) - {owner}:
            raise SemanticError("slice %d is not reduced from every rank" % idx)
        for start in edges:
            # every parent chain must end at the owner; a cycle among non-owners never delivers
            seen, rank = set(), start
            while rank != owner:
                if rank in seen:
                    raise SemanticError("slice %d's tree is not connected to its owner" % idx)
                seen.add(rank)
                rank = edges[rank].dst_rank
        delivered = {}

        def deliver(rank):
            """Id of the broadcast op that brings slice idx to ``rank`` (None at the owner)."""
            if rank == owner:
                return None
            if rank not in delivered:
                op = edges[rank]
                dep = deliver(op.dst_rank)
                delivered[rank] = "dual:" + op.operation_id
                ops.append(NetworkOperation(delivered[rank], "send", op.dst_rank, rank, op.channel, op.stage_id,
                                            frozenset({idx}), frozenset({idx}),
                                            frozenset({dep}) if dep else frozenset(), -op.priority_time, idx % q))
            return delivered[rank]

        for child in sorted(edges, key=lambda r: (-edges[r].priority_time, r)):
            deliver(child)
    timed = list_schedule(ops, topology, rs.slice_size_bytes)
    return NetworkCandidate(p, q, rs.slice_size_bytes, tuple(timed), origin, rs.channels)
