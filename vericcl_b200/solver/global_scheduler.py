"""Global channel assignment: every transfer's channel chosen with the whole schedule in view.

A channel is a thread-block pair: transfers on the same (sender, receiver,
channel) run one after another.  The composer deals channels round-robin per
directed link, which ignores when each transfer becomes ready.  Here the
transfers are list-scheduled in dependency order (ties by their current
priority); each takes, among the link's allowed channels, the one on which it
can start earliest, and among equally early ones the channel carrying the
least work so far, so channels of a link stay balanced.  Channel budgets per
rank are respected: a rank may open at most ``max_blocks_per_rank`` distinct
(peer, direction, channel) thread blocks, the runtime limit the admission
checks enforce.  Every (peer, direction) a rank needs keeps one block in
reserve, so extra channels early in the schedule never crowd out a
connection that opens later; below one block per connection each
connection gets exactly one (reference: vericcl/solver/global_scheduler.py:113-229, which
assigns channels and resource slots for the whole candidate at once).
"""
from __future__ import annotations

import heapq
from dataclasses import replace

from vericcl_b200.composer.compose import NetworkCandidate, list_schedule
from vericcl_b200.topology.model import LinkKey


def assign_channels(candidate: NetworkCandidate, topology, channels: int, *,
                    max_blocks_per_rank: int = 216) -> NetworkCandidate:
    ops = {op.operation_id: op for op in candidate.operations}
    if channels <= 1 or not ops:
        return candidate
    size = candidate.slice_size_bytes
    indeg = {k: len(op.dependencies) for k, op in ops.items()}
    succ = {k: [] for k in ops}
    for op in ops.values():
        for d in op.dependencies:
            succ[d].append(op.operation_id)
    ready_at = dict.fromkeys(ops, 0.0)
    heap = [(op.priority_time, k) for k, op in ops.items() if indeg[k] == 0]
    heapq.heapify(heap)
    free, work = {}, {}           # (src, dst, channel) -> time it frees up / work assigned so far
    blocks = {}                   # rank -> set of (peer, direction, channel) thread blocks in use
    # rank -> (peer, direction) pairs it must open at least one block for, and those it has opened
    needed, opened = {}, {}
    for op in ops.values():
        needed.setdefault(op.src_rank, set()).add((op.dst_rank, "send"))
        needed.setdefault(op.dst_rank, set()).add((op.src_rank, "recv"))

    def admits(rank, pair, channel):
        if (pair + (channel,)) in blocks.get(rank, ()):
            return True
        if pair not in opened.get(rank, ()):
            return True           # a connection's first block: reserved for it from the start
        # an extra channel: it must leave one block for every pair the rank has not opened yet
        unopened = len(needed[rank] - opened.get(rank, set()))
        return len(blocks.get(rank, ())) + unopened + 1 <= max_blocks_per_rank

    chosen = {}
    while heap:
        _, key = heapq.heappop(heap)
        op = ops[key]
        link = topology.link(LinkKey(op.src_rank, op.dst_rank))
        dur = link.time_us(size)
        limit = max(1, min(channels, link.max_channels))
        best = None
        for c in range(limit):
            conn = (op.src_rank, op.dst_rank, c)
            if not (admits(op.src_rank, (op.dst_rank, "send"), c) and admits(op.dst_rank, (op.src_rank, "recv"), c)):
                continue
            start = max(ready_at[key], free.get(conn, 0.0))
            rank_key = (start, work.get(conn, 0.0), c)
            if best is None or rank_key < best[0]:
                best = (rank_key, c)
        c = best[1] if best is not None else 0      # unreachable: a connection's open channel is always admitted
        conn = (op.src_rank, op.dst_rank, c)
        start = max(ready_at[key], free.get(conn, 0.0))
        free[conn] = start + dur
        work[conn] = work.get(conn, 0.0) + dur
        blocks.setdefault(op.src_rank, set()).add((op.dst_rank, "send", c))
        blocks.setdefault(op.dst_rank, set()).add((op.src_rank, "recv", c))
        opened.setdefault(op.src_rank, set()).add((op.dst_rank, "send"))
        opened.setdefault(op.dst_rank, set()).add((op.src_rank, "recv"))
        chosen[key] = c
        for nxt in succ[key]:
            indeg[nxt] -= 1
            ready_at[nxt] = max(ready_at[nxt], start + dur)
            if indeg[nxt] == 0:
                heapq.heappush(heap, (ops[nxt].priority_time, nxt))
    relabelled = [replace(op, channel=chosen.get(op.operation_id, op.channel)) for op in candidate.operations]
    timed = list_schedule(relabelled, topology, size)
    return replace(candidate, operations=tuple(timed), origin=candidate.origin + "+channels",
                   channels=max(chosen.values(), default=0) + 1)
