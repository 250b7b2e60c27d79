"""Candidate paths between ranks (reference: vericcl/topology/paths.py:21)."""
from __future__ import annotations

from collections import deque

from vericcl_b200.topology.model import LinkKey, Topology


def shortest_path_set(topology: Topology, src: int, dst: int, *, limit: int = 16, allowed=None):
    """All minimum-hop paths from ``src`` to ``dst`` (at most ``limit``), as rank tuples."""
    allowed = set(range(topology.rank_count)) if allowed is None else set(allowed)
    dist = {src: 0}
    queue = deque([src])
    while queue:
        node = queue.popleft()
        for nxt in topology.out_neighbors(node):
            if nxt in allowed and nxt not in dist:
                dist[nxt] = dist[node] + 1
                queue.append(nxt)
    if dst not in dist:
        return []
    paths = []

    def walk(node, path):
        if len(paths) >= limit:
            return
        if node == dst:
            paths.append(tuple(path))
            return
        for nxt in topology.out_neighbors(node):
            if nxt in dist and dist[nxt] == dist[node] + 1 and nxt in allowed and dist[nxt] <= dist[dst]:
                walk(nxt, path + [nxt])

    walk(src, [src])
    return paths


def path_links(path):
    return tuple(LinkKey(a, b) for a, b in zip(path, path[1:]))


def path_time_us(topology: Topology, path, payload: int) -> float:
    return sum(topology.link(k).time_us(payload) for k in path_links(path))
