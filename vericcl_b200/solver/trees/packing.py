"""Bandwidth packing of broadcast arborescences (the fast constructive path).

Edmonds' branching theorem: a root can broadcast ``k`` unit slices to every
destination over edge-disjoint arborescences when every destination is
``k``-connected from the root.  With per-edge capacities ``c(e) = T / β(e)``
(slices an edge can carry within a time budget ``T``), the smallest feasible
``T`` is found by binary search over rational time units with an integer
max-flow rooted-cut test; the arborescences are then extracted greedily as
minimum arborescences on the residual capacities (reference:
vericcl/solver/trees/packing.py:19-51 and batch.py:36-154, which use the same
theorem).  Used when no shared resource constrains the links; otherwise
:mod:`columns` solves the general problem.
"""
from __future__ import annotations

from fractions import Fraction

import networkx as nx

from vericcl_b200.errors import SolverError
from vericcl_b200.topology.model import LinkKey


def _capacity_graph(topology, allowed, budget: Fraction, slice_bytes: int):
    g = nx.DiGraph()
    for key, link in topology.links.items():
        if key.src not in allowed or key.dst not in allowed:
            continue
        per_slice = Fraction(str(link.beta_us_per_byte)) * slice_bytes
        cap = int(budget / per_slice) if per_slice > 0 else 0
        if cap > 0:
            g.add_edge(key.src, key.dst, capacity=cap)
    return g


def rooted_cut_feasible(graph, root, dests, k: int) -> bool:
    """True when every destination has ``k`` edge-disjoint paths from ``root``."""
    for d in dests:
        if d not in graph or root not in graph:
            return False
        if nx.maximum_flow_value(graph, root, d, capacity="capacity") < k:
            return False
    return True


def min_time_budget(topology, root, dests, k: int, slice_bytes: int, allowed=None, iterations: int = 40):
    """Smallest per-link time budget (µs) that admits ``k`` disjoint arborescences."""
    allowed = set(range(topology.rank_count)) if allowed is None else set(allowed)
    worst = max(Fraction(str(l.beta_us_per_byte)) for l in topology.links.values()) * slice_bytes
    hi = worst * k
    if not rooted_cut_feasible(_capacity_graph(topology, allowed, hi, slice_bytes), root, dests, k):
        raise SolverError("destinations are not reachable from root %d" % root)
    lo = Fraction(0)
    for _ in range(iterations):
        mid = (lo + hi) / 2
        if rooted_cut_feasible(_capacity_graph(topology, allowed, mid, slice_bytes), root, dests, k):
            hi = mid
        else:
            lo = mid
        if hi - lo <= hi / 1000:
            break
    return hi


def extract_arborescences(topology, root, dests, k: int, slice_bytes: int, budget: Fraction, allowed=None):
    """Greedy extraction of ``k`` arborescences within ``budget`` (returns [(edges, count)])."""
    allowed = set(range(topology.rank_count)) if allowed is None else set(allowed)
    g = _capacity_graph(topology, allowed, budget, slice_bytes)
    trees = []
    remaining = k
    while remaining > 0:
        h = nx.DiGraph()
        for a, b, data in g.edges(data=True):
            if data["capacity"] > 0 and b != root:
                used = 1.0 / data["capacity"]
                h.add_edge(a, b, weight=used + 1e-3)
        try:
            arb = nx.minimum_spanning_arborescence(h.subgraph(nx.descendants(h, root) | {root}), attr="weight")
        except (nx.NetworkXException, ValueError):
            raise SolverError("arborescence extraction failed; capacities exhausted")
        if not set(dests) <= set(arb.nodes):
            raise SolverError("arborescence does not span the destinations")
        # prune branches that reach no destination
        keep = set()
        for d in dests:
            node = d
            while node != root:
                keep.add(node)
                node = next(iter(arb.predecessors(node)))
        edges = tuple(sorted((a, b) for a, b in arb.edges() if b in keep))
        bottleneck = min(g[a][b]["capacity"] for a, b in edges)
        count = min(remaining, bottleneck)
        for a, b in edges:
            g[a][b]["capacity"] -= count
        trees.append((edges, count))
        remaining -= count
    return trees


def pack_bandwidth(topology, root, dests, k: int, slice_bytes: int, allowed=None):
    """Return (time budget, [(edges, slice count), ...]) for broadcasting ``k`` slices."""
    if not dests:
        return Fraction(0), []
    budget = min_time_budget(topology, root, dests, k, slice_bytes, allowed)
    for scale in (1, Fraction(5, 4), Fraction(3, 2), 2, 4):
        try:
            return budget * scale, extract_arborescences(topology, root, dests, k, slice_bytes, budget * scale,
                                                         allowed)
        except SolverError:
            continue
    raise SolverError("could not extract arborescences for root %d" % root)


def uses_shared_resources(topology) -> bool:
    return any(len(r.links) > 1 for r in topology.resources.values())


def edge_key(a, b):
    return LinkKey(a, b)
