"""Lower bounds on T_pred for pruning parameter choices before synthesis.

Dependency bound: every output slot needs each of its contributing slices,
which start on their source rank, so some chain of transfers must carry a
slice (or a partial result of at least one slice) from the source to the
output rank.  Each hop of such a chain is an operation of at least one
slice: it pays its startup α and moves S bytes at no more than the fastest
rate the cost model allows for that link (its own 1/β or any measured
concurrency profile).  The bound is the largest, over required (source,
output rank) pairs, shortest-path time with those hop times; it holds for
every schedule with slice size S under the model, because contention and
waits only add time (reference: vericcl/solver/lower_bounds.py:134-186,
``dependency_time_lower_bound``).  The throughput side is the directed-cut
bound of :mod:`vericcl_b200.verification.global_bound`.
"""
from __future__ import annotations

import heapq
from fractions import Fraction

from vericcl_b200.semantics.collective import required_outputs, source_rank
from vericcl_b200.topology.model import LinkKey


def _fastest_profile_rate(model) -> Fraction:
    best = Fraction(0)
    for profile in getattr(model, "profiles", ()):
        for rate in profile.rates.values():
            best = max(best, Fraction(str(rate)))
    return best


def hop_time(model, topology, src: int, dst: int, size: int):
    """Smallest time of one operation moving ``size`` bytes from ``src`` to ``dst`` (None: no link)."""
    if not topology.has_link(src, dst):
        return None
    fastest = _fastest_profile_rate(model) if model is not None else Fraction(0)
    best = None
    for key in ("link:%d:%d" % (src, dst), "rrc:%d:%d" % (src, dst)):
        cost = model.service_for(key, size) if model is not None else None
        if cost is None:
            continue
        rate = max(1 / Fraction(str(cost.beta_us_per_byte)), fastest)
        t = Fraction(str(cost.alpha_us)) + Fraction(size) / rate
        best = t if best is None else min(best, t)
    if best is None:
        link = topology.link(LinkKey(src, dst))
        rate = max(1 / Fraction(str(link.beta_us_per_byte)), fastest)
        best = Fraction(str(link.alpha_us)) + Fraction(size) / rate
    return best


def _shortest_from(model, topology, src: int, size: int) -> dict:
    dist = {src: Fraction(0)}
    heap = [(Fraction(0), src)]
    while heap:
        d, u = heapq.heappop(heap)
        if d > dist.get(u, d):
            continue
        for v in topology.out_neighbors(u):
            w = hop_time(model, topology, u, v, size)
            if w is None:
                continue
            nd = d + w
            if v not in dist or nd < dist[v]:
                dist[v] = nd
                heapq.heappush(heap, (nd, v))
    return dist


def dependency_lower_bound(request, topology, model, slice_bytes: int | None = None) -> Fraction:
    """Lower bound (µs) on T_pred of any schedule of ``request`` with slices of ``slice_bytes``."""
    size = slice_bytes or request.hyperparameters.slice_size_bytes
    total = request.hyperparameters.total_size_bytes
    slices = max(1, total // size)
    p = request.rank_count
    pairs = set()
    for slot, contributors in required_outputs(request.collective, p, slices).items():
        for c in contributors:
            src = source_rank(c, slices)
            if src != slot.rank:
                pairs.add((src, slot.rank))
    if not pairs:
        return Fraction(0)
    dists = {}
    bound = Fraction(0)
    for src, dst in sorted(pairs):
        if src not in dists:
            dists[src] = _shortest_from(model, topology, src, size)
        d = dists[src].get(dst)
        if d is None:
            continue   # unreachable pairs are the semantic checks' business, not the bound's
        bound = max(bound, d)
    return bound
