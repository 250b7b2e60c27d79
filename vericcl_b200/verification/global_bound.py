"""Directed information-cut lower bound and no-improvement certificate.

For every non-empty proper rank subset X, data that some rank outside X needs
and that only exists inside X must cross the directed cut X → X̄ at least
once: a whole original slice for data-movement collectives, at least one
slice-sized partial result per logical index for reductions.  The cut's
service rate is bounded by its links and by the shared resources (NVLink
ports, NICs) of the links that cross it.  ``T_lb = max_X bytes(X) /
rate(X) + α_min``.  When ``T_lb`` equals a candidate's exact ``T_pred`` the
candidate is optimal under the model and the run may stop (reference:
vericcl/verification/global_bound.py:59-77).
"""
from __future__ import annotations

from dataclasses import dataclass
from fractions import Fraction
from itertools import combinations

from vericcl_b200.semantics.collective import CollectiveKind, required_outputs

MAX_EXACT_RANKS = 16


@dataclass(frozen=True)
class CutBound:
    lower_bound_us: float
    subset: tuple
    bytes_crossing: int
    rate_bytes_per_us: float
    exact: tuple


def _flow_link(flow_id: str):
    """(src, dst) of a transfer flow id ``kind:src:dst:c<channel>``; None for local work."""
    parts = str(flow_id).split(":")
    if len(parts) >= 3 and parts[0] in ("send", "rrc") and parts[1].isdigit() and parts[2].isdigit():
        return int(parts[1]), int(parts[2])
    return None


def _link_cap(topology, model, key) -> Fraction:
    """Fastest rate (bytes/µs) any operation can reach on link ``key`` under the model: its own service
    curves, and the measured rates of sharing modes for flows on this very link."""
    rates = []
    if model is not None:
        for name in ("link:%d:%d" % (key.src, key.dst), "rrc:%d:%d" % (key.src, key.dst)):
            rates += [1 / Fraction(str(c.beta_us_per_byte)) for c in model.services.get(name, ())]
        for profile in model.profiles:
            rates += [Fraction(str(r)) for flow, r in profile.rates.items() if _flow_link(flow) == (key.src, key.dst)]
    if not rates:
        rates = [Fraction(1) / Fraction(str(topology.links[key].beta_us_per_byte))]
    return max(rates)


def _resource_cap(model, rid, links, nominal) -> Fraction | None:
    """Capacity of a shared resource under the model: its modelled capacity, raised to the largest combined
    rate any measured sharing mode reached through it (a measured mode may beat the nominal share)."""
    # with a model, only the resources it constrains bound the cut (an unmodelled resource never slows a
    # predicted schedule, so using it here could put the bound above T_pred)
    capacity = nominal if model is None else model.resources.get(rid)
    if capacity is None:
        return None
    best = Fraction(str(capacity))
    if model is not None:
        members = {(l.src, l.dst) for l in links}
        for profile in model.profiles:
            through = sum((Fraction(str(r)) for flow, r in profile.rates.items() if _flow_link(flow) in members),
                          Fraction(0))
            best = max(best, through)
    return best


def _rate(topology, inside, model=None):
    """Upper bound on the service rate (bytes/µs) across the cut inside → outside.

    Any family of capacity constraints that covers every crossing link bounds
    the cut rate by the sum of its capacities; the smallest of the families
    tried (all links, any single covering resource, the senders' ports, the
    receivers' ports, a greedy cheapest cover) is returned.  With a cost
    model, link rates are the model's fastest for the link and resource
    capacities the model's, each raised to the largest combined rate a
    measured sharing mode reached through it, so the bound stays valid when
    a measured mode beats a nominal share.
    """
    outside = set(range(topology.rank_count)) - set(inside)
    crossing = {k for k in topology.links if k.src in inside and k.dst in outside}
    if not crossing:
        return Fraction(0)
    caps = {k: _link_cap(topology, model, k) for k in crossing}
    bound = sum(caps.values())
    families = {}
    for rid, res in topology.resources.items():
        members = frozenset(l for l in res.links if l in crossing)
        capacity = _resource_cap(model, rid, res.links, res.capacity_bytes_per_us)
        if members and capacity is not None:
            families[rid] = (members, capacity)
    for rid, (members, cap) in families.items():
        if members == crossing:
            bound = min(bound, cap)
    for side in ("src", "dst"):
        covered, total = set(), Fraction(0)
        for rid, (members, cap) in families.items():
            res = topology.resources[rid]
            if all(getattr(l, side) == getattr(next(iter(res.links)), side) for l in res.links):
                covered |= members
                total += cap
        if covered == crossing:
            bound = min(bound, total)
    # greedy cover: resources or single links, cheapest capacity per newly covered link first
    uncovered, total = set(crossing), Fraction(0)
    options = list(families.values()) + [(frozenset({k}), caps[k]) for k in crossing]
    while uncovered:
        members, cap = min(options, key=lambda o: cap_per(o, uncovered))
        if not members & uncovered:
            break
        uncovered -= members
        total += cap
    if not uncovered:
        bound = min(bound, total)
    return bound


def cap_per(option, uncovered):
    members, cap = option
    gain = len(members & uncovered)
    return cap / gain if gain else Fraction(10 ** 18)


def _required_bytes(request, inside):
    spec = request.collective
    p, n = request.rank_count, request.hyperparameters.slice_count
    s = request.hyperparameters.slice_size_bytes
    outside = set(range(p)) - set(inside)
    need = set()
    for slot, contributors in required_outputs(spec, p, n).items():
        if slot.rank not in outside:
            continue
        from_inside = {c for c in contributors if c // n in inside}
        if not from_inside:
            continue
        if spec.kind in (CollectiveKind.ALL_REDUCE, CollectiveKind.REDUCE, CollectiveKind.REDUCE_SCATTER):
            need.add(("partial", min(contributors) % n))
        else:
            need.update(("slice", c) for c in from_inside)
    return len(need) * s


def certify_global_cut(request, topology, model=None):
    p = request.rank_count
    if p > MAX_EXACT_RANKS:
        return None
    alphas = [l.alpha_us for l in topology.links.values()]
    if model is not None:
        alphas += [c.alpha_us for segs in model.services.values() for c in segs]
    alpha = min(alphas, default=0.0)
    best = None
    for size in range(1, p):
        for inside in combinations(range(p), size):
            rate = _rate(topology, set(inside), model)
            need = _required_bytes(request, set(inside))
            if need == 0 or rate == 0:
                continue
            t = Fraction(need) / rate + Fraction(str(alpha))
            if best is None or t > best[0]:
                best = (t, inside, need, rate)
    if best is None:
        return CutBound(0.0, (), 0, 0.0, (0, 1))
    t, inside, need, rate = best
    return CutBound(float(t), tuple(inside), need, float(rate), (t.numerator, t.denominator))


def check_global_cut(bound: CutBound, t_pred_us: float, *, tolerance: float = 1e-9) -> bool:
    """True when the bound certifies that no schedule beats ``t_pred_us`` under the model."""
    return bound is not None and t_pred_us is not None and t_pred_us <= bound.lower_bound_us * (1 + tolerance)
