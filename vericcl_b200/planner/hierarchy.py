"""Hierarchical plans: group-local stages around an inter-group (rail) stage.

For AllReduce over groups G_1..G_k (nodes, explicit ``topology.groups`` or
cost-threshold components): (0) reduce each slice inside every group into the
group's rail member, (1) reduce across groups among rail members into the
slice owner, (2) broadcast across groups among rail members, (3) broadcast
inside every group.  AllGather uses the last two stages per source slice
(gather to the source group's rail is not needed: the source is its own rail
member).  Rails pair the i-th member of every group (reference:
vericcl/planner/group_search.py:81-547).  With a single group the direct
plan is returned.
"""
from __future__ import annotations

from vericcl_b200.planner.direct import build_direct_plan, slice_owner
from vericcl_b200.planner.model import PlanDAG, PlanEdge, PlanNode, PlanningMode, StageInterface
from vericcl_b200.semantics.collective import CollectiveKind, OutputSlot


def candidate_partitions(request, topology):
    """Rank partitions to try, most structured first."""
    out = []
    if len(topology.nodes) > 1:
        out.append(tuple(tuple(n.ranks) for n in topology.nodes))
    if topology.groups:
        groups = tuple(tuple(g) for g in topology.groups)
        if sorted(r for g in groups for r in g) == list(range(topology.rank_count)) and groups not in out:
            out.append(groups)
    # cost-threshold components: ranks joined by links at least as fast as the fastest link / 2
    if topology.links:
        best = min(l.beta_us_per_byte for l in topology.links.values())
        parent = list(range(topology.rank_count))

        def find(x):
            while parent[x] != x:
                parent[x] = parent[parent[x]]
                x = parent[x]
            return x

        for key, link in topology.links.items():
            if link.beta_us_per_byte <= 2 * best:
                a, b = find(key.src), find(key.dst)
                if a != b:
                    parent[a] = b
        comps = {}
        for r in range(topology.rank_count):
            comps.setdefault(find(r), []).append(r)
        part = tuple(tuple(sorted(c)) for c in sorted(comps.values()))
        if 1 < len(part) < topology.rank_count and part not in out:
            out.append(part)
    return out


def _equal_groups(groups):
    return len({len(g) for g in groups}) == 1


def build_group_plan(request, topology, groups) -> PlanDAG:
    spec = request.collective
    p = request.rank_count
    n = request.hyperparameters.slice_count
    k = len(groups)
    size = len(groups[0])
    group_of = {r: gi for gi, g in enumerate(groups) for r in g}
    pos_of = {r: g.index(r) for g in groups for r in g}
    nodes, edges = [], []
    if spec.kind is CollectiveKind.ALL_REDUCE:
        for index in range(n):
            owner, _ = slice_owner(index, n, p)
            rail = pos_of[owner]
            rails = tuple(g[rail] for g in groups)
            full = frozenset(r * n + index for r in range(p))
            partial = {}
            for gi, g in enumerate(groups):
                member = g[rail]
                contrib = frozenset(r * n + index for r in g)
                partial[member] = contrib
                nid = "h-rs-g%d-a%08d" % (gi, index)
                nodes.append(PlanNode(nid, 0, CollectiveKind.REDUCE, tuple(g), member,
                                      StageInterface({OutputSlot(r, index): frozenset({r * n + index}) for r in g}),
                                      StageInterface({OutputSlot(member, index): contrib})))
            cross = "h-xr-a%08d" % index
            nodes.append(PlanNode(cross, 1, CollectiveKind.REDUCE, rails, owner,
                                  StageInterface({OutputSlot(m, index): c for m, c in partial.items()}),
                                  StageInterface({OutputSlot(owner, index): full})))
            for gi in range(k):
                edges.append(PlanEdge("h-rs-g%d-a%08d" % (gi, index), cross))
            bcast = "h-xb-a%08d" % index
            nodes.append(PlanNode(bcast, 2, CollectiveKind.BROADCAST, rails, owner,
                                  StageInterface({OutputSlot(owner, index): full}),
                                  StageInterface({OutputSlot(m, index): full for m in rails})))
            edges.append(PlanEdge(cross, bcast))
            for gi, g in enumerate(groups):
                member = g[rail]
                nid = "h-ag-g%d-a%08d" % (gi, index)
                nodes.append(PlanNode(nid, 3, CollectiveKind.BROADCAST, tuple(g), member,
                                      StageInterface({OutputSlot(member, index): full}),
                                      StageInterface({OutputSlot(r, index): full for r in g})))
                edges.append(PlanEdge(bcast, nid))
    elif spec.kind is CollectiveKind.ALL_GATHER:
        for src in range(p):
            rail = pos_of[src]
            rails = tuple(g[rail] for g in groups)
            for index in range(n):
                sid = src * n + index
                value = frozenset({sid})
                cross = "h-xb-s%08d" % sid
                nodes.append(PlanNode(cross, 0, CollectiveKind.BROADCAST, rails, src,
                                      StageInterface({OutputSlot(src, index): value}),
                                      StageInterface({OutputSlot(m, sid): value for m in rails})))
                for gi, g in enumerate(groups):
                    member = g[rail]
                    nid = "h-ag-g%d-s%08d" % (gi, sid)
                    nodes.append(PlanNode(nid, 1, CollectiveKind.BROADCAST, tuple(g), member,
                                          StageInterface({OutputSlot(member, sid if member != src else index): value}),
                                          StageInterface({OutputSlot(r, sid) for r in g} and
                                                         {OutputSlot(r, sid): value for r in g})))
                    edges.append(PlanEdge(cross, nid))
    else:
        return build_direct_plan(request, topology, reason="hierarchy_unsupported_collective")
    return PlanDAG(spec, p, n, tuple(nodes), tuple(edges), PlanningMode.HIERARCHY, "groups=%s" % (groups,),
                   {"groups": [list(g) for g in groups]})


def plan_hierarchy(request, topology) -> PlanDAG:
    """Best-structured plan: the first equal-size multi-group partition, else direct."""
    for groups in candidate_partitions(request, topology):
        if len(groups) > 1 and _equal_groups(groups) and request.collective.kind in (
                CollectiveKind.ALL_REDUCE, CollectiveKind.ALL_GATHER):
            return build_group_plan(request, topology, groups)
    return build_direct_plan(request, topology, reason="single_group")


def enumerate_hierarchy_plans(request, topology):
    """All hierarchy candidates (lazy), followed by the direct plan."""
    for groups in candidate_partitions(request, topology):
        if len(groups) > 1 and _equal_groups(groups) and request.collective.kind in (
                CollectiveKind.ALL_REDUCE, CollectiveKind.ALL_GATHER):
            yield build_group_plan(request, topology, groups)
    yield build_direct_plan(request, topology, reason="direct_fallback")
