"""Hierarchy search: rank partitions, rails, gateway plans, streamed from coarse to fine.

The ``hierarchy`` method composes an AllReduce or AllGather from stages on
communication groups (reference: vericcl/planner/group_search.py:81-547 and
vericcl/planner/hierarchy.py:497,713).  This module decides *which* groups and
*which* members carry the inter-group traffic, for any topology the request
describes:

* **Partitions.**  Topology nodes, explicit ``topology.groups``, and for every
  distinct link-cost level the connected components of the links at most that
  slow.  Groups may differ in size.
* **Rails** (:func:`discover_rails`).  For every slice owner (AllReduce) or
  source (AllGather) one member of every group takes part in the inter-group
  stage.  The owner's own group is represented by the owner; every other
  group by the member reached most cheaply from the owner (β of the direct
  link, plus the β of its shared resources), breaking ties so that the owners
  of one group spread over different members.  Groups with gateways
  (``nodes[].gateways``) choose among their gateways only.
* **Gateway plans.**  One fixed member per group (its first gateway, else its
  lowest rank) carries every slice; the inter-group reduction ends at the
  owner group's gateway.
* **Streaming.**  Every (partition, rail mode) pair is a coarse candidate with
  a cheap score: the busiest shared resource's load (bytes × β summed over
  the plan's transfers on it, star trees inside every stage) plus the α of
  its stage chain.  :class:`CandidateStream` builds plan DAGs lazily in score
  order, so the workflow synthesizes (the fine, per-node solve) only the
  most promising few.
"""
from __future__ import annotations

import heapq
from dataclasses import dataclass, field, replace

from vericcl_b200.planner.direct import build_direct_plan, slice_owner
from vericcl_b200.planner.model import PlanDAG, PlanEdge, PlanNode, PlanningMode, StageInterface
from vericcl_b200.semantics.collective import CollectiveKind, OutputSlot
from vericcl_b200.topology.model import LinkKey

SUPPORTED = (CollectiveKind.ALL_REDUCE, CollectiveKind.ALL_GATHER)


def _components(ranks: int, joined) -> tuple:
    parent = list(range(ranks))

    def root(x):
        while parent[x] != x:
            parent[x] = parent[parent[x]]
            x = parent[x]
        return x

    for a, b in joined:
        ra, rb = root(a), root(b)
        if ra != rb:
            parent[ra] = rb
    comps = {}
    for r in range(ranks):
        comps.setdefault(root(r), []).append(r)
    return tuple(sorted(tuple(sorted(c)) for c in comps.values()))


def _strongly_connected(topology, group) -> bool:
    """Every member reaches every other over links inside the group (a stage stays inside its group)."""
    members = set(group)
    for start in (group[0],):
        for reverse in (False, True):
            seen, todo = {start}, [start]
            while todo:
                v = todo.pop()
                nbrs = topology.in_neighbors(v) if reverse else topology.out_neighbors(v)
                for w in nbrs:
                    if w in members and w not in seen:
                        seen.add(w)
                        todo.append(w)
            if seen != members:
                return False
    return True


def partition_candidates(topology) -> list:
    """Distinct partitions into at least two strongly connected groups, most structured first (sizes may differ)."""
    out = []

    def add(part):
        part = tuple(tuple(sorted(g)) for g in part)
        part = tuple(sorted(part))
        if 1 < len(part) < topology.rank_count + 1 and part not in out and \
                sorted(r for g in part for r in g) == list(range(topology.rank_count)) and \
                all(_strongly_connected(topology, g) for g in part):
            out.append(part)

    if len(topology.nodes) > 1:
        add([n.ranks for n in topology.nodes])
    if topology.groups:
        add(topology.groups)
    levels = sorted({link.beta_us_per_byte for link in topology.links.values()})
    for level in levels[:-1]:
        comps = _components(topology.rank_count, [(k.src, k.dst) for k, l in topology.links.items()
                                                  if l.beta_us_per_byte <= level])
        if len(comps) < topology.rank_count:
            add(comps)
    return out


def _edge_cost(topology, a: int, b: int) -> float:
    """β of the link a→b plus the β implied by each shared resource on it (inf when there is no link)."""
    if a == b:
        return 0.0
    if not topology.has_link(a, b):
        return float("inf")
    link = topology.link(LinkKey(a, b))
    cost = link.beta_us_per_byte
    for rid in link.resource_ids:
        res = topology.resources.get(rid)
        if res is not None:
            cost = max(cost, 1.0 / res.capacity_bytes_per_us)
    return cost


def _gateways(topology, group) -> tuple:
    members = set(group)
    gws = []
    for node in topology.nodes:
        gws.extend(g for g in getattr(node, "gateways", ()) if g in members)
    return tuple(sorted(set(gws))) or tuple(group)


def discover_rails(topology, groups, owners) -> dict:
    """``{owner: (member of group 0, member of group 1, ...)}`` with the owner representing its own group."""
    group_of = {r: gi for gi, g in enumerate(groups) for r in g}
    load = {}                         # member -> owners it already serves (spreads ties)
    rails = {}
    for owner in owners:
        members = []
        for gi, g in enumerate(groups):
            if gi == group_of[owner]:
                members.append(owner)
                continue
            pool = _gateways(topology, g)
            best = min(pool, key=lambda m: (_edge_cost(topology, owner, m) + _edge_cost(topology, m, owner),
                                            load.get(m, 0), (m - owner) % topology.rank_count))
            load[best] = load.get(best, 0) + 1
            members.append(best)
        rails[owner] = tuple(members)
    return rails


def gateway_rails(topology, groups, owners) -> dict:
    """Every owner's slice crosses groups through one fixed gateway per group (the owner's group included)."""
    gws = tuple(_gateways(topology, g)[0] for g in groups)
    return {o: gws for o in owners}


def build_group_plan(request, topology, groups, rails: dict, *, mode: str = "rails") -> PlanDAG:
    """Stage DAG over ``groups`` with the given inter-group members per owner / source.

    AllReduce, per slice: reduce inside every group into its rail member →
    reduce across groups into the owner group's rail member → broadcast back
    across groups → broadcast inside every group.  AllGather, per source
    slice: move it to the source group's rail member (when that is not the
    source), broadcast across groups, broadcast inside every group.
    """
    spec = request.collective
    p, n = request.rank_count, request.hyperparameters.slice_count
    group_of = {r: gi for gi, g in enumerate(groups) for r in g}
    nodes, edges = [], []
    if spec.kind is CollectiveKind.ALL_REDUCE:
        for index in range(n):
            owner, _ = slice_owner(index, n, p)
            members = rails[owner]
            root = members[group_of[owner]]
            full = frozenset(r * n + index for r in range(p))
            partial = {}
            for gi, g in enumerate(groups):
                m = members[gi]
                contrib = frozenset(r * n + index for r in g)
                partial[m] = contrib
                nodes.append(PlanNode("g-rs-%d-%08d" % (gi, index), 0, CollectiveKind.REDUCE, tuple(g), m,
                                      StageInterface({OutputSlot(r, index): frozenset({r * n + index}) for r in g}),
                                      StageInterface({OutputSlot(m, index): contrib})))
            cross = "g-xr-%08d" % index
            nodes.append(PlanNode(cross, 1, CollectiveKind.REDUCE, tuple(members), root,
                                  StageInterface({OutputSlot(m, index): c for m, c in partial.items()}),
                                  StageInterface({OutputSlot(root, index): full})))
            edges.extend(PlanEdge("g-rs-%d-%08d" % (gi, index), cross) for gi in range(len(groups)))
            bcast = "g-xb-%08d" % index
            nodes.append(PlanNode(bcast, 2, CollectiveKind.BROADCAST, tuple(members), root,
                                  StageInterface({OutputSlot(root, index): full}),
                                  StageInterface({OutputSlot(m, index): full for m in members})))
            edges.append(PlanEdge(cross, bcast))
            for gi, g in enumerate(groups):
                m = members[gi]
                nid = "g-ag-%d-%08d" % (gi, index)
                nodes.append(PlanNode(nid, 3, CollectiveKind.BROADCAST, tuple(g), m,
                                      StageInterface({OutputSlot(m, index): full}),
                                      StageInterface({OutputSlot(r, index): full for r in g})))
                edges.append(PlanEdge(bcast, nid))
    elif spec.kind is CollectiveKind.ALL_GATHER:
        for src in range(p):
            members = rails[src]
            head = members[group_of[src]]
            for index in range(n):
                sid = src * n + index
                value = frozenset({sid})
                first_stage, start_slot = 0, OutputSlot(src, index)
                prev = None
                if head != src:
                    # bring the slice to its group's inter-group member first
                    prev = "g-up-%08d" % sid
                    g = groups[group_of[src]]
                    nodes.append(PlanNode(prev, 0, CollectiveKind.BROADCAST, tuple(g), src,
                                          StageInterface({OutputSlot(src, index): value}),
                                          StageInterface({OutputSlot(r, sid): value for r in g})))
                    first_stage, start_slot = 1, OutputSlot(head, sid)
                cross = "g-xb-%08d" % sid
                others = tuple(m for gi, m in enumerate(members) if gi != group_of[src])
                nodes.append(PlanNode(cross, first_stage, CollectiveKind.BROADCAST, (head,) + others, head,
                                      StageInterface({start_slot: value}),
                                      StageInterface({OutputSlot(m, sid): value for m in (head,) + others})))
                if prev is not None:
                    edges.append(PlanEdge(prev, cross))
                for gi, g in enumerate(groups):
                    if gi == group_of[src] and prev is not None:
                        continue          # the source group already holds the slice everywhere
                    m = members[gi]
                    nid = "g-ag-%d-%08d" % (gi, sid)
                    slot = OutputSlot(m, index if m == src else sid)
                    nodes.append(PlanNode(nid, first_stage + 1, CollectiveKind.BROADCAST, tuple(g), m,
                                          StageInterface({slot: value}),
                                          StageInterface({OutputSlot(r, sid): value for r in g})))
                    edges.append(PlanEdge(cross, nid))
    else:
        return build_direct_plan(request, topology, reason="hierarchy_unsupported_collective")
    return PlanDAG(spec, p, n, tuple(nodes), tuple(edges), PlanningMode.HIERARCHY,
                   "%s groups=%s" % (mode, groups), {"groups": [list(g) for g in groups], "rail_mode": mode})


def coarse_score(request, topology, groups, rails) -> float:
    """Busiest-resource load plus the α of the stage chain, for one slice size S (µs).

    Every stage is costed as a star (all its transfers leave or reach the
    stage's root directly); the load of a resource is the sum of S / capacity
    over the transfers that cross it, a link without a shared resource
    counting as its own resource of capacity 1/β.
    """
    p, n = request.rank_count, request.hyperparameters.slice_count
    size = request.hyperparameters.slice_size_bytes or 1
    group_of = {r: gi for gi, g in enumerate(groups) for r in g}
    load = {}

    def transfer(a, b) -> float:
        """Add one S-byte transfer a→b to the loads; return its α."""
        if a == b:
            return 0.0
        if not topology.has_link(a, b):
            return float("inf")
        link = topology.link(LinkKey(a, b))
        for key in ("link:%d:%d" % (a, b),) + tuple(link.resource_ids):
            res = topology.resources.get(key)
            cap = res.capacity_bytes_per_us if res is not None else 1.0 / link.beta_us_per_byte
            load[key] = load.get(key, 0.0) + size / cap
        return link.alpha_us

    chain = 0.0
    if request.collective.kind is CollectiveKind.ALL_REDUCE:
        for index in range(n):
            owner, _ = slice_owner(index, n, p)
            members = rails[owner]
            root = members[group_of[owner]]
            up = max((transfer(r, members[gi]) for gi, g in enumerate(groups) for r in g), default=0.0)
            down = max((transfer(members[gi], r) for gi, g in enumerate(groups) for r in g), default=0.0)
            xr = max((transfer(m, root) for m in members), default=0.0)
            xb = max((transfer(root, m) for m in members), default=0.0)
            chain = max(chain, up + xr + xb + down)
    else:
        for src in range(p):
            members = rails[src]
            head = members[group_of[src]]
            for _ in range(n):
                up = max((transfer(src, r) for r in groups[group_of[src]]), default=0.0) if head != src else 0.0
                xb = max((transfer(head, m) for m in members), default=0.0)
                down = max((transfer(members[gi], r) for gi, g in enumerate(groups)
                            if not (gi == group_of[src] and head != src) for r in g), default=0.0)
                chain = max(chain, up + xb + down)
    return max(load.values(), default=0.0) + chain


@dataclass(order=True)
class _Coarse:
    score: float
    seq: int
    groups: tuple = field(compare=False)
    mode: str = field(compare=False)
    rails: dict = field(compare=False)


class CandidateStream:
    """Hierarchy plans of a request, best coarse score first, built only when asked for."""

    def __init__(self, request, topology):
        self.request, self.topology = request, topology
        self._heap: list = []
        if request.collective.kind not in SUPPORTED:
            return
        p = request.rank_count
        seq = 0
        for groups in partition_candidates(topology):
            for mode, rails_of in (("rails", discover_rails), ("gateways", gateway_rails)):
                rails = rails_of(topology, groups, range(p))
                score = coarse_score(request, topology, groups, rails)
                if score == float("inf"):
                    continue          # some stage would need a link the topology does not have
                heapq.heappush(self._heap, _Coarse(score, seq, groups, mode, rails))
                seq += 1

    def __iter__(self):
        seen = set()
        while self._heap:
            item = heapq.heappop(self._heap)
            key = (item.groups, tuple(sorted(item.rails.items())))
            if key in seen:
                continue          # a gateway plan that coincides with the rail plan
            seen.add(key)
            plan = build_group_plan(self.request, self.topology, item.groups, item.rails, mode=item.mode)
            yield replace(plan, metadata=dict(plan.metadata, coarse_score_us=item.score))

    def scores(self) -> list:
        return sorted((c.score, c.mode, c.groups) for c in self._heap)
