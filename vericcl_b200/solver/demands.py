"""Plan nodes → transfer demands with candidate trees.

A broadcast demand moves one value from its root to every other holder of an
output slot; a reduce demand combines the group members' values into the
root.  Candidate trees are enumerated per demand (direct star, BFS shortest
path tree, binomial tree, chain) over the links the node may use; the route
MILP picks one per demand (reference: vericcl/solver/demands.py:57-559 and
vericcl/solver/templates.py:856 for the isomorphic-template grouping, which
here is the ``signature`` of a demand).
"""
from __future__ import annotations

import heapq
from collections import deque
from dataclasses import dataclass, field

from vericcl_b200.errors import SemanticError
from vericcl_b200.planner.model import PlanDAG, PlanNode
from vericcl_b200.semantics.collective import CollectiveKind
from vericcl_b200.topology.model import LinkKey, Topology


@dataclass(frozen=True)
class Tree:
    """Directed tree edges (parent, child) for broadcast, (child, parent) for reduce."""

    name: str
    edges: tuple                 # ((src, dst), ...) in data-flow direction
    depth: int


@dataclass(frozen=True)
class TransferDemand:
    demand_id: str
    node_id: str
    stage_id: int
    kind: str                    # broadcast | reduce
    root: int
    members: tuple               # broadcast: destinations; reduce: sources (excluding root)
    index: int                   # logical slice position
    contributors: dict = field(default_factory=dict, hash=False, compare=False)
    target: frozenset = frozenset()
    local: bool = False          # broadcast to the root's own output slot only
    candidates: tuple = ()

    def signature(self):
        """Shape of the demand independent of slice index (template key)."""
        return (self.kind, self.root, self.members, tuple(t.edges for t in self.candidates))


def _usable(topology: Topology, node: PlanNode, a: int, b: int, index: int, forbidden) -> bool:
    if not topology.has_link(a, b):
        return False
    if node.forbidden_edges and any((sid, a, b) in node.forbidden_edges for sid in forbidden):
        return False
    return True


def _bfs_tree(topology, node, root, targets, allowed, sids, reverse=False):
    """Shortest-path arborescence from ``root`` (or into it when ``reverse``)."""
    parent = {root: None}
    queue = deque([root])
    while queue:
        cur = queue.popleft()
        nbrs = topology.in_neighbors(cur) if reverse else topology.out_neighbors(cur)
        for nxt in nbrs:
            if nxt in parent or nxt not in allowed:
                continue
            a, b = (nxt, cur) if reverse else (cur, nxt)
            if not _usable(topology, node, a, b, 0, sids):
                continue
            parent[nxt] = cur
            queue.append(nxt)
    if not set(targets) <= set(parent):
        return None
    needed = set()
    for t in targets:
        while t is not None and t != root:
            needed.add(t)
            t = parent[t]
    edges = []
    depth = {root: 0}
    order = sorted(needed, key=lambda r: (_dist(parent, r), r))
    for r in order:
        p = parent[r]
        edges.append((r, p) if reverse else (p, r))
        depth[r] = depth.get(p, 0) + 1
    return edges, max(depth.values(), default=0)


def _fastest_tree(topology, node, root, targets, allowed, sids, reverse=False):
    """Arborescence of least per-byte time paths (sum of link β) from ``root`` (or into it)."""
    best = {root: 0.0}
    parent = {root: None}
    heap = [(0.0, root)]
    done = set()
    while heap:
        d, cur = heapq.heappop(heap)
        if cur in done:
            continue
        done.add(cur)
        nbrs = topology.in_neighbors(cur) if reverse else topology.out_neighbors(cur)
        for nxt in nbrs:
            if nxt not in allowed:
                continue
            a, b = (nxt, cur) if reverse else (cur, nxt)
            if not _usable(topology, node, a, b, 0, sids):
                continue
            nd = d + topology.link(LinkKey(a, b)).beta_us_per_byte
            if nd < best.get(nxt, float("inf")) - 1e-15:
                best[nxt], parent[nxt] = nd, cur
                heapq.heappush(heap, (nd, nxt))
    if not set(targets) <= set(parent):
        return None
    needed = set()
    for t in targets:
        while t is not None and t != root:
            needed.add(t)
            t = parent[t]
    order = sorted(needed, key=lambda r: (_dist(parent, r), r))
    edges = [((r, parent[r]) if reverse else (parent[r], r)) for r in order]
    return edges, max((_dist(parent, r) for r in needed), default=0)


def _dist(parent, r):
    d = 0
    while parent[r] is not None:
        r = parent[r]
        d += 1
    return d


def _binomial(root, members, reverse):
    order = [root] + list(members)
    edges = []
    n = len(order)
    step = 1
    while step < n:
        for i in range(0, n, 2 * step):
            j = i + step
            if j < n:
                edges.append((order[j], order[i]) if reverse else (order[i], order[j]))
        step *= 2
    depth = max(1, (n - 1).bit_length())
    return edges, depth


def candidate_trees(topology: Topology, node: PlanNode, kind: str, root: int, members, sids, *,
                    limit: int = 4, slice_bytes: int | None = None):
    allowed = set(node.group) | set(node.relay_ranks)
    reverse = kind == "reduce"
    out = []
    star = [((m, root) if reverse else (root, m)) for m in members]
    if all(_usable(topology, node, a, b, 0, sids) for a, b in star):
        out.append(Tree("star", tuple(star), 1))
    bfs = _bfs_tree(topology, node, root, members, allowed, sids, reverse)
    if bfs is not None and tuple(bfs[0]) not in {t.edges for t in out}:
        out.append(Tree("bfs", tuple(bfs[0]), bfs[1]))
    # on links of unequal speed a relay can beat the direct hop
    fast = _fastest_tree(topology, node, root, members, allowed, sids, reverse)
    if fast is not None and tuple(fast[0]) not in {t.edges for t in out}:
        out.append(Tree("fastest", tuple(fast[0]), fast[1]))
    if len(members) > 2:
        edges, depth = _binomial(root, sorted(members), reverse)
        if all(_usable(topology, node, a, b, 0, sids) for a, b in edges):
            out.append(Tree("binomial", tuple(edges), depth))
        chain_order = sorted(members, key=lambda m: (m - root) % topology.rank_count)
        if reverse:
            seq = list(reversed(chain_order)) + [root]
        else:
            seq = [root] + chain_order
        edges = list(zip(seq, seq[1:]))
        if all(_usable(topology, node, a, b, 0, sids) for a, b in edges):
            out.append(Tree("chain", tuple(edges), len(edges)))
    if len(members) > 1 and slice_bytes and not _uniform(topology):
        # the fine MILP's tree over every usable link (it can find relays the menu above does not hold)
        from vericcl_b200.solver.flow_milp import solve_tree_milp
        found = solve_tree_milp(topology, root, members, allowed, reverse=reverse, slice_bytes=slice_bytes,
                                usable=lambda a, b: _usable(topology, node, a, b, 0, sids))
        if found is not None and tuple(found[0]) not in {t.edges for t in out}:
            out.insert(min(len(out), limit - 1), Tree("milp", tuple(found[0]), found[1]))
    if not out:
        raise SemanticError("no legal route tree for node %s (root %d)" % (node.node_id, root))
    return tuple(out[:limit])


def _uniform(topology: Topology) -> bool:
    """Every rank linked to every other with the same α and β (one switch): the star is already optimal."""
    if not topology.is_complete():
        return False
    costs = {(l.alpha_us, l.beta_us_per_byte) for l in topology.links.values()}
    return len(costs) <= 1


def build_demands(plan: PlanDAG, topology: Topology, slice_bytes: int | None = None):
    """Return the transfer demands of every plan node, in plan order (``slice_bytes`` enables the fine MILP)."""
    n = plan.slice_count
    demands = []
    for node in plan.nodes:
        if node.reducing:
            if len(node.logical_output.values) != 1:
                raise SemanticError("a reduce node must have exactly one output slot")
            (slot, target), = node.logical_output.values.items()
            inputs = dict(node.logical_input.values)
            members = tuple(sorted({s.rank for s in inputs} - {slot.rank}))
            contributors = {s.rank: c for s, c in inputs.items()}
            sids = sorted(target)
            trees = candidate_trees(topology, node, "reduce", slot.rank, members, sids,
                                    slice_bytes=slice_bytes) if members else ()
            demands.append(TransferDemand("d-" + node.node_id, node.node_id, node.stage_id, "reduce", slot.rank,
                                          members, min(target) % n, contributors, frozenset(target),
                                          candidates=trees))
        elif node.kind in (CollectiveKind.BROADCAST, CollectiveKind.ALL_GATHER, CollectiveKind.GATHER,
                           CollectiveKind.SCATTER, CollectiveKind.ALL_TO_ALL):
            if len(node.logical_input.values) != 1:
                raise SemanticError("a broadcast node must have exactly one input state")
            (src_slot, value), = node.logical_input.values.items()
            dests = tuple(sorted({s.rank for s in node.logical_output.values} - {src_slot.rank}))
            sids = sorted(value)
            trees = candidate_trees(topology, node, "broadcast", src_slot.rank, dests, sids,
                                    slice_bytes=slice_bytes) if dests else ()
            demands.append(TransferDemand("d-" + node.node_id, node.node_id, node.stage_id, "broadcast",
                                          src_slot.rank, dests, min(value) % n, {src_slot.rank: value},
                                          frozenset(value), local=not dests, candidates=trees))
        else:
            raise SemanticError("plan node kind %s must be decomposed before solving" % node.kind.value)
    return tuple(demands)
