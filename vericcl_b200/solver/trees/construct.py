"""Method ``constructive_trees``: batched tree construction for all slices.

Demands are grouped by root (AllGather: one group per source rank; AllReduce:
a reduction group into each slice owner plus the owner's broadcast group).
Without shared resources on a symmetric topology the fast path packs
edge-disjoint arborescences by max-flow (:mod:`packing`); otherwise tree
columns are generated against the shared-resource master (:mod:`columns`),
one master for the reduction trees and one for the broadcast trees.
Each slice is then bound to one chosen tree, and the fixed routes are
composed and timed like any other plan (reference:
vericcl/solver/constructive.py:27-36, vericcl/solver/trees/operators.py:537).
"""
from __future__ import annotations

from collections import defaultdict

from vericcl_b200.composer import compose_routes
from vericcl_b200.errors import SolverError
from vericcl_b200.planner.direct import build_direct_plan
from vericcl_b200.solver.demands import Tree, build_demands
from vericcl_b200.solver.trees.columns import generate_trees
from vericcl_b200.solver.trees.packing import pack_bandwidth, uses_shared_resources


def _groups(demands):
    groups = defaultdict(list)
    for d in demands:
        if d.kind == "broadcast" and not d.members:
            continue
        groups[(d.kind, d.root, tuple(d.members))].append(d)
    return groups


def construct_trees(request, topology, demands, slice_bytes, *, time_limit: float = 30.0):
    """Return {demand_id: Tree} binding every demand to a constructed tree."""
    groups = _groups(demands)
    fast = not uses_shared_resources(topology)
    chosen = {}
    if fast:
        for (kind, root, members), ds in groups.items():
            if kind == "reduce":
                # reduction trees are the reversed broadcast arborescences of the transposed topology
                trees = _reverse_pack(topology, root, members, len(ds), slice_bytes)
            else:
                _, trees = pack_bandwidth(topology, root, list(members), len(ds), slice_bytes)
            _assign(ds, trees, chosen)
        return chosen
    spec = []
    for index, ((kind, root, members), ds) in enumerate(groups.items()):
        spec.append({"id": "g%d" % index, "root": root, "dests": list(members), "slices": len(ds),
                     "reverse": kind == "reduce"})
    # an owner broadcasts a slice only after its reduction tree has delivered it, so the reduction trees and the
    # broadcast trees are two phases: each phase gets its own master and balances its own load (one joint master
    # may load a rank's receive share with two reductions and leave it idle in the broadcasts, doubling the time)
    picks = {}
    for phase in (True, False):
        part = [g for g in spec if g["reverse"] is phase]
        if part:
            picks.update(generate_trees(topology, part, slice_bytes, time_limit=time_limit)[0])
    for index, ((kind, root, members), ds) in enumerate(groups.items()):
        _assign(ds, picks["g%d" % index], chosen)
    return chosen


def _reverse_pack(topology, root, members, k, slice_bytes):
    from vericcl_b200.topology.model import DirectedLink, LinkKey, Topology
    flipped = {}
    for key, link in topology.links.items():
        rk = LinkKey(key.dst, key.src)
        flipped[rk] = DirectedLink(rk, link.alpha_us, link.beta_us_per_byte, link.max_channels)
    t = Topology(topology.name + "-transposed", topology.rank_count, topology.nodes, flipped)
    _, trees = pack_bandwidth(t, root, list(members), k, slice_bytes)
    return [(tuple(sorted((b, a) for a, b in edges)), count) for edges, count in trees]


def _assign(demands, trees, chosen):
    queue = []
    for edges, count in trees:
        queue.extend([edges] * count)
    if len(queue) < len(demands):
        raise SolverError("tree construction produced %d trees for %d slices" % (len(queue), len(demands)))
    for d, edges in zip(sorted(demands, key=lambda x: x.index), queue):
        depth = _depth(edges, d.root, d.kind == "reduce")
        chosen[d.demand_id] = Tree("constructed", tuple(edges), depth)


def _depth(edges, root, reverse):
    parent = {}
    for a, b in edges:
        if reverse:
            parent[a] = b
        else:
            parent[b] = a
    best = 0
    for node in parent:
        d, cur = 0, node
        while cur in parent and d <= len(parent):
            cur = parent[cur]
            d += 1
        best = max(best, d)
    return best


def construct_network(request, topology, model, *, channels: int = 1):
    plan = build_direct_plan(request, topology, reason="constructive_trees")
    demands = build_demands(plan, topology)
    slice_bytes = request.hyperparameters.slice_size_bytes
    trees = construct_trees(request, topology, demands, slice_bytes,
                            time_limit=request.solver.per_model_timeout_s)
    for d in demands:
        if d.candidates and d.demand_id not in trees:
            trees[d.demand_id] = d.candidates[0]
    return compose_routes(plan, demands, trees, topology, slice_bytes, channels=channels,
                          origin="constructive_trees")
