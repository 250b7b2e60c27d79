"""Arborescence column generation for broadcast/reduce trees under shared resources.

Master problem (LP, then integer): choose how many slices ``y[d,t]`` of demand
group ``d`` follow tree ``t`` so that every demand group sends all of its
slices and the busiest resource (a link, or a shared resource such as an
NVLink port or a NIC) is busy for at most ``z`` µs; minimise ``z``.  Pricing:
for each demand group, a minimum-cost arborescence under the master's dual
prices (edge cost = Σ over the edge's resources of dual × per-slice busy
time), found with Edmonds' algorithm; columns with negative reduced cost are
added until none remains.  The prices are the LP's own duals (HiGHS
marginals), so the loop stops at the LP optimum over all trees the pricing
can find (reference: vericcl/solver/trees/operators.py:204-533, which uses a
SCIP integer master with lazily generated tree columns).
"""
from __future__ import annotations

import networkx as nx

from vericcl_b200.errors import SolverError
from vericcl_b200.solver.milp import Model
from vericcl_b200.topology.model import LinkKey


def _resources(topology, a, b):
    link = topology.link(LinkKey(a, b))
    out = [("link:%d:%d" % (a, b), link.beta_us_per_byte)]
    for rid in link.resource_ids:
        out.append((rid, 1.0 / topology.resources[rid].capacity_bytes_per_us))
    return out


def _tree_usage(topology, edges, slice_bytes):
    usage = {}
    for a, b in edges:
        for rid, per_byte in _resources(topology, a, b):
            usage[rid] = usage.get(rid, 0.0) + per_byte * slice_bytes
    return usage


def _star(root, dests, reverse):
    return tuple(sorted(((d, root) if reverse else (root, d)) for d in dests))


def _price(topology, root, dests, allowed, duals, slice_bytes, reverse):
    g = nx.DiGraph()
    for key in topology.links:
        a, b = key.src, key.dst
        if a not in allowed or b not in allowed:
            continue
        if reverse:
            a, b = b, a            # build the in-tree as an out-tree on the reversed graph
        if b == root:
            continue
        cost = sum(duals.get(rid, 0.0) * per * slice_bytes for rid, per in _resources(topology, key.src, key.dst))
        g.add_edge(a, b, weight=cost + 1e-9)
    reach = (nx.descendants(g, root) if root in g else set()) | {root}
    cut_off = sorted(set(dests) - reach)
    if cut_off:
        raise SolverError("no tree from rank %d reaches ranks %s over the allowed links" % (root, cut_off))
    arb = nx.minimum_spanning_arborescence(g.subgraph(reach), attr="weight")
    keep = set()
    for d in dests:
        node = d
        while node != root:
            keep.add(node)
            node = next(iter(arb.predecessors(node)))
    edges = [(a, b) for a, b in arb.edges() if b in keep]
    if reverse:
        edges = [(b, a) for a, b in edges]
    cost = sum(g[b][a]["weight"] if reverse else g[a][b]["weight"] for a, b in edges)
    return tuple(sorted(edges)), cost


def generate_trees(topology, groups, slice_bytes, *, max_rounds: int = 30, time_limit: float = 30.0):
    """Column generation.

    ``groups``: list of dicts {id, root, dests, slices, reverse, allowed}.
    Returns ({group id: [(edges, count)]}, makespan bound µs).
    """
    columns = {g["id"]: [_star(g["root"], g["dests"], g["reverse"])] for g in groups}
    for g in groups:
        allowed = set(g.get("allowed") or range(topology.rank_count))
        if not all(topology.has_link(*e) for e in columns[g["id"]][0]):
            edges, _ = _price(topology, g["root"], g["dests"], allowed, {}, slice_bytes, g["reverse"])
            columns[g["id"]] = [edges]
    duals = {}
    for _ in range(max_rounds):
        lp, cons, z = _master(topology, groups, columns, slice_bytes, integer=False)
        sol, row_duals = lp.solve_lp_duals(time_limit=time_limit)
        if not sol.usable:
            raise SolverError("tree master LP failed: " + sol.message)
        duals = _duals(lp, groups, cons, row_duals)
        added = 0
        for g in groups:
            allowed = set(g.get("allowed") or range(topology.rank_count))
            edges, cost = _price(topology, g["root"], g["dests"], allowed, duals["res"], slice_bytes, g["reverse"])
            if edges not in columns[g["id"]] and cost < duals["demand"].get(g["id"], 0.0) - 1e-9:
                columns[g["id"]].append(edges)
                added += 1
        if not added:
            break
    mip, cons, z = _master(topology, groups, columns, slice_bytes, integer=True)
    sol = mip.solve(time_limit=time_limit)
    if not sol.usable:
        raise SolverError("tree master MILP failed: " + sol.message)
    out = {}
    for g in groups:
        picks = []
        for t, edges in enumerate(columns[g["id"]]):
            count = int(round(sol.values["y:%s:%d" % (g["id"], t)]))
            if count:
                picks.append((edges, count))
        out[g["id"]] = picks
    return out, sol.values["z"]


def _master(topology, groups, columns, slice_bytes, integer):
    m = Model("tree-master")
    z = m.continuous("z")
    usage = {}
    for g in groups:
        ys = []
        for t, edges in enumerate(columns[g["id"]]):
            y = m.add_var("y:%s:%d" % (g["id"], t), 0, g["slices"], integer)
            ys.append((1, y))
            for rid, busy in _tree_usage(topology, edges, slice_bytes).items():
                usage.setdefault(rid, []).append((busy, y))
        m.add_eq(ys, g["slices"], name="demand:%s" % g["id"])
    cons = {}
    for rid, terms in usage.items():
        cons[rid] = len(m.rows)
        m.add_le(terms + [(-1, z)], 0.0, name="res:" + rid)
    m.minimize([(1, z)])
    return m, cons, z


def _duals(model, groups, cons, row_duals):
    """Dual prices of the master LP.

    With resource rows ``Σ busy·y − z ≤ 0`` (dual π_r ≥ 0) and demand rows
    ``Σ_t y = slices`` (dual μ_d), a tree column of group d has reduced cost
    ``Σ_r π_r · busy_r(tree) − μ_d``; pricing adds the cheapest tree when that
    is negative.  HiGHS reports ∂objective/∂bound, which is −π_r for a
    resource row and μ_d for a demand row.
    """
    res = {rid: max(0.0, -row_duals[row]) for rid, row in cons.items()}
    demand = {}
    for g in groups:
        row = next(i for i, r in enumerate(model.rows) if r[3] == "demand:%s" % g["id"])
        demand[g["id"]] = row_duals[row]
    return {"res": res, "demand": demand}
