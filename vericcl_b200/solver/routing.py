"""Coarse route MILP: choose one candidate tree per demand.

Binary ``x[d,t]`` selects tree ``t`` for demand ``d``.  Each shared resource
(and each directed link) accumulates ``bytes × β`` of the chosen trees'
edges; the objective is lexicographic: minimise the maximum resource busy
time, then the summed tree depth (latency), then total hops.  Isomorphic
demands (same signature) are solved once and the choice is reused (template
reuse, reference: vericcl/solver/routing_milp.py:295-730).
"""
from __future__ import annotations

from vericcl_b200.solver.milp import Model, solve_lexicographic
from vericcl_b200.topology.model import LinkKey


def _edge_resources(topology, edge):
    a, b = edge
    link = topology.link(LinkKey(a, b))
    return ("link:%d:%d" % (a, b),) + tuple(link.resource_ids), link


def choose_trees(demands, topology, slice_bytes: int, *, time_limit: float = 30.0, mip_gap: float = 0.0,
                 owned: bool = False):
    """Return ``{demand_id: Tree}``.  Falls back to the first candidate if the MILP fails."""
    active = [d for d in demands if d.candidates]
    choice = {d.demand_id: d.candidates[0] for d in active}
    if not active or all(len(d.candidates) == 1 for d in active):
        return choice
    model = Model("routes")
    x = {}
    load = {}
    depth_terms, hop_terms = [], []
    for d in active:
        vars_ = []
        for t_index, tree in enumerate(d.candidates):
            var = model.binary("x:%s:%d" % (d.demand_id, t_index))
            x[d.demand_id, t_index] = var
            vars_.append((1, var))
            depth_terms.append((tree.depth, var))
            hop_terms.append((len(tree.edges), var))
            for edge in tree.edges:
                names, link = _edge_resources(topology, edge)
                for name in names:
                    if name.startswith("link:"):
                        weight = slice_bytes * link.beta_us_per_byte
                    else:
                        weight = slice_bytes / topology.resources[name].capacity_bytes_per_us
                    load.setdefault(name, []).append((weight, var))
        model.add_eq(vars_, 1, name="one:" + d.demand_id)
    z = model.continuous("max_load")
    for name, terms in load.items():
        model.add_le(list(terms) + [(-1, z)], 0.0, name="load:" + name)
    sol = solve_lexicographic(model, [[(1, z)], depth_terms, hop_terms], time_limit=time_limit,
                              mip_gap=mip_gap, owned=owned)
    if not sol.usable:
        return choice
    for d in active:
        for t_index, tree in enumerate(d.candidates):
            if sol.values[x[d.demand_id, t_index].name] > 0.5:
                choice[d.demand_id] = tree
    return choice
