"""Coarse route MILP: choose one candidate tree per demand.

Tree ``t`` is chosen for demand ``d`` through template counts (below).  Each shared resource
(and each directed link) accumulates ``bytes × β`` of the chosen trees'
edges; the objective is lexicographic: minimise the maximum resource busy
time, then the summed tree depth (latency), then total hops.  Demands of
the same signature share one template of integer counts (reference:
vericcl/solver/routing_milp.py:295-730 and solver/templates.py:856, which
group isomorphic subproblems).
"""
from __future__ import annotations

from vericcl_b200.solver.milp import Model, solve_lexicographic
from vericcl_b200.topology.model import LinkKey


def _edge_resources(topology, edge):
    a, b = edge
    link = topology.link(LinkKey(a, b))
    return ("link:%d:%d" % (a, b),) + tuple(link.resource_ids), link


def _interleave(counts: dict) -> list:
    """Tree indices in an order that spreads each tree's uses evenly (stride scheduling)."""
    marks = [((k + 0.5) / c, t) for t, c in counts.items() for k in range(c)]
    return [t for _, t in sorted(marks)]


def choose_trees(demands, topology, slice_bytes: int, *, time_limit: float = 30.0, mip_gap: float = 0.0,
                 owned: bool = False):
    """Return ``{demand_id: Tree}``.  Falls back to the first candidate if the MILP fails.

    Demands with the same signature (kind, root, members, candidate trees)
    are interchangeable for the objective, so they form one template: an
    integer ``y[g,t]`` counts how many of group ``g`` take tree ``t``
    (``Σ_t y[g,t] = |g|``) instead of one binary per demand.  The group's
    members, in slice order, are then dealt to the trees by stride
    scheduling so each tree's uses spread across the slices.
    """
    active = [d for d in demands if d.candidates]
    choice = {d.demand_id: d.candidates[0] for d in active}
    if not active or all(len(d.candidates) == 1 for d in active):
        return choice
    groups = {}
    for d in active:
        groups.setdefault(d.signature(), []).append(d)
    model = Model("routes")
    y = {}
    load = {}
    depth_terms, hop_terms = [], []
    for g_index, (sig, members) in enumerate(groups.items()):
        terms = []
        for t_index, tree in enumerate(members[0].candidates):
            var = model.add_var("y:%d:%d" % (g_index, t_index), 0.0, float(len(members)), integer=True)
            y[sig, t_index] = var
            terms.append((1, var))
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
        model.add_eq(terms, len(members), name="count:%d" % g_index)
    z = model.continuous("max_load")
    for name, terms in load.items():
        model.add_le(list(terms) + [(-1, z)], 0.0, name="load:" + name)
    sol = solve_lexicographic(model, [[(1, z)], depth_terms, hop_terms], time_limit=time_limit,
                              mip_gap=mip_gap, owned=owned)
    if not sol.usable:
        return choice
    for sig, members in groups.items():
        counts = {}
        for t_index in range(len(members[0].candidates)):
            c = int(round(sol.values[y[sig, t_index].name]))
            if c > 0:
                counts[t_index] = c
        order = _interleave(counts)
        if len(order) != len(members):            # rounding noise: keep the fallback for this group
            continue
        for d, t_index in zip(sorted(members, key=lambda d: (d.index, d.demand_id)), order):
            choice[d.demand_id] = d.candidates[t_index]
    return choice
