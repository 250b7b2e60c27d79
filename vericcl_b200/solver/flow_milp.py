"""Fine tree MILP: the route tree of one demand chosen from all links, not from a menu.

For a broadcast from ``root`` to ``members`` (a reduction is the same problem
on the reversed links) the model has

* a binary ``x[a,b]`` per usable link inside the node's group and relays;
* per destination ``d`` a unit of flow from the root to ``d``
  (``f[a,b,d] <= x[a,b]``, conservation at every rank), so the chosen links
  connect the root to every destination;
* at most one chosen link into every rank (exactly one into a destination,
  none into the root), so the links form an arborescence;
* arrival times with big-M precedence along chosen links:
  ``t[b] >= t[a] + α(a,b) + β(a,b)·S - M·(1 - x[a,b])``;
* a load per shared resource and per link: ``copies · S / capacity`` for every
  chosen link on it (``copies`` demands of the same template share the tree);
* a makespan ``T`` at least every arrival and every load.

The objective is lexicographic: the makespan, then the number of links
(fewer transfers), then the summed arrival times (shallower trees).
(Reference: vericcl/solver/milp.py:273-651 ``_build_model``, whose fine model
also carries channels and resource slots; here channels are assigned after
the tree by the composer.)  Results are cached by the problem's content.
"""
from __future__ import annotations

from vericcl_b200.solver.milp import Model, solve_lexicographic
from vericcl_b200.topology.model import LinkKey

_CACHE: dict = {}


def _links(topology, allowed, usable):
    out = []
    for a in sorted(allowed):
        for b in sorted(allowed):
            if a != b and topology.has_link(a, b) and usable(a, b):
                out.append((a, b))
    return out


def solve_tree_milp(topology, root: int, members, allowed, *, reverse: bool, slice_bytes: int, copies: int = 1,
                    usable=lambda a, b: True, time_limit: float = 5.0):
    """``(edges in data-flow direction, depth)`` of the best tree, or None when no tree is found."""
    members = tuple(sorted(members))
    allowed = tuple(sorted(set(allowed) | {root} | set(members)))
    # search on the graph in which data flows from the root outwards
    flow_links = [(b, a) for (a, b) in _links(topology, allowed, usable)] if reverse else \
        _links(topology, allowed, usable)
    real = (lambda a, b: (b, a)) if reverse else (lambda a, b: (a, b))
    key = (topology.signature().__repr__(), root, members, allowed, reverse, slice_bytes, copies, tuple(flow_links))
    if key in _CACHE:
        return _CACHE[key]
    dur, uses = {}, {}
    for a, b in flow_links:
        link = topology.link(LinkKey(*real(a, b)))
        dur[a, b] = link.time_us(slice_bytes)
        uses[a, b] = [("link:%d:%d" % real(a, b), 1.0 / link.beta_us_per_byte)] + \
            [(r, topology.resources[r].capacity_bytes_per_us) for r in link.resource_ids if r in topology.resources]
    horizon = sum(sorted(dur.values())[-len(allowed):]) + 1.0 if dur else 1.0
    m = Model("tree")
    x = {e: m.binary("x:%d:%d" % e) for e in flow_links}
    t = {v: m.continuous("t:%d" % v, 0.0, horizon) for v in allowed}
    z = m.continuous("T", 0.0, horizon * (copies + 1))
    m.add_eq([(1, t[root])], 0.0)
    for v in allowed:
        into = [(1, x[e]) for e in flow_links if e[1] == v]
        if v == root:
            if into:
                m.add_eq(into, 0.0)
        elif v in members:
            if not into:
                _CACHE[key] = None
                return None
            m.add_eq(into, 1.0)
        elif into:
            m.add_le(into, 1.0)
    for d in members:
        f = {e: m.continuous("f:%d:%d:%d" % (e[0], e[1], d), 0.0, 1.0) for e in flow_links}
        for e in flow_links:
            m.add_le([(1, f[e]), (-1, x[e])], 0.0)
        for v in allowed:
            terms = [(1, f[e]) for e in flow_links if e[0] == v] + [(-1, f[e]) for e in flow_links if e[1] == v]
            rhs = 1.0 if v == root else (-1.0 if v == d else 0.0)
            if terms:
                m.add_eq(terms, rhs)
    for (a, b), var in x.items():
        m.add_ge([(1, t[b]), (-1, t[a]), (-horizon, var)], dur[a, b] - horizon)
    for v in members:
        m.add_le([(1, t[v]), (-1, z)], 0.0)
    load = {}
    for e, var in x.items():
        for rid, cap in uses[e]:
            load.setdefault(rid, []).append((copies * slice_bytes / cap, var))
    for rid, terms in load.items():
        m.add_le(list(terms) + [(-1, z)], 0.0)
    objectives = [[(1, z)], [(1, var) for var in x.values()], [(1, t[v]) for v in members]]
    sol = solve_lexicographic(m, objectives, time_limit=time_limit, tolerance=1e-7)
    if not sol.usable:
        _CACHE[key] = None
        return None
    chosen = [e for e, var in x.items() if sol.values[var.name] > 0.5]
    parent = {b: a for a, b in chosen}
    # keep only links on the way to a destination (a relay that feeds nobody is dropped)
    needed = set()
    for d in members:
        v = d
        while v != root and v not in needed:
            needed.add(v)
            v = parent[v]
    edges, depth = [], {root: 0}

    def level(v):
        if v not in depth:
            depth[v] = level(parent[v]) + 1
        return depth[v]

    for v in sorted(needed, key=lambda r: (level(r), r)):
        edges.append(real(parent[v], v))
    result = (tuple(edges), max((level(v) for v in needed), default=0))
    _CACHE[key] = result
    return result
