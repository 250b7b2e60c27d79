"""Fine tree MILP (vericcl_b200/solver/flow_milp.py): trees chosen from every usable link."""
from vericcl_b200.input.loader import resolve_documents
from vericcl_b200.examples import example_documents
from vericcl_b200.solver.flow_milp import solve_tree_milp
from vericcl_b200.topology import load_topology
from vericcl_b200.topology.nvswitch import nvswitch_topology


def _topology(slow_pairs, ranks=4, factor=20.0):
    doc = nvswitch_topology(ranks, nvls=False)
    for edge in doc["directed_links"]:
        if (edge["src"], edge["dst"]) in slow_pairs:
            edge["beta_us_per_byte"] *= factor
            edge["alpha_us"] *= factor
    d = example_documents("allgather", "hierarchy", ranks, total_size_bytes=1 << 20, slice_size_bytes=1 << 20,
                          topology=doc)
    return load_topology(resolve_documents(d))


def test_broadcast_relays_around_a_slow_link():
    topo = _topology({(0, 3)})
    edges, depth = solve_tree_milp(topo, 0, (1, 2, 3), range(4), reverse=False, slice_bytes=1 << 20)
    assert (0, 3) not in edges and len(edges) == 3 and depth == 2
    parent = {b: a for a, b in edges}
    assert parent[3] in (1, 2) and parent[1] == 0 and parent[2] == 0


def test_reduction_tree_points_at_the_root_and_avoids_the_slow_link():
    topo = _topology({(3, 0)})
    edges, _ = solve_tree_milp(topo, 0, (1, 2, 3), range(4), reverse=True, slice_bytes=1 << 20)
    assert (3, 0) not in edges
    assert {a for a, _ in edges} == {1, 2, 3}                     # every member sends exactly once
    children = {}
    for a, b in edges:
        children.setdefault(b, []).append(a)
    seen, todo = set(), [0]
    while todo:                                                 # every member reaches the root
        v = todo.pop()
        for c in children.get(v, ()):
            seen.add(c)
            todo.append(c)
    assert seen == {1, 2, 3}


def test_port_load_spreads_a_broadcast_over_relays():
    """With a port that holds 1.5 transfers' worth per makespan unit, a star is slower than a two-level tree."""
    doc = nvswitch_topology(5, nvls=False)
    for res in doc["shared_resources"]:
        if res["id"] == "nvlink-tx-0":
            res["capacity_bytes_per_us"] /= 4.0
    d = example_documents("allgather", "hierarchy", 5, total_size_bytes=1 << 20, slice_size_bytes=1 << 20,
                          topology=doc)
    topo = load_topology(resolve_documents(d))
    edges, depth = solve_tree_milp(topo, 0, (1, 2, 3, 4), range(5), reverse=False, slice_bytes=1 << 20)
    assert sum(1 for a, _ in edges if a == 0) < 4 and depth >= 2


def _arborescence(edges, root, members):
    parent = {}
    for a, b in edges:
        assert b not in parent, "two links into %d" % b
        parent[b] = a
    assert root not in parent
    for m in members:
        seen, v = set(), m
        while v != root:
            assert v not in seen, "cycle through %d" % v
            seen.add(v)
            v = parent[v]
    return parent


def test_random_topologies_give_arborescences_that_reach_every_member():
    """Flow conservation and in-degree rules rule out cycles detached from the root, even free ones."""
    import random
    for seed in range(12):
        rng = random.Random(seed)
        ranks = rng.randrange(3, 7)
        doc = nvswitch_topology(ranks, nvls=False)
        for edge in doc["directed_links"]:
            if rng.random() < 0.3:
                edge["beta_us_per_byte"] *= rng.choice([5.0, 20.0])
            if rng.random() < 0.2:
                edge["alpha_us"] = 0.0          # free links must not form a detached cycle either
        d = example_documents("allgather", "hierarchy", ranks, total_size_bytes=1 << 16, slice_size_bytes=1 << 16,
                              topology=doc)
        topo = load_topology(resolve_documents(d))
        root = rng.randrange(ranks)
        members = tuple(r for r in range(ranks) if r != root)
        for reverse in (False, True):
            edges, depth = solve_tree_milp(topo, root, members, range(ranks), reverse=reverse, slice_bytes=1 << 16)
            flow = [(b, a) for a, b in edges] if reverse else list(edges)
            parent = _arborescence(flow, root, members)
            assert depth == max(_depth(parent, m, root) for m in members)


def _depth(parent, v, root):
    d = 0
    while v != root:
        v = parent[v]
        d += 1
    return d


def test_equal_makespan_prefers_fewer_transfers():
    """When a relay path is exactly as fast as the direct link, the second objective keeps the direct link."""
    doc = nvswitch_topology(3, nvls=False)
    for edge in doc["directed_links"]:
        edge["alpha_us"] = 0.0
        edge["beta_us_per_byte"] = 1e-6
    for edge in doc["directed_links"]:
        if (edge["src"], edge["dst"]) == (0, 2):
            edge["beta_us_per_byte"] = 2e-6           # direct 0->2 costs what 0->1->2 costs
    for res in doc["shared_resources"]:
        res["capacity_bytes_per_us"] = 1e9            # ports never bind
    d = example_documents("allgather", "hierarchy", 3, total_size_bytes=1 << 16, slice_size_bytes=1 << 16,
                          topology=doc)
    topo = load_topology(resolve_documents(d))
    edges, _ = solve_tree_milp(topo, 0, (2,), range(3), reverse=False, slice_bytes=1 << 16)
    assert edges == ((0, 2),)


def test_shared_template_copies_raise_the_port_load():
    """With many demands sharing one tree, the root's port load dominates and the tree fans out through relays."""
    doc = nvswitch_topology(6, nvls=False)
    d = example_documents("allgather", "hierarchy", 6, total_size_bytes=1 << 20, slice_size_bytes=1 << 20,
                          topology=doc)
    topo = load_topology(resolve_documents(d))
    one, _ = solve_tree_milp(topo, 0, (1, 2, 3, 4, 5), range(6), reverse=False, slice_bytes=1 << 20, copies=1)
    many, _ = solve_tree_milp(topo, 0, (1, 2, 3, 4, 5), range(6), reverse=False, slice_bytes=1 << 20, copies=8)
    out_of_root = lambda edges: sum(1 for a, _ in edges if a == 0)       # noqa: E731
    assert out_of_root(many) <= out_of_root(one)
