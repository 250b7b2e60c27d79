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
