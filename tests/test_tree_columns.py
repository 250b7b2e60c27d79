"""Tree column generation against the shared-resource master, with the LP's own duals."""
from vericcl_b200.examples import example_documents
from vericcl_b200.input.loader import resolve_documents
from vericcl_b200.solver.milp import Model
from vericcl_b200.solver.trees.columns import generate_trees
from vericcl_b200.topology.nvswitch import multinode_topology


def test_lp_duals_match_the_textbook_signs():
    # min x + 2y  s.t.  x + y >= 3 (dual 1: raising 3 costs 1 per unit),  y <= 5,  x <= 2 (binds: dual -1)
    m = Model("duals")
    x, y = m.continuous("x"), m.continuous("y")
    m.add_ge([(1, x), (1, y)], 3.0, name="cover")
    m.add_le([(1, y)], 5.0, name="ycap")
    m.add_le([(1, x)], 2.0, name="xcap")
    m.minimize([(1, x), (2, y)])
    sol, duals = m.solve_lp_duals()
    assert abs(sol.objective - 4.0) < 1e-9
    assert abs(duals[0] - 2.0) < 1e-9 and abs(duals[1]) < 1e-9 and abs(duals[2] + 1.0) < 1e-9


def _shared_nic_topology():
    from vericcl_b200.topology import load_topology
    d = example_documents("allgather", "constructive_trees", 4, total_size_bytes=4 << 20, slice_size_bytes=1 << 20,
                          topology=multinode_topology(2, 2, inter_gbps=25.0, rank_shares=True))
    return load_topology(resolve_documents(d))


def test_shared_nics_get_relay_trees():
    """2 groups × 2 ranks, one 25 GB/s NIC per group, each rank's receive share half of it.

    A star from every root crosses the NIC twice per slice; a tree that crosses
    once and relays inside the other group halves the NIC time, and the LP's
    duals find it.  Each group's NIC carries its two roots' slices: 2 roots × 4
    slices × 2 crossings × 42 µs with stars, half that with relay trees.
    """
    topo = _shared_nic_topology()
    slice_bytes = 1 << 20
    groups = [{"id": "g%d" % r, "root": r, "dests": [d for d in range(4) if d != r], "slices": 4,
               "reverse": False} for r in range(4)]
    picks, z = generate_trees(topo, groups, slice_bytes)
    star_z = 2 * 4 * 2 * slice_bytes / 25e3
    assert z <= star_z / 2 + 1e-6
    for gid, chosen in picks.items():
        assert sum(count for _, count in chosen) == 4
        for edges, _ in chosen:
            assert len([(a, b) for a, b in edges if a // 2 != b // 2]) == 1     # one NIC crossing per slice


def test_lp_duals_of_equality_and_ranged_rows():
    # min 3a + b  s.t.  a + b = 4 (free dual),  1 <= a <= 10 (ranged; the lower side binds: dual 2)
    m = Model("ranged")
    a, b = m.continuous("a"), m.continuous("b")
    m.add_eq([(1, a), (1, b)], 4.0, name="sum")
    m.add([(1, a)], 1.0, 10.0, name="range")
    m.minimize([(3, a), (1, b)])
    sol, duals = m.solve_lp_duals()
    assert abs(sol.values["a"] - 1.0) < 1e-9 and abs(sol.values["b"] - 3.0) < 1e-9
    assert abs(duals[0] - 1.0) < 1e-9 and abs(duals[1] - 2.0) < 1e-9


def test_reduction_trees_cross_the_nic_once():
    """Reduce groups are in-trees: every rank's slice reaches the owner with one NIC crossing per slice."""
    topo = _shared_nic_topology()
    slice_bytes = 1 << 20
    groups = [{"id": "r%d" % r, "root": r, "dests": [d for d in range(4) if d != r], "slices": 2,
               "reverse": True} for r in range(4)]
    picks, z = generate_trees(topo, groups, slice_bytes)
    assert z <= 2 * 2 * slice_bytes / 25e3 + 1e-6          # two owners per group × 2 slices × one crossing
    for gid, chosen in picks.items():
        owner = int(gid[1:])
        for edges, _ in chosen:
            assert all(b == owner or any(a2 == b for a2, _ in edges) for _, b in edges)   # edges point to the owner
            assert len([(a, b) for a, b in edges if a // 2 != b // 2]) == 1


def test_an_unreachable_destination_is_a_solver_error():
    import pytest
    from vericcl_b200.errors import SolverError
    topo = _shared_nic_topology()
    groups = [{"id": "g0", "root": 0, "dests": [1, 2, 3], "slices": 1, "reverse": False, "allowed": [0, 1, 2]}]
    with pytest.raises(SolverError, match="reaches ranks \\[3\\]"):
        generate_trees(topo, groups, 1 << 20)


def _spans(edges, root, dests, reverse):
    parent = {}
    for a, b in edges:
        child, up = (a, b) if reverse else (b, a)
        assert child not in parent, "two parents for rank %d" % child
        parent[child] = up
    for d in dests:
        node, hops = d, 0
        while node != root:
            node = parent[node]
            hops += 1
            assert hops <= len(parent), "cycle above rank %d" % d
    return True


def test_random_shared_nic_topologies_give_spanning_trees_no_worse_than_stars():
    from hypothesis import given, settings, strategies as st
    from vericcl_b200.solver.trees.columns import _master, _star
    from vericcl_b200.topology import load_topology

    @settings(max_examples=12, deadline=None)
    @given(groups_n=st.integers(2, 3), per=st.integers(1, 3), shares=st.booleans(), reverse=st.booleans(),
           slices=st.integers(1, 3), gbps=st.sampled_from([12.5, 25.0, 50.0]))
    def check(groups_n, per, shares, reverse, slices, gbps):
        ranks = groups_n * per
        d = example_documents("allgather", "constructive_trees", ranks, total_size_bytes=ranks * 4096,
                              slice_size_bytes=4096,
                              topology=multinode_topology(groups_n, per, inter_gbps=gbps, rank_shares=shares))
        topo = load_topology(resolve_documents(d))
        spec = [{"id": "g%d" % r, "root": r, "dests": [x for x in range(ranks) if x != r], "slices": slices,
                 "reverse": reverse} for r in range(ranks)]
        picks, z = generate_trees(topo, spec, 1 << 20)
        stars = {g["id"]: [_star(g["root"], g["dests"], reverse)] for g in spec}
        star_sol = _master(topo, spec, stars, 1 << 20, integer=True)[0].solve()
        assert z <= star_sol.values["z"] + 1e-6
        for g in spec:
            assert sum(count for _, count in picks[g["id"]]) == slices
            for edges, _ in picks[g["id"]]:
                assert all(topo.has_link(a, b) for a, b in edges)
                assert _spans(edges, g["root"], g["dests"], reverse)

    check()


def test_allreduce_trees_balance_each_phase_on_eight_ranks_behind_two_nics():
    """2 groups × 4 ranks, 25 GB/s NICs with per-rank receive shares, AllReduce of 8 × 1 MiB slices.

    Balancing reduction and broadcast trees in one master let a rank's receive
    share take two reductions and no broadcast, so the broadcasts waited for a
    doubled reduction phase (T_pred 693 µs); a master per phase keeps the
    schedule within 15 % of the hierarchy plan (375 µs).
    """
    from vericcl_b200.synthesis import synthesize
    times = {}
    for method in ("constructive_trees", "hierarchy"):
        d = example_documents("allreduce", method, 8, total_size_bytes=8 << 20, slice_size_bytes=1 << 20,
                              topology=multinode_topology(2, 4, inter_gbps=25.0, rank_shares=True))
        d["sketch"]["calibration"]["enabled"] = False
        bundle = synthesize(resolve_documents(d))
        assert bundle.can_execute, bundle.checks
        times[method] = bundle.t_pred_us
    assert times["constructive_trees"] <= 1.15 * times["hierarchy"]


def test_lp_duals_of_an_infeasible_model_are_unusable():
    m = Model("infeasible")
    x = m.continuous("x")
    m.add_ge([(1, x)], 2.0, name="low")
    m.add_le([(1, x)], 1.0, name="high")
    m.minimize([(1, x)])
    sol, duals = m.solve_lp_duals()
    assert sol.status == "infeasible" and not sol.usable and duals == []
