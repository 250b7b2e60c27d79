"""MILP layer (vericcl_b200/solver/milp.py): models, owned solves, cache, lexicographic objectives."""
import pytest

from vericcl_b200.errors import SolverError
from vericcl_b200.solver import milp
from vericcl_b200.solver.milp import Model, solve_lexicographic, solve_owned


def knapsack():
    m = Model("knap")
    xs = [m.binary("x%d" % i) for i in range(4)]
    weights, values = [3, 4, 5, 6], [4, 5, 7, 8]
    m.add_le([(w, x) for w, x in zip(weights, xs)], 10)
    m.minimize([(-v, x) for v, x in zip(values, xs)])
    return m


def test_inline_and_owned_agree_and_cache():
    m = knapsack()
    inline = m.solve()
    assert inline.status == "optimal" and inline.objective == pytest.approx(-13)   # weights 4+6: values 5+8
    milp._CACHE.clear()
    owned = solve_owned(m, time_limit=10)
    assert owned.status == "optimal" and owned.objective == pytest.approx(inline.objective)
    assert not m.violated(owned.values)
    assert m.evaluate(owned.values) == pytest.approx(owned.objective)
    again = solve_owned(m, time_limit=10)
    assert again is owned                      # proven outcome served from the fingerprint cache
    m.add_le([(1, m.by_name["x3"])], 0)         # a changed model has another fingerprint
    assert solve_owned(m, time_limit=10).objective > owned.objective


def test_duplicate_variable_and_infeasible():
    m = Model()
    x = m.continuous("x", 0, 1)
    with pytest.raises(SolverError):
        m.add_var("x")
    m.add_ge([(1, x)], 2)
    m.minimize([(1, x)])
    assert m.solve().status == "infeasible"
    assert solve_owned(m, time_limit=5, use_cache=False).status == "infeasible"


def test_disjunction_orders_two_jobs():
    m = Model("order")
    a0, a1, b0, b1 = (m.continuous(n) for n in ("a0", "a1", "b0", "b1"))
    m.add_eq([(1, a1), (-1, a0)], 3)
    m.add_eq([(1, b1), (-1, b0)], 2)
    o = m.binary("a_first")
    m.disjunction(a1, b0, b1, a0, o, big_m=100, name="ab")
    span = m.continuous("span")
    m.add_ge([(1, span), (-1, a1)], 0)
    m.add_ge([(1, span), (-1, b1)], 0)
    m.minimize([(1, span)])
    sol = m.solve()
    assert sol.objective == pytest.approx(5)
    assert sol["a0"] >= sol["b1"] - 1e-6 or sol["b0"] >= sol["a1"] - 1e-6


def test_lexicographic_keeps_the_first_optimum():
    m = Model("lex")
    x, y = m.continuous("x", 0, 10), m.continuous("y", 0, 10)
    m.add_ge([(1, x), (1, y)], 4)
    sol = solve_lexicographic(m, [[(1, x), (1, y)], [(1, x)]])
    assert sol["x"] + sol["y"] == pytest.approx(4, abs=1e-5) and sol["x"] == pytest.approx(0, abs=1e-5)
    k = knapsack()
    value = [(c, k.vars[i]) for i, c in k.objective.items()]
    # best value first, then the fewest items among the optimal packings
    owned = solve_lexicographic(k, [value, [(1, v) for v in k.vars]], owned=True)
    assert owned.usable and owned.objective == pytest.approx(2)


def test_owned_solve_is_bounded_by_its_lease():
    # a hard assignment-like model with a tiny time limit ends as a timeout or a feasible incumbent, never a hang
    m = Model("hard")
    n = 14
    xs = {(i, j): m.binary("x%d_%d" % (i, j)) for i in range(n) for j in range(n)}
    for i in range(n):
        m.add_eq([(1, xs[i, j]) for j in range(n)], 1)
        m.add_eq([(1, xs[j, i]) for j in range(n)], 1)
    m.minimize([(((i * 7 + j * 13) % 17) + 1, x) for (i, j), x in xs.items()])
    sol = solve_owned(m, time_limit=0.05, grace_s=5.0, use_cache=False)
    assert sol.status in ("optimal", "feasible", "timeout")


def test_route_templates_balance_interchangeable_demands():
    """Four identical broadcast demands share one template; the counts split them 2/2 and interleave."""
    from vericcl_b200.solver.demands import TransferDemand, Tree
    from vericcl_b200.solver.routing import _interleave, choose_trees
    from vericcl_b200.topology import topology_from_document
    from vericcl_b200.topology.nvswitch import nvswitch_topology
    doc = nvswitch_topology(3, nvls=False)
    for link in doc["directed_links"]:
        link["resources"] = []
    doc["shared_resources"] = []
    topo = topology_from_document(doc)
    direct = Tree("star", ((0, 1),), 1)
    relay = Tree("relay", ((0, 2), (2, 1)), 2)
    demands = [TransferDemand("d%d" % i, "n", 0, "broadcast", 0, (1,), i, candidates=(direct, relay))
               for i in range(4)]
    choice = choose_trees(demands, topo, 1 << 20)
    assert [choice["d%d" % i].name for i in range(4)] in (["star", "relay"] * 2, ["relay", "star"] * 2)
    assert _interleave({0: 3, 1: 1}) in ([0, 1, 0, 0], [0, 0, 1, 0])
    assert sorted(_interleave({0: 2, 1: 3})) == [0, 0, 1, 1, 1]


def test_owned_result_survives_solver_output():
    """Text the solver library writes to standard output does not corrupt the owned worker's result."""
    import os
    import pickle
    import subprocess
    import sys
    from pathlib import Path
    m = knapsack()
    code = """
import os
from vericcl_b200.solver import milp
real = milp._solve_arrays


def noisy(*args):
    os.write(1, b"solver chatter\\n")
    return real(*args)


milp._solve_arrays = noisy
milp._worker_main()
"""
    payload = pickle.dumps((m.arrays(), [v.name for v in m.vars], m.objective_constant, 10.0, 0.0))
    root = str(Path(__file__).resolve().parents[1])
    proc = subprocess.run([sys.executable, "-c", code], input=payload, capture_output=True, timeout=60,
                          env=dict(os.environ, PYTHONPATH=root))
    assert proc.returncode == 0, proc.stderr.decode()[-1000:]
    got = pickle.loads(proc.stdout)
    assert got.status == "optimal" and b"solver chatter" in proc.stderr


def test_in_process_solves_keep_standard_output_clean(capfd):
    """Solver library text goes to standard error, so a command's JSON lines stay parseable."""
    import os
    from vericcl_b200.solver import milp
    real = milp._solve_arrays

    def noisy(*args):
        os.write(1, b"solver chatter\n")
        return real(*args)

    milp._solve_arrays = noisy
    try:
        assert knapsack().solve().status == "optimal"
    finally:
        milp._solve_arrays = real
    print('{"ok": true}')
    out, err = capfd.readouterr()
    assert out.strip() == '{"ok": true}' and "solver chatter" in err


def test_template_counts_reach_the_per_demand_optimum():
    """Aggregating interchangeable demands into counts loses nothing: the max link load equals brute force."""
    import itertools
    import random
    from vericcl_b200.solver.demands import TransferDemand, Tree
    from vericcl_b200.solver.routing import choose_trees
    from vericcl_b200.topology import topology_from_document
    from vericcl_b200.topology.model import LinkKey
    from vericcl_b200.topology.nvswitch import nvswitch_topology
    rng = random.Random(5)
    for trial in range(6):
        doc = nvswitch_topology(3, nvls=False)
        for link in doc["directed_links"]:
            link["resources"] = []
            link["beta_us_per_byte"] = rng.choice([0.001, 0.002, 0.004])
        doc["shared_resources"] = []
        topo = topology_from_document(doc)
        trees = (Tree("direct", ((0, 1),), 1), Tree("relay", ((0, 2), (2, 1)), 2))
        k = rng.randint(1, 6)
        demands = [TransferDemand("d%d" % i, "n", 0, "broadcast", 0, (1,), i, candidates=trees) for i in range(k)]
        size = 1000

        def max_load(assign):
            load = {}
            for t in assign:
                for a, b in t.edges:
                    load[(a, b)] = load.get((a, b), 0.0) + size * topo.link(LinkKey(a, b)).beta_us_per_byte
            return max(load.values())

        best = min(max_load(c) for c in itertools.product(trees, repeat=k))
        got = choose_trees(demands, topo, size)
        assert max_load([got["d%d" % i] for i in range(k)]) == pytest.approx(best), trial
