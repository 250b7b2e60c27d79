from fractions import Fraction

import pytest

from vericcl_b200.errors import SemanticError
from vericcl_b200.performance import CostModel, Executable, RateProfile, ServiceCost, WorkOperation, predict
from vericcl_b200.performance.events import Movement


def model(**kw):
    services = {"link:0:1": (ServiceCost(1.0, 0.01),), "link:1:0": (ServiceCost(1.0, 0.01),),
                "copy:0": (ServiceCost(0.5, 0.001),)}
    return CostModel("m1", services, {"port": 50.0, "link:0:1": 100.0, "link:1:0": 100.0}, **kw)


def test_single_transfer_exact():
    ex = Executable((WorkOperation("a", "send", Movement("link:0:1", 1000), crosses=("link:0:1",), flow_id="f"),))
    p = predict(ex, model(), exact=True)
    assert p.t_pred_us == pytest.approx(11.0)
    assert p.exact_completion_ratio == (11, 1)


def test_fair_share_and_dependency():
    ops = (WorkOperation("a", "send", Movement("link:0:1", 1000), crosses=("link:0:1", "port"), flow_id="f1"),
           WorkOperation("b", "send", Movement("link:1:0", 1000), crosses=("link:1:0", "port"), flow_id="f2"),
           WorkOperation("c", "copy", Movement("copy:0", 1000), after=("a", "b")))
    p = predict(Executable(ops), model(), exact=True)
    # both share the 50 B/us port: 25 B/us each -> 1 + 40 us, then copy 0.5 + 1
    assert Fraction(*p.exact_completion_ratio) == Fraction(1) + Fraction(40) + Fraction(3, 2)
    assert p.model_coverage == "initial"


def test_measured_profile_overrides_sharing():
    prof = RateProfile("p", frozenset({"f1", "f2"}), {"f1": 40.0, "f2": 10.0})
    ops = (WorkOperation("a", "send", Movement("link:0:1", 1000), crosses=("link:0:1", "port"), flow_id="f1"),
           WorkOperation("b", "send", Movement("link:1:0", 1000), crosses=("link:1:0", "port"), flow_id="f2"))
    p = predict(Executable(ops), model(profiles=(prof,)), exact=True)
    # a: 1000/40 = 25 us after alpha; b then alone at 100 B/us for the rest
    assert p.end_times["a"] == pytest.approx(26.0)
    # then b runs alone, capped by the 50 B/us port
    assert p.t_pred_us == pytest.approx(26.0 + (1000 - 250) / 50.0)


def test_missing_component_reported():
    ex = Executable((WorkOperation("a", "send", Movement("link:0:2", 10), crosses=("link:0:2",), flow_id="f"),))
    p = predict(ex, model())
    assert p.t_pred_us is None and "service:link:0:2" in p.missing_components


def test_cycle_rejected():
    ops = (WorkOperation("a", "copy", Movement("copy:0", 1), after=("b",)),
           WorkOperation("b", "copy", Movement("copy:0", 1), after=("a",)))
    with pytest.raises(SemanticError):
        predict(Executable(ops), model())


def test_max_min_fairness_gives_unused_share_to_the_other_flow():
    """A flow held to 20 B/µs by its own link leaves 80 of the port's 100 B/µs to the other flow."""
    services = {"link:0:1": (ServiceCost(0.0, 0.05),), "link:0:2": (ServiceCost(0.0, 0.001),)}
    m = CostModel("mm", services, {"tx0": 100.0})
    ops = (WorkOperation("slow", "send", Movement("link:0:1", 200), crosses=("tx0",), flow_id="a"),
           WorkOperation("fast", "send", Movement("link:0:2", 800), crosses=("tx0",), flow_id="b"))
    p = predict(Executable(ops), m, exact=True)
    assert p.end_times["slow"] == pytest.approx(10.0)        # 200 B at 20 B/µs
    assert p.end_times["fast"] == pytest.approx(10.0)        # 800 B at 80 B/µs
    assert p.unmeasured_modes == (("a", "b"),)


def test_max_min_rates_progressive_filling():
    from vericcl_b200.performance.simulation import max_min_rates
    caps = {"x": Fraction(100), "y": Fraction(100), "z": Fraction(5)}
    cross = {"x": ("r1",), "y": ("r1", "r2"), "z": ("r2",)}
    rates = max_min_rates(caps, cross, {"r1": Fraction(30), "r2": Fraction(60)}, Fraction(0))
    # r1 saturates at 15 + 15; z is capped at 5; y stays at 15 (held by r1)
    assert rates == {"x": Fraction(15), "y": Fraction(15), "z": Fraction(5)}


def _chain_model_and_graph(rng, n_ops):
    """Random DAG of local work and network work on private resources: no two operations ever share."""
    services, resources, ops = {}, {}, []
    for i in range(n_ops):
        kind = rng.choice(["send", "copy", "nop"])
        prior = [o.operation_id for o in ops]
        deps = tuple(rng.sample(prior, min(len(prior), rng.randrange(3))))
        release = rng.randrange(0, 50) / 10
        if kind == "nop":
            ops.append(WorkOperation("o%d" % i, "nop", after=deps, release_us=release))
            continue
        key = "%s:%d" % ("link" if kind == "send" else "copy", i)
        services[key] = (ServiceCost(rng.randrange(0, 40) / 10, rng.choice([0.01, 0.02, 0.125, 0.3])),)
        res = ()
        if kind == "send":
            resources["wire%d" % i] = rng.choice([1000.0, 5.0, 2.5])
            res = ("wire%d" % i,)
        ops.append(WorkOperation("o%d" % i, kind, Movement(key, rng.randrange(1, 500)), after=deps, crosses=res,
                                 flow_id="f%d" % i if kind == "send" else None, release_us=release))
    return CostModel("chain", services, resources), Executable(tuple(ops))


def test_exact_replay_equals_longest_path_when_nothing_is_shared():
    """Without sharing, T_pred is the longest path of (release, α + n / min(1/β, capacity)) exactly."""
    import random
    rng = random.Random(7)
    for _ in range(40):
        model_, ex = _chain_model_and_graph(rng, rng.randrange(1, 25))
        p = predict(ex, model_, exact=True)
        q = lambda v: Fraction(repr(float(v)))
        end = {}
        for op in ex.operations:         # operations are listed after their dependencies
            t = max([q(op.release_us)] + [end[d] for d in op.after])
            if op.kind != "nop":
                seg = model_.service_for(op.component, op.nbytes)
                rate = 1 / q(seg.beta_us_per_byte)
                for r in op.crosses:
                    rate = min(rate, q(model_.resources[r]))
                t += q(seg.alpha_us) + op.nbytes / rate
            end[op.operation_id] = t
        assert Fraction(*p.exact_completion_ratio) == max(end.values())


def test_float_replay_tracks_the_exact_one_under_sharing():
    import random
    rng = random.Random(11)
    for trial in range(30):
        services = {"link:%d" % i: (ServiceCost(rng.randrange(0, 20) / 10, rng.choice([0.01, 0.03, 0.07])),)
                    for i in range(4)}
        services["copy:0"] = (ServiceCost(0.5, 0.002),)
        m = CostModel("share", services, {"tx": 40.0, "rx": 25.0})
        ops = []
        for i in range(16):
            prior = [o.operation_id for o in ops]
            deps = tuple(rng.sample(prior, min(len(prior), rng.randrange(2))))
            if rng.random() < 0.7:
                ops.append(WorkOperation("n%d" % i, "send", Movement("link:%d" % (i % 4), rng.randrange(10, 900)),
                                         after=deps, crosses=tuple(rng.sample(["tx", "rx"], rng.randrange(1, 3))),
                                         flow_id="f%d" % i, release_us=rng.randrange(0, 30) / 10))
            else:
                ops.append(WorkOperation("n%d" % i, "copy", Movement("copy:0", rng.randrange(10, 900)), after=deps))
        ex = Executable(tuple(ops))
        exact = predict(ex, m, exact=True)
        approx = predict(ex, m)
        assert approx.t_pred_us == pytest.approx(float(Fraction(*exact.exact_completion_ratio)), rel=1e-9)
        # every byte of every operation is accounted for by its rate segments
        moved = {}
        for key, t0, t1, rate, _src in exact.segments:
            moved[key] = moved.get(key, 0.0) + (t1 - t0) * rate
        for op in ops:
            assert moved[op.operation_id] == pytest.approx(op.nbytes, rel=1e-9)
