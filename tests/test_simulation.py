from fractions import Fraction

import pytest

from vericcl_b200.errors import SemanticError
from vericcl_b200.performance import CostModel, Executable, RateProfile, ServiceCost, WorkOperation, predict


def model(**kw):
    services = {"link:0:1": (ServiceCost(1.0, 0.01),), "link:1:0": (ServiceCost(1.0, 0.01),),
                "copy:0": (ServiceCost(0.5, 0.001),)}
    return CostModel("m1", services, {"port": 50.0, "link:0:1": 100.0, "link:1:0": 100.0}, **kw)


def test_single_transfer_exact():
    ex = Executable((WorkOperation("a", "send", "link:0:1", 1000, resources=("link:0:1",), flow_id="f"),))
    p = predict(ex, model(), exact=True)
    assert p.t_pred_us == pytest.approx(11.0)
    assert p.exact_completion_ratio == (11, 1)


def test_fair_share_and_dependency():
    ops = (WorkOperation("a", "send", "link:0:1", 1000, resources=("link:0:1", "port"), flow_id="f1"),
           WorkOperation("b", "send", "link:1:0", 1000, resources=("link:1:0", "port"), flow_id="f2"),
           WorkOperation("c", "copy", "copy:0", 1000, dependencies=("a", "b")))
    p = predict(Executable(ops), model(), exact=True)
    # both share the 50 B/us port: 25 B/us each -> 1 + 40 us, then copy 0.5 + 1
    assert Fraction(*p.exact_completion_ratio) == Fraction(1) + Fraction(40) + Fraction(3, 2)
    assert p.model_coverage == "initial"


def test_measured_profile_overrides_sharing():
    prof = RateProfile("p", frozenset({"f1", "f2"}), {"f1": 40.0, "f2": 10.0})
    ops = (WorkOperation("a", "send", "link:0:1", 1000, resources=("link:0:1", "port"), flow_id="f1"),
           WorkOperation("b", "send", "link:1:0", 1000, resources=("link:1:0", "port"), flow_id="f2"))
    p = predict(Executable(ops), model(profiles=(prof,)), exact=True)
    # a: 1000/40 = 25 us after alpha; b then alone at 100 B/us for the rest
    assert p.end_times["a"] == pytest.approx(26.0)
    # then b runs alone, capped by the 50 B/us port
    assert p.t_pred_us == pytest.approx(26.0 + (1000 - 250) / 50.0)


def test_missing_component_reported():
    ex = Executable((WorkOperation("a", "send", "link:0:2", 10, resources=("link:0:2",), flow_id="f"),))
    p = predict(ex, model())
    assert p.t_pred_us is None and "service:link:0:2" in p.missing_components


def test_cycle_rejected():
    ops = (WorkOperation("a", "copy", "copy:0", 1, dependencies=("b",)),
           WorkOperation("b", "copy", "copy:0", 1, dependencies=("a",)))
    with pytest.raises(SemanticError):
        predict(Executable(ops), model())
