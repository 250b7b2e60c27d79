"""Decision-scope certificates: exact LP-dual bounds and enumerated leaves, checked independently."""
from dataclasses import replace
from fractions import Fraction

import pytest

from vericcl_b200.errors import SemanticError
from vericcl_b200.examples import example_documents
from vericcl_b200.input.loader import resolve_documents
from vericcl_b200.performance.initial import initial_cost_model
from vericcl_b200.synthesis import Lowerer, synthesize
from vericcl_b200.topology import load_topology
from vericcl_b200.tuning.strategies import solve_repair
from vericcl_b200.verification.bottlenecks import analyze
from vericcl_b200.verification.proof_check import (certify_scope, check_no_improvement, fixed_work,
                                                    optimistic_relaxation, verify_lp_dual)


def test_lp_dual_certificate_exact():
    # min x1 + 2 x2  s.t.  x1 + x2 >= 3,  x2 >= 1  -> optimum 4 (x1=2, x2=1); y = (1, 1) proves it
    b = verify_lp_dual(matrix=[[1, 1], [0, 1]], rhs=[3, 1], objective=[1, 2], dual=[1, 1], model_version="m",
                       scope_id="s")
    assert b.value == Fraction(4) and len(b.digest) == 64
    with pytest.raises(SemanticError, match="nonnegative"):
        verify_lp_dual(matrix=[[1]], rhs=[1], objective=[1], dual=[-1], model_version="m", scope_id="s")
    with pytest.raises(SemanticError, match="A-transpose"):
        verify_lp_dual(matrix=[[1, 1], [0, 1]], rhs=[3, 1], objective=[1, 2], dual=[2, 1], model_version="m",
                       scope_id="s")
    with pytest.raises(SemanticError, match="dimensions"):
        verify_lp_dual(matrix=[[1]], rhs=[1, 2], objective=[1], dual=[1], model_version="m", scope_id="s")
    with pytest.raises(SemanticError):
        verify_lp_dual(matrix=[[1]], rhs=[1], objective=[1], dual=[1], model_version="", scope_id="s")


@pytest.fixture(scope="module")
def setting():
    req = resolve_documents(example_documents("allgather", "hierarchy", 4, total_size_bytes=1 << 18,
                                              slice_size_bytes=1 << 16, alpha_us=2.0, link_gbps=150.0))
    topo = load_topology(req)
    model = initial_cost_model(req)
    bundle = synthesize(req, model)
    analysis = analyze(bundle, model, batch_size=16)
    return req, topo, model, bundle, analysis, Lowerer(req, topo, model)


def test_relaxation_bounds_the_incumbent(setting):
    _, _, model, bundle, _, _ = setting
    a, b, c = optimistic_relaxation(bundle.executable, model)
    top = max(Fraction(v) for v in b)
    assert top <= Fraction(*bundle.prediction.exact_completion_ratio)


def test_leaves_certificate_agrees_with_repair(setting):
    _, _, model, bundle, analysis, lower = setting
    cert = certify_scope(bundle, analysis.strategies, model, lower=lower, use_bound=False)
    assert cert["leaves"] and cert["bound"] is None
    result = check_no_improvement(cert, bundle, analysis.strategies, model, lower=lower)
    repaired = solve_repair(bundle, analysis.strategies, lower=lower)
    if repaired.improved:
        assert result.status in ("improvement_exists", "proven_no_improvement")
    else:
        assert result.status == "proven_no_improvement" and result.checked_leaves == len(cert["leaves"])


def test_tampered_or_stale_certificates_are_rejected(setting):
    _, _, model, bundle, analysis, lower = setting
    cert = certify_scope(bundle, analysis.strategies, model, lower=lower, use_bound=False)
    valid = [i for i, leaf in enumerate(cert["leaves"]) if leaf["status"] == "valid"]
    assert valid
    bad = dict(cert, leaves=[dict(leaf) for leaf in cert["leaves"]])
    bad["leaves"][valid[0]]["t_pred"] = "1/1"
    assert check_no_improvement(bad, bundle, analysis.strategies, model, lower=lower).status == "invalid"
    missing = dict(cert, leaves=cert["leaves"][1:])
    assert check_no_improvement(missing, bundle, analysis.strategies, model, lower=lower).status == "incomplete"
    newer, _ = model.with_updates("other-version")
    assert check_no_improvement(cert, bundle, analysis.strategies, newer, lower=lower).status == "stale"


def test_bound_form_for_fixed_work_scopes(setting):
    from vericcl_b200.verification.bottlenecks import StrategyRecord
    _, _, model, bundle, _, lower = setting
    ops = [op.operation_id for op in bundle.network.operations][:2]
    fixed = [StrategyRecord("prio-t%d" % i, "order", (op,), (("advance", 1),)) for i, op in enumerate(ops)]
    assert fixed_work(fixed)
    # with an incumbent no slower than its own contention-free critical path, the relaxation closes the scope
    quick = replace(bundle, prediction=replace(bundle.prediction, exact_completion_ratio=(1, 10**9)))
    cert = certify_scope(quick, fixed, model, lower=lower)
    assert cert["bound"] is not None and not cert["leaves"]
    assert check_no_improvement(cert, quick, fixed, model, lower=lower).status == "proven_no_improvement"
    forged = dict(cert, bound=dict(cert["bound"], rhs=["0"] * len(cert["bound"]["rhs"])))
    assert check_no_improvement(forged, quick, fixed, model, lower=lower).status == "invalid"
    # the real incumbent is slower than the bound: the certificate falls back to enumerated leaves
    cert = certify_scope(bundle, fixed, model, lower=lower)
    assert cert["bound"] is None and len(cert["leaves"]) == len(fixed)
