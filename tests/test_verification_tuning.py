import pytest

from vericcl_b200.examples import example_documents
from vericcl_b200.input.loader import resolve_documents
from vericcl_b200.performance.initial import initial_cost_model
from vericcl_b200.synthesis import Lowerer, synthesize
from vericcl_b200.topology import load_topology
from vericcl_b200.topology.nvswitch import multinode_topology
from vericcl_b200.tuning.strategies import solve_repair, variant_path, variant_reshape
from vericcl_b200.verification.bdd import BDD, select_compatible
from vericcl_b200.verification.bottlenecks import analyze
from vericcl_b200.verification.global_bound import certify_global_cut, check_global_cut


def test_bdd_counts_and_selects():
    bdd = BDD()
    a, b, c = bdd.var("a"), bdd.var("b"), bdd.var("c")
    f = bdd.apply("and", bdd.apply("or", a, b), bdd.neg(c))
    assert bdd.count(f) == 3
    assert select_compatible(["a", "b", "c"], [("a", "b"), ("b", "c")]) == ["a", "c"]


def test_cut_bound_is_valid_and_tight_for_star():
    req = resolve_documents(example_documents("allgather", "hierarchy", 8, total_size_bytes=1 << 20,
                                              slice_size_bytes=1 << 18, alpha_us=2.0, link_gbps=150.0))
    bundle = synthesize(req)
    bound = certify_global_cut(req, load_topology(req))
    assert bound.lower_bound_us <= bundle.t_pred_us + 1e-9
    # every rank needs 7 MiB through its 150 GB/s receive port: 7*2^20/150e3 + 2 us
    assert bound.lower_bound_us == pytest.approx(7 * (1 << 20) / 150e3 + 2.0)


def test_repair_improves_or_keeps_and_never_regresses():
    req = resolve_documents(example_documents("allgather", "hierarchy", 8, total_size_bytes=1 << 20,
                                              slice_size_bytes=1 << 18, alpha_us=2.0, link_gbps=150.0))
    topo = load_topology(req)
    model = initial_cost_model(req)
    bundle = synthesize(req, model)
    analysis = analyze(bundle, model, batch_size=8)
    assert analysis.causes and analysis.strategies
    out = solve_repair(bundle, analysis.strategies, lower=Lowerer(req, topo, model))
    assert out.best.t_pred_us <= bundle.t_pred_us
    assert out.best.can_execute


def test_variants_keep_semantics():
    req = resolve_documents(example_documents("allreduce", "hierarchy", 8, total_size_bytes=8 * 1024,
                                              slice_size_bytes=1024))
    topo = load_topology(req)
    model = initial_cost_model(req)
    bundle = synthesize(req, model)
    lower = Lowerer(req, topo, model)
    send = next(op for op in bundle.network.operations if op.kind == "send")
    assert lower(variant_path(bundle.network, topo, send.operation_id)).can_execute
    rrc = [op for op in bundle.network.operations if op.kind == "rrc"][-1]
    assert lower(variant_reshape(bundle.network, topo, rrc.operation_id)).can_execute
