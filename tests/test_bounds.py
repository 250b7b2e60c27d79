"""Dependency lower bounds hold for synthesized schedules and prune parameter choices."""
import pytest

from vericcl_b200.examples import example_documents
from vericcl_b200.input.loader import resolve_documents
from vericcl_b200.performance.initial import initial_cost_model
from vericcl_b200.solver.bounds import dependency_lower_bound
from vericcl_b200.synthesis import synthesize
from vericcl_b200.topology import load_topology
from vericcl_b200.topology.nvswitch import multinode_topology


@pytest.mark.parametrize("op,p,method", [("allgather", 4, "hierarchy"), ("allreduce", 4, "hierarchy"),
                                         ("allgather", 8, "constructive_trees"), ("reduce_scatter", 4, "hierarchy"),
                                         ("broadcast", 4, "hierarchy")])
def test_bound_is_below_exact_prediction(op, p, method):
    req = resolve_documents(example_documents(op, method, p, total_size_bytes=p * 65536, slice_size_bytes=65536,
                                              alpha_us=2.0, link_gbps=150.0))
    model = initial_cost_model(req)
    bundle = synthesize(req, model)
    lb = dependency_lower_bound(req, load_topology(req), model)
    assert 0 < lb <= bundle.t_pred_us + 1e-9


def test_two_group_bound_counts_the_slow_link():
    docs = example_documents("allreduce", "hierarchy", 8, total_size_bytes=8 << 20, slice_size_bytes=1 << 20,
                             topology=multinode_topology(2, 4, inter_gbps=25.0))
    req = resolve_documents(docs)
    model = initial_cost_model(req)
    lb = dependency_lower_bound(req, load_topology(req), model)
    # a 1 MiB slice must cross the 25 GB/s inter-group link at least once
    assert lb >= (1 << 20) / 25e3
    assert lb <= synthesize(req, model).t_pred_us + 1e-9


def test_cut_bound_follows_a_faster_calibrated_model():
    from dataclasses import replace as dc_replace
    from vericcl_b200.program.native import build_executable
    from vericcl_b200.performance.initial import model_context
    from vericcl_b200.performance.simulation import predict
    from vericcl_b200.verification.global_bound import certify_global_cut
    req = resolve_documents(example_documents("allgather", "hierarchy", 4, total_size_bytes=4 * 65536,
                                              slice_size_bytes=65536, alpha_us=2.0, link_gbps=150.0))
    topo = load_topology(req)
    model = initial_cost_model(req)
    faster, _ = model.with_updates("faster", services={
        k: tuple(dc_replace(c, beta_us_per_byte=c.beta_us_per_byte / 4) for c in v)
        for k, v in model.services.items() if k.startswith(("link:", "rrc:"))},
        resources={k: v * 4 for k, v in model.resources.items()})
    bundle = synthesize(req, model)
    exe = build_executable(bundle.program, bundle.storage, req, topo, model_context(req))
    t_fast = predict(exe, faster, exact=True).t_pred_us
    nominal = certify_global_cut(req, topo)
    calibrated = certify_global_cut(req, topo, faster)
    assert calibrated.lower_bound_us <= t_fast + 1e-9
    assert calibrated.lower_bound_us < nominal.lower_bound_us
