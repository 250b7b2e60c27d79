import pytest

from vericcl_b200.examples import example_documents
from vericcl_b200.input.loader import resolve_documents
from vericcl_b200.performance.initial import initial_cost_model
from vericcl_b200.synthesis import Lowerer, synthesize
from vericcl_b200.topology import load_topology
from vericcl_b200.tuning.strategies import solve_repair, variant_path, variant_reshape
from vericcl_b200.verification.bdd import BDD, select_compatible
from vericcl_b200.verification.bottlenecks import analyze
from vericcl_b200.verification.global_bound import certify_global_cut


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


def test_measured_trace_tails_become_causes():
    """A trace report's slowest device steps map back to operations and lead the strategy list."""
    from vericcl_b200.program.device import compile_xml
    from vericcl_b200.verification.bottlenecks import trace_causes
    req = resolve_documents(example_documents("allgather", "hierarchy", 4, total_size_bytes=1 << 18,
                                              slice_size_bytes=1 << 16, alpha_us=2.0, link_gbps=150.0))
    model = initial_cost_model(req)
    bundle = synthesize(req, model)
    compiled = compile_xml(bundle.xml, nlanes=1)
    ops_of = {(b.rank, b.tb_id): [x.operation_id for x in b.steps] for b in bundle.program.blocks}
    network = {op.operation_id for op in bundle.network.operations}
    # the slow step: rank 2's first device step that carries a network transfer
    slow = next((2, b, s) for b, blk in enumerate(compiled.origins(2)) for s, (tb, step) in enumerate(blk)
                if tb >= 0 and ops_of[(2, tb)][step] in network)
    rows = []
    for r in range(4):
        for b, blk in enumerate(compiled.origins(r)):
            for s, (tb, step) in enumerate(blk):
                rows.append({"rank": r, "block": b, "step": s, "xml_tb": tb, "xml_step": step,
                             "duration_us": 1.0 + (50.0 if (r, b, s) == slow else 0.0), "wait_us": 0.0})
    report = {"timeline": rows, "global_span_us": 60.0}
    causes = trace_causes(report, bundle, tails=3)
    assert causes and causes[0].kind == "trace_tail" and causes[0].detail["rank"] == 2
    ops = {op.operation_id for op in bundle.network.operations}
    assert all(c.operation_id in ops for c in causes)
    analysis = analyze(bundle, model, trace=report)
    assert analysis.causes[0].kind == "trace_tail"
    assert any(causes[0].operation_id in s.operations for s in analysis.strategies)


def test_joint_repair_keeps_only_merges_the_exact_replay_confirms():
    """Column gains do not add: the greedy pass re-predicts every merge and drops the ones that do not help."""
    from dataclasses import replace
    from types import SimpleNamespace
    from vericcl_b200.composer.compose import NetworkCandidate, NetworkOperation
    from vericcl_b200.tuning.event_columns import solve_event_columns
    ops = tuple(NetworkOperation("op%d" % i, "send", 0, 1, 0, 0, frozenset({i}), frozenset({i}), frozenset(),
                                 float(i), i) for i in range(4))
    base = NetworkCandidate(2, 4, 1024, ops, "base")
    gain = {"op0": 3.0, "op1": 2.0, "op2": 1.5, "op3": 1.0}
    hurts = {("op0", "op2")}                  # these two changes collide when merged

    def lower(candidate):
        changed = sorted(op.operation_id for op in candidate.operations if op.channel == 1)
        t = 20.0 - sum(gain[k] for k in changed)
        if any(a in changed and b in changed for a, b in hurts):
            t += 10.0
        return SimpleNamespace(network=candidate, t_pred_us=t, can_execute=True)

    incumbent = SimpleNamespace(network=base, t_pred_us=20.0)
    improving = []
    for op in ops:
        variant = replace(base, operations=tuple(replace(o, channel=1) if o is op else o for o in ops))
        improving.append(("s", variant, lower(variant)))
    best = solve_event_columns(incumbent, improving, lower=lower)
    assert best is not None
    # op0 + op1 + op3 (op2 would cost 10 more): 20 - 3 - 2 - 1 = 14
    assert best.t_pred_us == pytest.approx(14.0)


def test_storage_reuse_edges_on_the_critical_path_are_named():
    """With the smallest scratch budget that fits, reuse edges appear; the analysis separates them from data edges."""
    from vericcl_b200.errors import ScratchBudgetError
    from vericcl_b200.verification.bottlenecks import dependency_kinds, storage_causes
    d = example_documents("allreduce", "hierarchy", 4, total_size_bytes=16 * 1024, slice_size_bytes=1024,
                          scratch_bytes=1024)
    with pytest.raises(ScratchBudgetError) as info:
        synthesize(resolve_documents(d))
    d["runtime"]["scratch_bytes_per_rank"] = info.value.needed_bytes
    req = resolve_documents(d)
    bundle = synthesize(req, timing=False)
    kinds = dependency_kinds(bundle.storage)
    assert "data" in kinds.values()
    if bundle.storage.reuse:
        assert "storage" in kinds.values() or all((r, rec["writer"]) in kinds for rec in bundle.storage.reuse
                                                  for r in rec["previous_readers"])
    path = bundle.prediction.critical_path(bundle.executable)
    for cause in storage_causes(bundle, path):
        assert cause.kind == "storage_wait"
        assert cause.detail["scratch_bytes_per_rank_to_remove"] > info.value.needed_bytes - 1
    analysis = analyze(bundle, initial_cost_model(req))
    assert analysis.causes
