"""Unit tests of helpers otherwise exercised only through the workflow: strict JSON, the isomorphism signature,
bandwidth packing of broadcast trees and the fixed-route timing MILP."""
import json

import pytest

from vericcl_b200.composer import compose_routes
from vericcl_b200.errors import InputValidationError
from vericcl_b200.examples import example_documents
from vericcl_b200.input.loader import resolve_documents
from vericcl_b200.solver.demands import build_demands
from vericcl_b200.solver.routing import choose_trees
from vericcl_b200.synthesis import plan_for
from vericcl_b200.topology import load_topology
from vericcl_b200.topology.nvswitch import grouped_topology, nvswitch_topology
from vericcl_b200.utils.jsonio import atomic_write_json, canonical_dumps, strict_load, strict_loads


def _topology(doc, ranks, coll="allgather", slices=1, size=1 << 20):
    d = example_documents(coll, "hierarchy", ranks, total_size_bytes=size * slices, slice_size_bytes=size,
                          topology=doc, scratch_bytes=size * slices * ranks)
    req = resolve_documents(d)
    return req, load_topology(req)


# -- strict JSON ---------------------------------------------------------------------------------------------------
def test_strict_json_rejects_duplicates_non_finite_and_deep_nesting():
    assert strict_loads('{"a": 1, "b": [1, 2.5]}') == {"a": 1, "b": [1, 2.5]}
    for bad in ('{"a": 1, "a": 2}', '{"a": NaN}', '[Infinity]', '{"a": -Infinity}', '{"a": '):
        with pytest.raises(InputValidationError):
            strict_loads(bad)
    with pytest.raises(InputValidationError):
        strict_loads("[" * 70 + "]" * 70)


def test_canonical_dumps_is_order_independent_and_atomic_write_round_trips(tmp_path):
    a, b = {"z": 1, "a": [1, {"y": 2, "b": 3}]}, {"a": [1, {"b": 3, "y": 2}], "z": 1}
    assert canonical_dumps(a) == canonical_dumps(b)
    with pytest.raises(InputValidationError):
        canonical_dumps({"x": float("nan")})
    path = atomic_write_json(tmp_path / "sub" / "doc.json", a)
    assert strict_load(path) == a and json.loads(path.read_text()) == a
    assert not [p for p in path.parent.iterdir() if p.name != "doc.json"]      # no temporary file left behind


# -- isomorphism signature -----------------------------------------------------------------------------------------
def _slow(pairs, ranks=4):
    doc = nvswitch_topology(ranks, nvls=False)
    for e in doc["directed_links"]:
        if (e["src"], e["dst"]) in pairs:
            e["beta_us_per_byte"] *= 4
    return doc


def test_signature_is_invariant_under_relabelling_and_sees_cost_changes():
    from vericcl_b200.topology.isomorphism import canonical_labelling, exact_domain_signature
    _, base = _topology(_slow({(0, 1), (1, 0)}), 4)             # one slow pair breaks the full symmetry
    _, moved = _topology(_slow({(2, 3), (3, 2)}), 4)            # the same domain with ranks relabelled
    assert exact_domain_signature(base) == exact_domain_signature(moved)
    sig, mapping = canonical_labelling(base)
    assert sorted(mapping) == [0, 1, 2, 3] and sorted(mapping.values()) == [0, 1, 2, 3]
    _, changed = _topology(_slow({(0, 1), (1, 0), (2, 3)}), 4)  # a third slow link: not isomorphic any more
    assert exact_domain_signature(changed) != sig
    _, full = _topology(_slow(set()), 4)
    assert exact_domain_signature(full) not in (sig, exact_domain_signature(changed))


# -- bandwidth packing ---------------------------------------------------------------------------------------------
def test_packing_spans_every_destination_and_respects_the_budget():
    from fractions import Fraction
    from vericcl_b200.solver.trees.packing import min_time_budget, pack_bandwidth
    _, topo = _topology(grouped_topology([2, 2], inter_gbps=25.0), 4)
    budget, trees = pack_bandwidth(topo, 0, [1, 2, 3], 4, 1 << 20)
    assert sum(count for _, count in trees) == 4
    for edges, _ in trees:
        reached = {0} | {b for _, b in edges}
        assert {1, 2, 3} <= reached
        assert all(b != 0 for _, b in edges)                   # nothing flows back into the root
    assert budget >= min_time_budget(topo, 0, [1, 2, 3], 4, 1 << 20)
    assert isinstance(budget, Fraction) and budget > 0


# -- fixed-route timing MILP ---------------------------------------------------------------------------------------
def test_timing_milp_respects_dependencies_and_connections():
    from vericcl_b200.solver.timing import makespan, optimize_fixed_routes
    s = 4096
    d = example_documents("allreduce", "hierarchy", 4, total_size_bytes=s * 8, slice_size_bytes=s,
                          max_channels=2, scratch_bytes=s * 8 * 4)
    req = resolve_documents(d)
    topo = load_topology(req)
    plan = plan_for(req, topo)
    dem = build_demands(plan, topo, s)
    net = compose_routes(plan, dem, choose_trees(dem, topo, s), topo, s, channels=2, origin="direct")
    timed = optimize_fixed_routes(net, topo, time_limit=2.0)
    assert "+timing" in timed.origin
    ops = {op.operation_id: op for op in timed.operations}
    from vericcl_b200.topology.model import LinkKey
    dur = {k: topo.link(LinkKey(op.src_rank, op.dst_rank)).time_us(s) for k, op in ops.items()}
    for op in ops.values():
        for dep in op.dependencies:
            assert op.priority_time >= ops[dep].priority_time + dur[dep] - 1e-6
    by_conn = {}
    for op in ops.values():
        by_conn.setdefault((op.src_rank, op.dst_rank, op.channel), []).append(op)
    for members in by_conn.values():
        members.sort(key=lambda o: o.priority_time)
        for a, b in zip(members, members[1:]):
            assert b.priority_time >= a.priority_time + dur[a.operation_id] - 1e-6
    assert makespan(timed, topo) > 0


# -- paths ---------------------------------------------------------------------------------------------------------
def test_shortest_path_sets_respect_allowed_ranks_and_hop_count():
    from vericcl_b200.topology.paths import path_links, path_time_us, shortest_path_set
    doc = nvswitch_topology(4, nvls=False)
    doc["directed_links"] = [e for e in doc["directed_links"] if (e["src"], e["dst"]) != (0, 3)]
    for res in doc["shared_resources"]:
        res["links"] = [pair for pair in res["links"] if tuple(pair) != (0, 3)]
    _, topo = _topology(doc, 4)
    paths = shortest_path_set(topo, 0, 3)
    assert sorted(paths) == [(0, 1, 3), (0, 2, 3)]                  # two hops, both relays
    assert shortest_path_set(topo, 0, 3, allowed={0, 2, 3}) == [(0, 2, 3)]
    assert shortest_path_set(topo, 0, 3, allowed={0, 3}) == []
    assert shortest_path_set(topo, 0, 3, limit=1) in ([(0, 1, 3)], [(0, 2, 3)])
    assert [(k.src, k.dst) for k in path_links((0, 2, 3))] == [(0, 2), (2, 3)]
    one = path_time_us(topo, (0, 2), 1 << 20)
    assert path_time_us(topo, (0, 2, 3), 1 << 20) == pytest.approx(2 * one)


# -- publication ---------------------------------------------------------------------------------------------------
def test_publication_writes_every_artifact_and_a_report(tmp_path):
    import zipfile
    from vericcl_b200.execution.context import RunContext
    from vericcl_b200.execution.publication import publish_results
    ctx = RunContext.create(tmp_path, "case", "solve", run_id="r1", input_files={})
    (ctx.process / "events.jsonl").write_text('{"event": "x"}\n')
    best = {"t_pred_us": 12.5, "model_version": "m1", "origin": "direct",
            "checks": {"semantic": {"status": "valid", "detail": None},
                       "storage": {"status": "valid", "detail": "a|b"}}}
    result = {"status": "ok", "stop_reason": "round limit",
              "recommendations": [{"kind": "slice", "parameters": {"slice_size_bytes": 4096},
                                   "reason_codes": ["step_limit"], "requires_resolve": True}]}
    publish_results(ctx, xml="<algo/>", sidecar={"a": 1}, model={"version": "m1"}, result=result, best=best)
    for name in ("schedule.xml", "schedule.json", "model.json", "report.md", "details.zip"):
        assert (ctx.directory / name).exists(), name
    report = (ctx.directory / "report.md").read_text()
    assert "T_pred: 12.500 us" in report and "| storage | valid | a/b |" in report
    assert "| slice | slice_size_bytes=4096 | step_limit | yes |" in report
    with zipfile.ZipFile(ctx.directory / "details.zip") as z:
        assert any(n.endswith("events.jsonl") for n in z.namelist())


# -- work graph records --------------------------------------------------------------------------------------------
def test_work_operations_validate_their_kind_rules():
    from vericcl_b200.errors import SemanticError
    from vericcl_b200.performance.events import COMM_KINDS, Executable, Movement, WorkOperation
    assert COMM_KINDS == {"send", "rrc", "mc_reduce", "mc_store"}
    send = WorkOperation("s", "send", Movement("link:0:1", 4096), flow_id="f", crosses=("nvlink-tx-0",))
    copy = WorkOperation("c", "copy", Movement("copy:0", 4096), after=("s",))
    nop = WorkOperation("n", "nop", after=("c",), release_us=2.5)
    exe = Executable((send, copy, nop), output_operations=("n",))
    assert exe.by_id()["c"].after == ("s",) and exe.output_operations == ("n",)
    assert (copy.component, copy.nbytes, nop.component, nop.nbytes) == ("copy:0", 4096, None, 0)
    bad = [lambda: WorkOperation("x", "teleport", Movement("k", 1)),
           lambda: WorkOperation("x", "send", Movement("k", 16)),              # network work without a flow
           lambda: WorkOperation("x", "copy"),                                # data work without a movement
           lambda: WorkOperation("x", "nop", Movement("k", 16)),              # a nop that moves data
           lambda: WorkOperation("x", "copy", Movement("k", 16), crosses=("r",)),   # local work on a shared resource
           lambda: Movement("k", 0),
           lambda: Movement("k", True),
           lambda: Movement("", 16),
           lambda: WorkOperation("x", "copy", Movement("k", 16), after=("a", "a")),
           lambda: WorkOperation("x", "copy", Movement("k", 16), estimated="yes"),
           lambda: Executable((copy,)),                                       # waits for an unknown operation
           lambda: Executable((send, send)),
           lambda: Executable((send,), output_operations=("zz",))]
    for make in bad:
        with pytest.raises(SemanticError):
            make()


# -- gradient bucket groups ----------------------------------------------------------------------------------------
def test_bucket_groups_cover_every_bucket_once_in_order():
    from vericcl_b200.models.grad_bucket import bucket_groups
    assert bucket_groups(611, 8) == [(i * 77, min(611, (i + 1) * 77)) for i in range(8)]
    assert bucket_groups(6, 3) == [(0, 2), (2, 4), (4, 6)]
    assert bucket_groups(5, 3) == [(0, 2), (2, 4), (4, 5)]
    assert bucket_groups(2, 8) == [(0, 1), (1, 2)]
    assert bucket_groups(3, 0) == [(0, 3)] and bucket_groups(0, 4) == []
    for n in range(1, 40):
        for g in range(1, 12):
            runs = bucket_groups(n, g)
            assert runs[0][0] == 0 and runs[-1][1] == n and len(runs) <= g
            assert all(a[1] == b[0] for a, b in zip(runs, runs[1:]))


# -- the largest communicator: 16 ranks ----------------------------------------------------------------------------
@pytest.mark.parametrize("coll,slices,variant", [("allreduce", 16, {}), ("allgather", 1, {}),
                                                  ("reduce_scatter", 16, {}), ("allgather", 1, {"push": True}),
                                                  ("allreduce", 16, {"multicast": True}),
                                                  ("allgather", 1, {"merge": False})])
def test_sixteen_rank_programs_on_the_cpu_oracle(coll, slices, variant):
    """The symmetric heap's limit is 16 ranks: schedules of that size compile and run correctly (CPU interpreter,
    seeded CTA order, two launches so flag epochs advance)."""
    import numpy as np
    from vericcl_b200.program.device import compile_xml, run_cpu
    from vericcl_b200.synthesis import schedule_xml
    p = 16
    compiled = compile_xml(schedule_xml(coll, p, slices), nlanes=2, niters=2, **variant)
    count = p * slices * 16
    rng = np.random.default_rng(16)
    inputs = [rng.uniform(-1, 1, count).astype(np.float32) for _ in range(p)]
    outs = run_cpu(compiled, inputs, seed=3, launches=2)
    total = np.sum(inputs, axis=0, dtype=np.float64)
    for r in range(p):
        if coll == "allreduce":
            np.testing.assert_allclose(outs[r][:count], total, rtol=1e-5, atol=1e-5)
        elif coll == "allgather":
            np.testing.assert_array_equal(outs[r][:count * p], np.concatenate(inputs))
        else:
            part = count // p
            np.testing.assert_allclose(outs[r][:part], total[r * part:(r + 1) * part], rtol=1e-5, atol=1e-5)


# -- experiments report pivot --------------------------------------------------------------------------------------
def test_report_pivot_tabulates_x_nccl_by_size(tmp_path, capsys):
    from vericcl_b200.experiments import load_points, main, pivot, report_rows

    def point(coll, gpus, size, x, variant=None, graph=False):
        d = {"coll": coll, "n_gpus": gpus, "bytes_per_rank": size, "time_us": 10.0, "busbw_gbs": 1.0,
             "path": "interp", "graph": graph, "nccl_time_us": 10.0 * x, "speedup_vs_nccl": x}
        if variant:
            d["variant"] = variant
        return json.dumps(d)

    log = tmp_path / "sweep.log"
    log.write_text("\n".join([point("allreduce", 8, 1 << 20, 1.5), point("allreduce", 8, 1 << 24, 0.9),
                              point("allgather", 8, 1 << 24, 1.1), point("allreduce", 8, 1 << 20, 2.0, "BULK=1"),
                              point("allreduce", 8, 1 << 10, 3.0, graph=True)]) + "\n")
    rows = report_rows(load_points([log]))
    table = pivot(rows)
    lines = table.splitlines()
    assert lines[0] == "| coll | GPUs | mode | 1 KiB | 1 MiB | 16 MiB |"
    assert "| allreduce | 8 | eager |  | 1.50 | 0.90* |" in lines
    assert "| allreduce | 8 | graph | 3.00 |  |  |" in lines
    assert "| allgather | 8 | eager |  |  | 1.10 |" in lines
    assert lines[-1] == "1 of 4 cells below 1.0 (marked *)"
    assert "2.00" in pivot(rows, variant="BULK=1") and "1.50" not in pivot(rows, variant="BULK=1")
    assert main(["report", str(log), "--pivot"]) == 0
    assert "0.90*" in capsys.readouterr().out


# -- slack and near-critical operations ----------------------------------------------------------------------------
def test_slack_index_finds_every_chain_that_ends_at_t_pred():
    from vericcl_b200.performance import CostModel, Executable, ServiceCost, WorkOperation, predict
    from vericcl_b200.performance.events import Movement
    from vericcl_b200.verification.bottlenecks import near_critical, slack_index
    services = {"copy:0": (ServiceCost(0.0, 0.01),), "copy:1": (ServiceCost(0.0, 0.01),),
                "copy:2": (ServiceCost(0.0, 0.01),)}
    model = CostModel("slack", services, {})
    ops = (WorkOperation("a1", "copy", Movement("copy:0", 1000)),                  # 10 µs
           WorkOperation("a2", "copy", Movement("copy:0", 1000), after=("a1",)),   # ends at 20
           WorkOperation("b1", "copy", Movement("copy:1", 2000)),                  # ends at 20: a second chain
           WorkOperation("c1", "copy", Movement("copy:2", 500)),                   # ends at 5: 15 µs of slack
           WorkOperation("end", "nop", after=("a2", "b1", "c1")))
    ex = Executable(ops)
    pred = predict(ex, model, exact=True)
    assert pred.t_pred_us == pytest.approx(20.0)
    slack = slack_index(ex, pred)
    assert slack["a1"] == pytest.approx(0.0) and slack["a2"] == pytest.approx(0.0)
    assert slack["b1"] == pytest.approx(0.0) and slack["c1"] == pytest.approx(15.0)
    crit = near_critical(ex, pred)
    assert set(crit) == {"a1", "a2", "b1"}                  # both chains, never the nop or the slack operation
    path = pred.critical_path(ex)
    assert not ({"a1", "a2"} <= set(path) and "b1" in path)  # the single critical path covers one chain only


# -- cut bound under measured sharing modes ------------------------------------------------------------------------
def test_cut_rate_uses_measured_modes_only_on_their_own_links_and_resources():
    from fractions import Fraction
    from vericcl_b200.performance import RateProfile
    from vericcl_b200.performance.initial import initial_cost_model
    from vericcl_b200.verification.global_bound import _rate
    req, topo = _topology(grouped_topology([2, 2], inter_gbps=25.0), 4, coll="allreduce", slices=4)
    model = initial_cost_model(req)
    base = _rate(topo, {0, 1}, model)
    assert base == Fraction(25000)                     # the group's NIC: 25 GB/s out of group {0, 1}
    # a measured mode of two NVLink flows inside group 0 must not lift the inter-group cut
    fast = RateProfile("nvlink-pair", frozenset({"send:0:1:c1", "send:1:0:c1"}),
                       {"send:0:1:c1": 700000.0, "send:1:0:c1": 700000.0})
    with_mode = model.with_updates("m2", profiles=(fast,))[0]
    assert _rate(topo, {0, 1}, with_mode) == base
    # a measured mode through the NIC that beats its nominal capacity raises the cut to what was measured
    nic = RateProfile("nic-pair", frozenset({"send:0:2:c1", "send:1:3:c1"}),
                      {"send:0:2:c1": 20000.0, "send:1:3:c1": 20000.0})
    with_nic = model.with_updates("m3", profiles=(nic,))[0]
    assert _rate(topo, {0, 1}, with_nic) == Fraction(40000)
