import random

import pytest

from vericcl_b200.examples import example_documents
from vericcl_b200.input.loader import resolve_documents
from vericcl_b200.online import campaign
from vericcl_b200.online.acceptance import compare_measured, one_sided_binomial, pair_order
from vericcl_b200.online.clock_sync import align_bracketed_globaltimers, ordered
from vericcl_b200.online.fitting import Sample, fit_curve, qualify
from vericcl_b200.online.probe_jobs import build_probe_xml, plan_probes
from vericcl_b200.online.statistical_ledger import StatisticalLedger
from vericcl_b200.online.trace import TraceRecord, analyze_trace_causality, parse_trace, write_trace
from vericcl_b200.performance.initial import initial_cost_model
from vericcl_b200.program.device import compile_xml, run_cpu
from vericcl_b200.topology import load_topology


def request(**kw):
    d = example_documents("allreduce", "hierarchy", 4, total_size_bytes=1 << 16, slice_size_bytes=1 << 14, **kw)
    d["sketch"]["calibration"]["enabled"] = True
    return resolve_documents(d)


def test_probe_plan_and_xml_compile():
    req = request()
    jobs = plan_probes(req, load_topology(req))
    assert jobs[0].group == "link_intra"
    assert any(j.mode == "shared" for j in jobs)
    assert all(len(j.payload_sizes) >= 3 for j in jobs)
    for job in jobs[:6] + [j for j in jobs if j.mode == "shared"][:2]:
        c = compile_xml(build_probe_xml(job, 4))
        import numpy as np
        outs = run_cpu(c, [np.ones(len(job.flows) * 8, np.float32)] * 4)
        assert all(np.isfinite(o).all() for o in outs)


def test_fit_curve_recovers_alpha_beta():
    samples = [Sample("link:0:1", b, 2.0 + b / 1000.0, "native_interpreter", l) for b in (1000, 4000, 16000)
               for l in range(3)]
    good, reasons = qualify(samples, max_cv=0.05)
    seg = fit_curve(good, max_relative_error=0.01)
    assert seg[0].alpha_us == pytest.approx(2.0, rel=1e-6)
    assert seg[0].beta_us_per_byte == pytest.approx(1e-3, rel=1e-6)


def test_simulated_samples_never_qualify():
    req = request()
    model, diff, report = campaign.run_calibration(req, load_topology(req), initial_cost_model(req),
                                                   campaign.simulated_executor(load_topology(req)))
    assert model.version.startswith("initial") and not diff


def test_campaign_publishes_measured_model(monkeypatch):
    req = request()
    topo = load_topology(req)
    executor = campaign.simulated_executor(topo, source="native_interpreter", noise=0.001)
    model, diff, report = campaign.run_calibration(req, topo, initial_cost_model(req), executor)
    assert model.version.startswith("measured-")
    assert model.service_for("link:0:1", 1 << 14).source == "measured"
    assert model.profiles, "shared modes must produce measured rate profiles"


def test_paired_acceptance_and_ledger(tmp_path):
    assert one_sided_binomial(10, 10) == pytest.approx(1 / 1024)
    assert sorted(pair_order(4, 1)).count("AB") == 2
    rng = random.Random(0)
    verdict = compare_measured(lambda label: (100.0 if label == "A" else 90.0) * (1 + rng.uniform(-.001, .001)),
                               pairs=20, seed=3, alpha=0.01, max_cv=0.05, max_rounds=3, min_relative_gain=0.05)
    assert verdict.accepted and verdict.median_gain == pytest.approx(0.1, abs=0.01)
    sim = compare_measured(lambda label: 1.0, pairs=4, seed=1, alpha=0.05, max_cv=0.05, max_rounds=1,
                           min_relative_gain=0.0, source="test_simulation")
    assert not sim.accepted
    ledger = StatisticalLedger(tmp_path / "ledger.jsonl", task_alpha=0.05)
    a1, a2 = ledger.allocate("x"), ledger.allocate("y")
    assert a1 == pytest.approx(0.025) and a2 == pytest.approx(0.0125)
    assert ledger.spent() <= 0.05 and ledger.verify()
    (tmp_path / "ledger.jsonl").write_text((tmp_path / "ledger.jsonl").read_text().replace("0.0125", "0.02"))
    assert not ledger.verify()


def test_clock_alignment_and_trace(tmp_path):
    maps = align_bracketed_globaltimers({0: [(1000 + i * 100, 500 + i * 100, 1010 + i * 100) for i in range(8)],
                                         1: [(1000 + i * 100, 9000 + i * 100, 1004 + i * 100) for i in range(8)]})
    assert maps[0].to_host(500) == pytest.approx(1005, abs=6)
    assert maps[1].to_host(9000) == pytest.approx(1002, abs=3)
    assert ordered((0, 1), (2, 3)) == "before" and ordered((0, 5), (2, 3)) == "uncertain"
    recs = [TraceRecord(0, 0, 0, 0, 0, s, 1, 500 + s * 10, 505 + s * 10, 2) for s in range(4)]
    write_trace(tmp_path / "t.bin", 0, 1, 4, recs)
    parsed = parse_trace((tmp_path / "t.bin").read_bytes())
    assert parsed["complete"] and parsed["records"] == recs
    partial = parse_trace((tmp_path / "t.bin").read_bytes()[:-10])
    assert not partial["complete"] and len(partial["records"]) == 3
    report = analyze_trace_causality({0: recs, 1: [r.__class__(1, *list(r.__dict__.values())[1:]) for r in recs]},
                                     maps)
    assert report["global_span_us"] > 0 and report["tails"]


def test_online_loop_two_groups_without_gpu(tmp_path, capsys):
    """The emulated 2×4 online loop runs end to end; without GPUs calibration and measurement are skipped."""
    import json
    from pathlib import Path
    from vericcl_b200.online import measure
    from vericcl_b200.online.loop import loop_documents, run_loop
    docs = loop_documents(groups=2, per_group=4, inter_gbps=25.0, size_bytes=1 << 23, rounds=1,
                          datatype="float32", pairs=4)
    assert docs["topology"]["ranks"] == 8
    assert any(r["kind"] == "nic" for r in docs["topology"]["shared_resources"])
    summary = run_loop(tmp_path, size_bytes=1 << 23, rounds=1, pairs=4, measure_final=False)
    assert summary["exit_code"] == 0
    assert summary["best"]["checks"]["semantic"]["status"] == "valid"
    assert len(summary["rounds"]) == 1
    assert summary["rounds"][0]["cut_lower_bound_us"] <= summary["rounds"][0]["start_t_pred_us"]
    # the measure CLI re-predicts the solved schedule from its sidecar (no GPU: prediction only)
    run = Path(summary["run"])
    capsys.readouterr()
    assert measure.main(["--inputs", str(tmp_path / "inputs" / "online-loop"), "--xml", str(run / "schedule.xml"),
                         "--sidecar", str(run / "schedule.json"), "--no-measure"]) == 0
    out = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    assert abs(out["t_pred_us"] - summary["best"]["t_pred_us"]) < 1e-6 * out["t_pred_us"]


def test_trace_buffer_decoding_with_uneven_blocks():
    """Records are decoded per block: block 0 has 3 steps, block 1 has 1 step, two iterations, two lanes."""
    from vericcl_b200.online.trace import records_from_buffer
    nblocks, nlanes, max_steps, niters = 2, 2, 3, 2
    buf = [0] * (nblocks * nlanes * max_steps * niters * 3)
    block_ops = [[1, 2, 0], [4]]
    for cta in range(nblocks * nlanes):
        nsteps = len(block_ops[cta // nlanes])
        for it in range(niters):
            for s in range(nsteps):
                base = (cta * max_steps * niters + it * nsteps + s) * 3
                buf[base:base + 3] = [1000 * cta + 100 * it + 10 * s + 1, 1000 * cta + 100 * it + 10 * s + 5, 2]
    recs = records_from_buffer(0, buf, nblocks=nblocks, nlanes=nlanes, steps_per_iter=max_steps, niters=niters,
                               block_ops=block_ops)
    assert len(recs) == 2 * 2 * 3 + 2 * 2 * 1
    for r in recs:
        assert r.start_ns == 1000 * r.cta + 100 * r.iteration + 10 * r.step + 1
        assert r.op == block_ops[r.block][r.step]


def test_trace_timeline_offsets():
    from vericcl_b200.online.clock_sync import ClockMap
    from vericcl_b200.online.trace import TraceRecord
    from vericcl_b200.online.trace_worker import timeline
    traces = {0: [TraceRecord(0, 0, 0, 0, 0, 0, 1, 1000, 3000, 500), TraceRecord(0, 0, 0, 0, 0, 1, 2, 5000, 6000, 0)],
              1: [TraceRecord(1, 0, 0, 0, 0, 0, 1, 10_000, 11_000, 100)]}
    clocks = {0: ClockMap(0.0, 0.0, 10.0), 1: ClockMap(-8000.0, 0.0, 10.0)}
    rows = {(r["rank"], r["step"]): r for r in timeline(traces, clocks)}
    assert rows[(0, 0)]["start_us"] == 0.0 and rows[(0, 1)]["local_start_us"] == 4.0
    assert rows[(1, 0)]["start_us"] == 1.0 and rows[(1, 0)]["local_start_us"] == 0.0
    assert rows[(0, 0)]["duration_us"] == 2.0 and rows[(0, 0)]["wait_us"] == 0.5


def test_step_counters_accumulate_over_launches():
    from vericcl_b200.online.trace import TraceRecord, step_counters
    recs = [TraceRecord(0, 0, 1, 0, 0, 2, 5, 100, 150, 30), TraceRecord(0, 1, 1, 1, 0, 2, 5, 300, 370, 10),
            TraceRecord(0, 0, 1, 0, 0, 2, 5, 1000, 1040, 0), TraceRecord(1, 0, 0, 0, 0, 0, 1, 50, 60, 5)]
    c = step_counters(recs)
    a = c[(0, 1, 2)]
    assert a["samples"] == 3 and a["service_ns"] == 50 + 70 + 40 and a["dependency_wait_ns"] == 40
    assert a["max_service_ns"] == 70 and a["first_ns"] == 100 and a["last_ns"] == 1040
    assert a["mean_service_ns"] == pytest.approx(160 / 3) and a["mean_wait_ns"] == pytest.approx(40 / 3)
    assert c[(1, 0, 0)]["samples"] == 1


def test_bracket_fit_recovers_offset_and_drift_and_drops_a_contradicting_sample():
    import random
    from vericcl_b200.online.clock_sync import fit_transform
    rng = random.Random(3)
    offset, drift = 12_345.0, 3e-6
    samples = []
    for i in range(24):
        g = 1_000_000.0 + i * 50_000.0
        true = offset + g * (1 + drift)
        samples.append((true - rng.uniform(50, 400), g, true + rng.uniform(50, 400)))
    m = fit_transform(samples)
    assert m.method == "bracket-lp" and m.samples_used == 24
    for lo, g, hi in samples:
        assert lo - 1e-6 <= m.to_host(g) <= hi + 1e-6          # inside every bracket
    assert abs(m.to_host(2_000_000.0) - (offset + 2_000_000.0 * (1 + drift))) <= m.uncertainty_ns + 400
    # a sample whose GPU read came 5 µs late contradicts the rest and is dropped
    bad = samples + [(offset + 1_500_000.0, 1_500_000.0 + 5_000.0, offset + 1_500_000.0 + 2_000.0)]
    m2 = fit_transform(bad)
    assert m2.method == "bracket-lp" and m2.samples_used == 24


def test_link_class_probing_measures_representatives_and_covers_every_link():
    """On 2 x 4 groups, a few probe jobs (two links per class, one rank per node, one shared mode per resource
    class) stand in for the 168 of per-link probing; every link and local component ends up measured."""
    from vericcl_b200.online.loop import loop_documents
    from vericcl_b200.online.probe_jobs import link_classes, plan_probes
    docs = loop_documents(groups=2, per_group=4, inter_gbps=25.0, size_bytes=8 << 20, rounds=1,
                          datatype="float32", pairs=2)
    req = resolve_documents(docs)
    topo = load_topology(req)
    assert docs["sketch"]["calibration"]["probe_scope"] == "link_classes"
    jobs = plan_probes(req, topo)
    every = dict(docs)
    every["sketch"] = dict(docs["sketch"], calibration=dict(docs["sketch"]["calibration"], probe_scope="every_link"))
    assert len(jobs) < len(plan_probes(resolve_documents(every), topo)) // 5
    assert len(link_classes(topo)) == 2                 # intra-group and inter-group links
    shared = {j.resources[0] for j in jobs if j.mode == "shared"}
    # one NVLink port, one group NIC and one rank's share of it: three classes, each probed once
    assert any(r.startswith("nvlink-") for r in shared) and any(r.startswith("nic-share-rx-") for r in shared)
    assert any(r.startswith("nic-") and "share" not in r for r in shared)
    model = initial_cost_model(req)
    executor = campaign.simulated_executor(topo, source="native_interpreter", noise=0.001)
    new_model, _, report = campaign.run_calibration(req, topo, model, executor)
    for key in new_model.services:
        if key.split(":")[0] in ("link", "rrc", "copy", "reduce"):
            assert new_model.services[key][0].source == "measured", key
    assert report["represented"]


def test_rank_shares_describe_the_emulated_link():
    """With rank shares every rank reads from the other groups through its own inter_gbps / group-size resource."""
    from vericcl_b200.topology.nvswitch import grouped_topology, multinode_topology
    doc = multinode_topology(2, 4, inter_gbps=25.0, rank_shares=True)
    shares = {r["id"]: r for r in doc["shared_resources"] if r["id"].startswith("nic-share-rx-")}
    assert sorted(shares) == ["nic-share-rx-%d" % r for r in sorted(range(8), key=lambda r: "nic-share-rx-%d" % r)]
    for rid, res in shares.items():
        rank = int(rid.rsplit("-", 1)[1])
        assert res["capacity_bytes_per_us"] == 25.0 * 1000.0 / 4
        assert all(dst == rank and src // 4 != rank // 4 for src, dst in res["links"])
    plain = grouped_topology([3, 1], rank_shares=False)
    assert not any(r["id"].startswith("nic-share") for r in plain["shared_resources"])
    uneven = grouped_topology([3, 1], inter_gbps=30.0, rank_shares=True)
    caps = {r["id"]: r["capacity_bytes_per_us"] for r in uneven["shared_resources"] if "share" in r["id"]}
    assert caps["nic-share-rx-0"] == 10000.0 and caps["nic-share-rx-3"] == 30000.0


def test_online_loop_dry_run_adopts_a_measured_improvement(tmp_path):
    """The 2 x 4 loop end to end on the host: the probe campaign runs on an analytic executor, and the paired
    acceptance measures a stand-in device whose times follow the exact prediction (with 0.2 % noise), so a
    candidate the model predicts faster is adopted through the statistics, with its ledger entries written."""
    import random
    from types import SimpleNamespace
    from vericcl_b200.execution.context import RunContext
    from vericcl_b200.input.loader import load_request
    from vericcl_b200.examples import write_documents
    from vericcl_b200.online.acceptance import compare_measured
    from vericcl_b200.online.loop import loop_documents
    from vericcl_b200.workflow import PrimaryWorkflow
    docs = loop_documents(groups=2, per_group=4, inter_gbps=25.0, size_bytes=128 << 20, rounds=2,
                          datatype="float32", pairs=6)
    files = write_documents(tmp_path / "in", docs)
    req = load_request(files)
    topo = load_topology(req)
    ctx = RunContext.create(tmp_path, "c", "solve", run_id="r", input_files=files)
    ctx.update_run_json(effective_request=dict(req.request_config))
    rng = random.Random(5)
    verdicts = []

    def measure(incumbent, candidate):
        times = {"A": incumbent.t_pred_us, "B": candidate.t_pred_us}
        verdict = compare_measured(lambda label: times[label] * (1 + rng.uniform(-0.002, 0.002)), pairs=6,
                                   seed=1, alpha=0.05, max_cv=0.05, max_rounds=2, min_relative_gain=0.0)
        verdicts.append(verdict)
        return verdict
    executor = campaign.simulated_executor(topo, source="native_interpreter", noise=0.001)
    wf = PrimaryWorkflow(req, ctx, probe_executor=executor, measure=measure)
    result = wf.run()
    assert result.status == "ok"
    assert verdicts and all(v.accepted for v in verdicts), verdicts
    adopted = [r for r in result.rounds if r.get("result") == "improved"]
    assert len(adopted) == len(verdicts)
    for r in adopted:
        assert r["t_pred_us"] < r["start_t_pred_us"]
        # the cut bound under the calibrated model stays the link bound: 128 MiB into a group over 25 GB/s
        assert r["cut_lower_bound_us"] == pytest.approx((128 << 20) / 25e3, rel=1e-3)
    assert (ctx.process / "reports" / "calibration.json").exists()


def test_recalibration_replaces_measured_sharing_modes():
    """Publishing a second calibration of the same modes keeps one mode per flow set (no duplicate ids)."""
    from vericcl_b200.performance import RateProfile
    base = initial_cost_model(resolve_documents(example_documents("allgather", "hierarchy", 4,
                                                                  total_size_bytes=1 << 20,
                                                                  slice_size_bytes=1 << 18)))
    mode = RateProfile("shared-x-0", frozenset({"send:0:1:c1", "send:2:1:c1"}),
                       {"send:0:1:c1": 300.0, "send:2:1:c1": 300.0})
    first, _ = campaign.publish_model(base, {}, (mode,), stamp="2026-01-01T00:00:00+00:00")
    again = RateProfile("shared-x-0", mode.flows, {"send:0:1:c1": 320.0, "send:2:1:c1": 310.0})
    second, _ = campaign.publish_model(first, {}, (again,), stamp="2026-01-02T00:00:00+00:00")
    assert [p.rates["send:0:1:c1"] for p in second.profiles] == [320.0]
    renamed = RateProfile("shared-y-0", mode.flows, {"send:0:1:c1": 330.0, "send:2:1:c1": 330.0})
    third, _ = campaign.publish_model(second, {}, (renamed,), stamp="2026-01-03T00:00:00+00:00")
    assert [p.profile_id for p in third.profiles] == ["shared-y-0"]


def test_calibrated_model_round_trips_into_verify_and_tune(tmp_path):
    """A solve calibrated on the analytic executor publishes a model with measured sharing modes; verifying and
    tuning the published schedule under that model keeps the cut bound at the link bound and never gets worse."""
    from vericcl_b200.execution.context import RunContext
    from vericcl_b200.examples import write_documents
    from vericcl_b200.input.loader import load_request
    from vericcl_b200.online.loop import loop_documents
    from vericcl_b200.performance.model import CostModel
    from vericcl_b200.utils.jsonio import strict_load
    from vericcl_b200.workflow import PrimaryWorkflow
    docs = loop_documents(groups=2, per_group=2, inter_gbps=25.0, size_bytes=8 << 20, rounds=1,
                          datatype="float32", pairs=4)
    docs["sketch"]["trace_and_measure"]["enabled"] = False
    files = write_documents(tmp_path / "in", docs)
    req = load_request(files)
    topo = load_topology(req)
    ctx = RunContext.create(tmp_path, "c", "solve", run_id="r", input_files=files)
    ctx.update_run_json(effective_request=dict(req.request_config))
    executor = campaign.simulated_executor(topo, source="native_interpreter", noise=0.001)
    solved = PrimaryWorkflow(req, ctx, probe_executor=executor).run()
    assert solved.status == "ok"
    model = CostModel.from_json(strict_load(ctx.directory / "model.json"))
    assert model.profiles and model.version.startswith("measured-")
    req2 = load_request(files, purpose="verify")
    ctx2 = RunContext.create(tmp_path, "c", "verify", run_id="v", input_files=files)
    ctx2.update_run_json(effective_request=dict(req2.request_config))
    verified = PrimaryWorkflow(req2, ctx2, purpose="verify", tune=True, model=model,
                               verify_inputs={"xml": (ctx.directory / "schedule.xml").read_text(),
                                              "sidecar": strict_load(ctx.directory / "schedule.json")}).run()
    assert verified.status == "ok"
    assert verified.best["t_pred_us"] <= solved.best["t_pred_us"] + 1e-9
    bound = verified.rounds[0]["cut_lower_bound_us"]
    assert (8 << 20) / 25e3 <= bound <= verified.best["t_pred_us"]
