import json
import os
import subprocess
import sys
from pathlib import Path

import pytest

from vericcl_b200.cli.main import main
from vericcl_b200.examples import example_documents, write_documents

ROOT = Path(__file__).resolve().parents[1]


def _args(indir, project, case, run_id):
    return ["--project-root", str(project), "--case", case, "--run-id", run_id,
            "--topology", str(indir / "topology.json"), "--sketch", str(indir / "sketch.json"),
            "--atom", str(indir / "atom.json"), "--runtime", str(indir / "runtime.json")]


@pytest.fixture
def inputs(tmp_path):
    d = example_documents("allgather", "hierarchy", 4, total_size_bytes=1 << 16, slice_size_bytes=1 << 14,
                          tuning_rounds=2, alpha_us=2.0, link_gbps=150.0)
    write_documents(tmp_path / "in", d)
    return tmp_path / "in"


def test_solve_publishes_and_verify_roundtrip(inputs, tmp_path, capsys):
    assert main(["solve"] + _args(inputs, tmp_path, "c", "s1")) == 0
    run = tmp_path / "examples" / "c" / "output" / "s1"
    for name in ("run.json", "report.md", "schedule.xml", "schedule.json", "model.json", "details.zip",
                 "checkpoint.json", "process/events.jsonl"):
        assert (run / name).exists(), name
    meta = json.loads((run / "run.json").read_text())
    assert meta["status"] == "finished" and meta["best"]["t_pred_us"] > 0
    assert meta["value_sources"]["sketch.collective.operator"]["kind"] == "input"
    rc = main(["verify"] + _args(inputs, tmp_path, "c", "v1") + ["--xml", str(run / "schedule.xml"), "--sidecar",
                                                                 str(run / "schedule.json"), "--model",
                                                                 str(run / "model.json")])
    assert rc == 0
    vmeta = json.loads((tmp_path / "examples" / "c" / "output" / "v1" / "run.json").read_text())
    assert vmeta["best"]["t_pred_us"] == pytest.approx(meta["best"]["t_pred_us"])
    assert main(["inspect", "--run", str(run)]) == 0


def test_invalid_input_exit_code(inputs, tmp_path):
    rc = main(["solve"] + _args(inputs, tmp_path, "c", "bad") + ["--set", "sketch.collective.datatype=\"int8\""])
    assert rc == 2


def test_resume_after_interruption(inputs, tmp_path):
    from vericcl_b200.execution.context import RunContext
    from vericcl_b200.input.loader import load_request
    from vericcl_b200.workflow import PrimaryWorkflow
    files = {k: inputs / (k + ".json") for k in ("topology", "sketch", "atom", "runtime")}
    req = load_request(files)
    ctx = RunContext.create(tmp_path, "c", "solve", run_id="r", input_files=files)
    ctx.update_run_json(effective_request=dict(req.request_config))
    wf = PrimaryWorkflow(req, ctx)
    wf.initial_candidates()         # interrupted after the initial stage's checkpoint
    assert main(["resume", "--run", str(ctx.directory)]) == 0
    meta = json.loads((ctx.directory / "run.json").read_text())
    assert meta["status"] == "finished" and meta["best"] is not None


def test_module_entry_point(inputs, tmp_path):
    env = dict(os.environ, PYTHONPATH=str(ROOT))
    proc = subprocess.run([sys.executable, "-m", "vericcl_b200", "--version"], capture_output=True, text=True,
                          env=env, timeout=120)
    assert proc.returncode == 0 and "vericcl_b200" in proc.stdout


def test_measured_rejection_is_not_repeated(tmp_path):
    """A repair candidate the paired measurement rejected is not measured again in later rounds."""
    from types import SimpleNamespace

    from vericcl_b200.execution.context import RunContext
    from vericcl_b200.input.loader import load_request
    from vericcl_b200.online.loop import loop_documents
    from vericcl_b200.workflow import PrimaryWorkflow
    docs = loop_documents(groups=2, per_group=4, inter_gbps=25.0, size_bytes=128 << 20, rounds=3,
                          datatype="float32", pairs=4)
    docs["sketch"]["calibration"]["enabled"] = False
    files = write_documents(tmp_path / "in", docs)
    req = load_request(files)
    ctx = RunContext.create(tmp_path, "c", "solve", run_id="r", input_files=files)
    ctx.update_run_json(effective_request=dict(req.request_config))
    calls = []

    def measure(incumbent, candidate):
        calls.append(candidate.xml)
        return SimpleNamespace(accepted=False, reason="slower")
    wf = PrimaryWorkflow(req, ctx, measure=measure)
    result = wf.run()
    assert result.status == "ok"
    assert calls and len(calls) == len(set(calls))
    assert len(result.rounds) == 3


def test_experiment_report_tables(tmp_path):
    from vericcl_b200.experiments import load_points, markdown, matrix_commands, report_rows
    log = tmp_path / "sweep.log"
    log.write_text("noise line\n"
                   '{"coll": "allreduce", "n_gpus": 4, "bytes_per_rank": 1024, "time_us": 6.1, "busbw_gbs": 0.25, '
                   '"path": "oneshot", "nvls": true, "graph": true, "nccl_time_us": 18.7, "speedup_vs_nccl": 3.08, '
                   '"max_rel_err_vs_fp64": 0.002}\n'
                   '{"summary": true, "points": 1}\n')
    rows = report_rows(load_points([log]))
    assert len(rows) == 1 and rows[0]["path"] == "one-shot NVLS" and rows[0]["size"] == "1 KiB"
    table = markdown(rows)
    assert "| allreduce | 4 | graph | 1 KiB | one-shot NVLS |  | 6.1 |" in table
    # one-shot NVLS lines: 2 bytes of line per payload byte, multicast into all 4 GPUs: 8 KiB in 6.1 µs
    assert rows[0]["nvlink_gbs"] == round(8192 / 6.1e-6 / 1e9, 1)
    # a reference sweep point of the same (collective, GPUs, size) fills the reference columns
    log.write_text(log.read_text() + '{"impl": "reference", "coll": "allreduce", "bytes_per_rank": 1024, '
                   '"ranks": 4, "us": 30.5, "busbw_gbs": 0.05}\n')
    rows = report_rows(load_points([log]))
    assert len(rows) == 1 and rows[0]["ref_us"] == 30.5 and rows[0]["x_ref"] == 5.0
    cmds = matrix_commands([2, 8], graph=True)
    assert cmds[1][4] == "--nproc-per-node=8" and cmds[1][-1] == "--graph"


def test_calibration_reuse_adopts_a_cached_model(tmp_path):
    from vericcl_b200.execution.context import RunContext
    from vericcl_b200.input.loader import load_request
    from vericcl_b200.online.campaign import save_calibration
    from vericcl_b200.workflow import PrimaryWorkflow
    index = tmp_path / "calibrations.json"
    d = example_documents("allgather", "hierarchy", 4, total_size_bytes=1 << 16, slice_size_bytes=1 << 14,
                          calibration=True)
    d["sketch"]["history"] = {"calibration_reuse": True, "calibration_index": str(index),
                              "calibration_max_age_s": 3600}
    files = write_documents(tmp_path / "in", d)
    req = load_request(files)
    ctx = RunContext.create(tmp_path, "c", "solve", run_id="r1", input_files=files)

    def no_probes(job):
        raise AssertionError("a fresh cached calibration must not run probes")
    wf = PrimaryWorkflow(req, ctx, probe_executor=no_probes)
    cached, _ = wf.model.with_updates("measured-cached")
    save_calibration(index, wf._calibration_identity(), cached)
    assert wf.calibration() is True and wf.model.version == "measured-cached"
    # a different workload (datatype) has another identity and falls back to probing (none here: skipped)
    d["sketch"]["collective"]["datatype"] = "bfloat16"
    files2 = write_documents(tmp_path / "in2", d)
    wf2 = PrimaryWorkflow(load_request(files2), RunContext.create(tmp_path, "c", "solve", run_id="r2",
                                                                  input_files=files2))
    assert wf2.calibration() is False and wf2.model.version != "measured-cached"


def test_tuning_with_a_slice_chosen_by_the_parameter_domain(tmp_path):
    """No fixed slice size: the domain picks it, and the tuning round's cut bound uses the incumbent's slices."""
    d = example_documents("reduce_scatter", "hierarchy", 4, total_size_bytes=256 << 10, slice_size_bytes=None,
                          tuning_rounds=1, calibration=False)
    write_documents(tmp_path / "in", d)
    assert main(["solve"] + _args(tmp_path / "in", tmp_path, "c", "auto-slice")) == 0
    meta = json.loads((tmp_path / "examples" / "c" / "output" / "auto-slice" / "run.json").read_text())
    assert meta["best"]["slice_size_bytes"] > 0 and meta["result"]["rounds"]


def test_history_lookup_without_a_fixed_slice(tmp_path):
    from vericcl_b200.input.loader import resolve_documents
    from vericcl_b200.solver.history import find_schedules, save_schedule
    from vericcl_b200.synthesis import synthesize
    from vericcl_b200.topology import load_topology
    fixed = resolve_documents(example_documents("allgather", "hierarchy", 4, total_size_bytes=64 << 10,
                                                slice_size_bytes=16 << 10))
    bundle = synthesize(fixed)
    index = tmp_path / "index.json"
    save_schedule(index, fixed, load_topology(fixed), bundle.xml, bundle.t_pred_us)
    auto = resolve_documents(example_documents("allgather", "hierarchy", 4, total_size_bytes=64 << 10,
                                               slice_size_bytes=None))
    found = find_schedules(index, auto, load_topology(auto), tolerance=0.01, limit=4)
    assert len(found) == 1 and found[0]["t_pred_us"] == bundle.t_pred_us
    other = resolve_documents(example_documents("allgather", "hierarchy", 4, total_size_bytes=64 << 10,
                                                slice_size_bytes=8 << 10))
    assert find_schedules(index, other, load_topology(other), tolerance=0.01, limit=4) == []
