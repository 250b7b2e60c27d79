"""Recommended input changes for rejected schedules and empty parameter domains."""
import json

import pytest

from vericcl_b200.cli.main import main
from vericcl_b200.errors import InputValidationError, ScratchBudgetError
from vericcl_b200.examples import example_documents, write_documents
from vericcl_b200.input.loader import resolve_documents
from vericcl_b200.program.recommendations import merge, recommend_for_domain, recommend_for_program
from vericcl_b200.synthesis import synthesize


def _docs(op, steps_per_tb=None, **kw):
    d = example_documents(op, "hierarchy", 4, **kw)
    if steps_per_tb:
        d["runtime"]["limits"] = {"steps_per_tb": steps_per_tb}
    return d


def test_step_limit_recommends_channels_and_a_larger_slice():
    d = _docs("allgather", 8, total_size_bytes=16 * 1024, slice_size_bytes=1024)
    bundle = synthesize(resolve_documents(d))
    assert bundle.checks["launch"]["status"] == "invalid"
    recs = recommend_for_program(bundle.program, bundle.request, bundle.checks)
    kinds = {r["kind"]: r for r in recs}
    assert kinds["increase_channels"]["parameters"] == {"max_channels": 2}
    assert kinds["increase_slice_size"]["parameters"] == {"slice_size_bytes": 2048}
    assert all(r["requires_resolve"] and r["reason_codes"] == ["steps_per_tb"] for r in recs)
    # both changes, applied, give a schedule that passes every check
    assert synthesize(resolve_documents(d), channels=2).can_execute
    d["sketch"]["hyperparameters"]["slice_size_bytes"] = 2048
    assert synthesize(resolve_documents(d)).can_execute


def test_valid_program_needs_nothing():
    bundle = synthesize(resolve_documents(_docs("allreduce", total_size_bytes=16 * 1024, slice_size_bytes=1024)))
    assert bundle.can_execute and recommend_for_program(bundle.program, bundle.request, bundle.checks) == []


def test_scratch_failure_reports_the_smallest_budget_that_fits():
    d = _docs("allreduce", total_size_bytes=16 * 1024, slice_size_bytes=1024, scratch_bytes=1024)
    with pytest.raises(ScratchBudgetError) as info:
        synthesize(resolve_documents(d))
    need = info.value.needed_bytes
    assert need > 1024 and need % 1024 == 0
    d["runtime"]["scratch_bytes_per_rank"] = need
    assert synthesize(resolve_documents(d)).can_execute
    d["runtime"]["scratch_bytes_per_rank"] = need - 1024
    with pytest.raises(ScratchBudgetError):
        synthesize(resolve_documents(d))


def test_empty_domain_recommendations():
    d = _docs("allreduce", 8, total_size_bytes=16 * 1024, slice_size_bytes=1024)
    recs = {r["kind"]: r["parameters"] for r in recommend_for_domain(resolve_documents(d))}
    # N = 16 slices need 2N / C <= 8 steps per TB: four channels, or 4 KiB slices on the one allowed
    assert recs == {"increase_channels": {"max_channels": 4}, "use_slice_size": {"slice_size_bytes": 4096}}
    d = _docs("allreduce", 8, total_size_bytes=1 << 20, slice_size_bytes=None, scratch_bytes=8)
    recs = recommend_for_domain(resolve_documents(d))
    assert [(r["kind"], r["parameters"]) for r in recs] == [
        ("increase_scratch_budget", {"scratch_bytes_per_rank": 1 << 18})]
    assert recs[0]["requires_resolve"] is False


def test_merge_keeps_the_most_demanding_parameters():
    a = [{"kind": "increase_channels", "priority": 2, "parameters": {"max_channels": 2}, "reason_codes": ["x"],
          "requires_resolve": True}]
    b = [{"kind": "increase_channels", "priority": 2, "parameters": {"max_channels": 3}, "reason_codes": ["y"],
          "requires_resolve": True}]
    (got,) = merge([a, b])
    assert got["parameters"] == {"max_channels": 3} and got["reason_codes"] == ["x", "y"]


def _args(indir, project, run_id):
    return ["--project-root", str(project), "--case", "r", "--run-id", run_id,
            "--topology", str(indir / "topology.json"), "--sketch", str(indir / "sketch.json"),
            "--atom", str(indir / "atom.json"), "--runtime", str(indir / "runtime.json")]


def test_solve_reports_recommendations(tmp_path):
    d = _docs("allgather", 8, total_size_bytes=16 * 1024, slice_size_bytes=1024, calibration=False)
    write_documents(tmp_path / "in", d)
    main(["solve"] + _args(tmp_path / "in", tmp_path, "rec"))
    run = tmp_path / "examples" / "r" / "output" / "rec"
    report = (run / "report.md").read_text()
    assert "## Recommended input changes" in report and "increase_channels" in report
    meta = json.loads((run / "run.json").read_text())
    assert meta["best"] is None


def test_solve_with_empty_domain_names_the_fix(tmp_path):
    d = _docs("allreduce", 8, total_size_bytes=1 << 20, slice_size_bytes=None, scratch_bytes=8, calibration=False)
    req = resolve_documents(d)
    from vericcl_b200.planner.parameters import initial_parameter_domain
    with pytest.raises(InputValidationError):
        initial_parameter_domain(req)
    write_documents(tmp_path / "in", d)
    assert main(["solve"] + _args(tmp_path / "in", tmp_path, "dom")) == 2
