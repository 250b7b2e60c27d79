"""Pipeline wall-clock attribution and schedule replay timing (vericcl_b200/overhead.py)."""
import json

import pytest

from vericcl_b200.examples import example_documents, write_documents
from vericcl_b200.experiments import main
from vericcl_b200.overhead import PHASES, PhaseTimer, instrument


def test_phase_timer_nests_and_restores():
    ticks = iter(range(0, 1000, 10))
    timer = PhaseTimer(clock=lambda: next(ticks))
    with timer.span("outer"):
        with timer.span("inner"):
            pass
    assert [(s["name"], s["depth"]) for s in timer.spans] == [("inner", 1), ("outer", 0)]
    assert timer.totals() == {"inner": 10, "outer": 30} and timer.top_level_ns() == 30
    with pytest.raises(ValueError):
        with timer.span("bad"):
            raise ValueError()
    assert timer.spans[-1]["error"] == "ValueError"
    import vericcl_b200.synthesis as synthesis
    before = synthesis.build_demands
    with instrument(PhaseTimer()):
        assert synthesis.build_demands is not before
    assert synthesis.build_demands is before


def test_solve_and_replay_attribution(tmp_path):
    write_documents(tmp_path / "in", example_documents("allreduce", "hierarchy", 4, total_size_bytes=64 << 10,
                                                       slice_size_bytes=16 << 10))
    out = tmp_path / "solve.json"
    assert main(["overhead", "solve", "--inputs", str(tmp_path / "in"), "--repeats", "2", "--out", str(out)]) == 0
    doc = json.loads(out.read_text())
    assert doc["outcome"]["can_execute"] and len(doc["runs"]) == 2
    phases = doc["summary"]["median_ms"]
    for name in ("plan", "demands", "route_milp", "storage", "lowering", "prediction", "checks"):
        assert phases[name] > 0, name
    run = doc["runs"][0]
    assert sum(t for n, t in run["totals_ns"].items() if n in {p for _, _, p in PHASES}) > 0
    assert 0 <= run["unattributed_ns"] <= run["total_ns"]
    # replay the schedule of a CLI solve
    from vericcl_b200.cli.main import main as cli
    args = ["--project-root", str(tmp_path), "--case", "o", "--run-id", "s"]
    for k in ("topology", "sketch", "atom", "runtime"):
        args += ["--" + k, str(tmp_path / "in" / (k + ".json"))]
    assert cli(["solve"] + args) == 0
    run_dir = tmp_path / "examples" / "o" / "output" / "s"
    rep = tmp_path / "replay.json"
    assert main(["overhead", "replay", "--inputs", str(tmp_path / "in"), "--xml", str(run_dir / "schedule.xml"),
                 "--sidecar", str(run_dir / "schedule.json"), "--repeats", "2", "--out", str(rep)]) == 0
    r = json.loads(rep.read_text())
    assert r["outcome"]["can_execute"] and r["summary"]["median_ms"]["checks"] > 0
    assert "route_milp" not in r["summary"]["median_ms"]          # replay re-checks; it does not re-solve
