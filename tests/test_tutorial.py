"""Repair tutorial (vericcl_b200/tutorial.py): repair, history reuse, resynthesis."""
import json

from vericcl_b200.input.loader import resolve_documents
from vericcl_b200.performance.initial import initial_cost_model
from vericcl_b200.topology import load_topology
from vericcl_b200.tutorial import SLOW_BETA, direct_broadcast, main, tutorial_documents
from vericcl_b200.verification.bottlenecks import analyze
from vericcl_b200.synthesis import Lowerer


def test_slow_direct_link_yields_a_relay_strategy():
    req = resolve_documents(tutorial_documents())
    model = initial_cost_model(req)
    bundle = Lowerer(req, load_topology(req), model)(direct_broadcast(req))
    analysis = analyze(bundle, model, batch_size=8)
    relays = [c.detail.get("relay") for c in analysis.causes if c.kind == "critical_service"]
    assert relays and set(relays) == {2}
    assert any(s.family == "path" and dict(s.parameters).get("via") == 2 for s in analysis.strategies)


def test_tutorial_run(tmp_path, capsys):
    assert main(["--project-root", str(tmp_path), "--run-id", "t"]) == 0
    run = tmp_path / "examples" / "repair-tutorial" / "output" / "t"
    steps = json.loads((run / "tutorial.json").read_text())
    direct = steps["direct"]["t_pred_us"]
    # four 1 KiB slices over the slow link dominate the direct schedule
    assert direct >= 4 * 1024 * SLOW_BETA
    assert steps["repair"]["improved"] and steps["repair"]["t_pred_us"] < direct / 3
    assert [0, 1] not in steps["repair"]["routes"] and [2, 1] in steps["repair"]["routes"]
    assert steps["history"]["found"] == 1
    assert steps["resynthesis"]["best_t_pred_us"] <= steps["repair"]["t_pred_us"]
    assert (run / "schedule.xml").exists() and (run / "process" / "repaired.xml").exists()
    meta = json.loads((run / "run.json").read_text())
    assert meta["status"] == "finished"
