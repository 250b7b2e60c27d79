"""Experiment matrix stages: plan, solve, benchmark, summarize, resume (vericcl_b200/experiment_matrix.py)."""
import json

from vericcl_b200.experiment_matrix import (benchmark_matrix, main, parse_size, plan_matrix, solve_matrix,
                                            summarize)


def test_matrix_stages_and_resume(tmp_path):
    assert parse_size("4m") == 4 << 20 and parse_size("1g") == 1 << 30 and parse_size("512") == 512
    exp = tmp_path / "exp"
    manifest = plan_matrix(exp, groups=(1, 2), per_group=2, colls=("allgather", "allreduce"), sizes=(64 << 10,))
    assert len(manifest["cases"]) == 4
    path = exp / "manifest.json"
    first = solve_matrix(path)
    assert all(r["status"] == "passed" and r["t_pred_us"] > 0 for r in first)
    again = solve_matrix(path, resume=True)
    assert [r["run"] for r in again] == [r["run"] for r in first]          # reused, not re-solved
    # a changed input invalidates its record
    case = manifest["cases"][0]
    sk = exp / case["documents"] / "sketch.json"
    doc = json.loads(sk.read_text())
    doc["hyperparameters"]["slice_size_bytes"] //= 2
    sk.write_text(json.dumps(doc))
    third = solve_matrix(path, resume=True)
    assert third[0]["run"] != first[0]["run"] and [r["run"] for r in third[1:]] == [r["run"] for r in first[1:]]

    seen = []

    def fake_measure(xml, request):
        import os
        seen.append(os.environ.get("VERICCL_EMULATE"))
        return 10.0
    bench = benchmark_matrix(path, measure=fake_measure)
    assert all(r["status"] == "passed" and r["measured_us"] == 10.0 for r in bench)
    assert seen.count("group=2,gbps=25") == 2 and seen.count(None) == 2
    assert benchmark_matrix(path, measure=lambda x, r: 1 / 0, resume=True) == bench   # all reused
    rows = summarize(path)
    assert all(r["solve"] == "passed" and r["benchmark"] == "passed" for r in rows)
    assert all(r["measured_over_predicted"] > 0 for r in rows)
    assert main(["summarize", "--manifest", str(path), "--markdown"]) == 0


def test_failed_measurement_is_recorded(tmp_path):
    exp = tmp_path / "exp"
    plan_matrix(exp, groups=(1,), per_group=2, colls=("allreduce",), sizes=(64 << 10,))
    path = exp / "manifest.json"
    solve_matrix(path)

    def broken(xml, request):
        raise RuntimeError("no GPU")
    (rec,) = benchmark_matrix(path, measure=broken)
    assert rec["status"] == "failed" and "no GPU" in rec["error"]
    assert summarize(path)[0]["benchmark"] == "failed"
