"""Inventory coverage report (vericcl_b200/coverage.py) and the example catalog runner."""
import json
from pathlib import Path

from vericcl_b200.coverage import DEFAULT_REQUIREMENTS, coverage, main, render

ROOT = Path(__file__).resolve().parents[1]

JUNIT = """<?xml version="1.0"?>
<testsuites><testsuite name="pytest">
<testcase classname="tests.test_input" name="test_a" time="0.1"/>
<testcase classname="tests.test_input" name="test_b" time="0.1"><skipped message="x"/></testcase>
<testcase classname="tests.test_milp" name="test_c" time="0.2"><failure message="boom"/></testcase>
<testcase classname="tests.test_semantics" name="test_d" time="0.1"/>
</testsuite></testsuites>
"""


def test_every_inventory_row_is_mapped_to_existing_tests():
    reqs = json.loads(DEFAULT_REQUIREMENTS.read_text())
    inventory_rows = set()
    for row in reqs:
        for f in reqs[row]:
            assert (ROOT / f).exists(), (row, f)
        inventory_rows.add(row)
    # the K, M, N and P rows of the component inventory
    expected = {"P%d" % i for i in range(1, 37)} | {"P5L", "P20L", "P24L"} | {"N%d" % i for i in range(1, 13)} \
        | {"N1e"} | {"M%d" % i for i in range(1, 10)} | {"K%d" % i for i in range(1, 15)}
    assert inventory_rows == expected


def test_report_statuses(tmp_path):
    junit = tmp_path / "r.xml"
    junit.write_text(JUNIT)
    rep = coverage(junit)
    assert rep["P2"]["status"] == "passed_with_skips" and rep["P2"]["tests"] == 2
    assert rep["P15"]["status"] == "failed"
    assert rep["P4"]["status"] == "passed"
    assert rep["K9"]["status"] == "not_executed" and rep["K8"]["files"] == ["tests/test_gpu_single.py"]
    out = tmp_path / "c.md"
    assert main(["--junit", str(junit), "--out", str(out)]) == 0
    text = out.read_text()
    assert "| P15 | failed |" in text and "rows by status:" in text
    assert render(rep) == text


def test_example_catalog_runs_through_the_cli(tmp_path):
    from vericcl_b200.examples import example_cases, run_examples
    assert len(example_cases()) >= 9
    results = run_examples(tmp_path, "t", ["allreduce-p4", "alltoall-p4"])
    assert {n: r["exit_code"] for n, r in results.items()} == {"allreduce-p4": 0, "alltoall-p4": 0}
    assert all(r["t_pred_us"] > 0 and set(r["checks"].values()) <= {"valid", "not_run"} for r in results.values())
    index = tmp_path / "examples" / "examples" / "output" / "t-index"
    assert json.loads((index / "examples.json").read_text()).keys() == results.keys()
