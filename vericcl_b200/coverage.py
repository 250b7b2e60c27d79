"""Map test results to inventory requirements.

    python -m pytest tests -q --junitxml results.xml
    python -m vericcl_b200.coverage --junit results.xml --out coverage.md

``tests/requirements.json`` maps each inventory row (P1 … K14) to the test
files that exercise it.  The report gives every row the outcome of its
tests in that JUnit file: ``passed``, ``passed_with_skips``, ``failed``,
``skipped`` or ``not_executed`` (its tests did not run, e.g. GPU tests on a
CPU machine, or it lists none).  Passing mapped tests shows the row is
exercised, not that it is complete (reference: tools/coverage_report.py).
"""
from __future__ import annotations

import argparse
import json
import sys
import xml.etree.ElementTree as ET
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
DEFAULT_REQUIREMENTS = ROOT / "tests" / "requirements.json"


def read_junit(path) -> list:
    """Test cases of a JUnit XML file: id, file, status, time."""
    out = []
    for case in ET.parse(path).iter("testcase"):
        status = "passed"
        for tag, kind in (("failure", "failed"), ("error", "error"), ("skipped", "skipped")):
            if case.find(tag) is not None:
                status = kind
                break
        classname = case.get("classname", "")
        out.append({"id": classname + "::" + case.get("name", ""),
                    "file": classname.replace(".", "/") + ".py", "status": status,
                    "time_s": float(case.get("time", 0) or 0)})
    return out


def summarize(tests: list, files: list) -> dict:
    chosen = [t for t in tests if t["file"] in files]
    counts = {k: sum(t["status"] == k for t in chosen) for k in ("passed", "failed", "error", "skipped")}
    if not chosen:
        status = "not_executed"
    elif counts["failed"] or counts["error"]:
        status = "failed"
    elif counts["skipped"]:
        status = "passed_with_skips" if counts["passed"] else "skipped"
    else:
        status = "passed"
    return {"status": status, "counts": counts, "tests": len(chosen)}


def coverage(junit, requirements=DEFAULT_REQUIREMENTS) -> dict:
    reqs = json.loads(Path(requirements).read_text())
    tests = read_junit(junit)
    return {row: dict(summarize(tests, files), files=files) for row, files in reqs.items()}


def render(report: dict) -> str:
    lines = ["| row | status | tests | passed | failed | skipped | files |", "|---|---|---|---|---|---|---|"]
    for row, r in report.items():
        c = r["counts"]
        lines.append("| %s | %s | %d | %d | %d | %d | %s |" % (
            row, r["status"], r["tests"], c["passed"], c["failed"] + c["error"], c["skipped"],
            ", ".join(Path(f).name for f in r["files"]) or "—"))
    totals = {}
    for r in report.values():
        totals[r["status"]] = totals.get(r["status"], 0) + 1
    lines += ["", "rows by status: " + ", ".join("%s %d" % kv for kv in sorted(totals.items()))]
    return "\n".join(lines) + "\n"


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="vericcl_b200.coverage")
    ap.add_argument("--junit", required=True)
    ap.add_argument("--requirements", default=str(DEFAULT_REQUIREMENTS))
    ap.add_argument("--out")
    args = ap.parse_args(argv)
    text = render(coverage(args.junit, args.requirements))
    if args.out:
        Path(args.out).write_text(text)
    else:
        sys.stdout.write(text)
    return 0


if __name__ == "__main__":
    sys.exit(main())
