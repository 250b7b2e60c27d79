"""Final publication of a run's results.

Writes ``schedule.xml``, ``schedule.json`` (the sidecar), ``model.json``,
``report.md`` and ``details.zip`` (an archive copy of ``process/``), and
updates ``run.json`` with the file index (reference:
vericcl/execution/publication.py:51).
"""
from __future__ import annotations

import zipfile
from pathlib import Path

from vericcl_b200.utils.jsonio import atomic_write_json, atomic_write_text


def write_report(ctx, result: dict, best: dict | None) -> Path:
    lines = ["# Run %s" % ctx.run_id, "", "* command: `%s`" % ctx.command,
             "* status: %s" % result.get("status"), "* stop reason: %s" % result.get("stop_reason")]
    if best:
        lines += ["* T_pred: %.3f us (model %s)" % (best["t_pred_us"], best.get("model_version")),
                  "* origin: %s" % best.get("origin")]
        checks = best.get("checks", {})
        if checks:
            lines += ["", "## Checks", "", "| check | status | detail |", "|---|---|---|"]
            for key, value in sorted(checks.items()):
                detail = str(value.get("detail", ""))[:120].replace("|", "/")
                lines.append("| %s | %s | %s |" % (key, value.get("status"), detail))
    recs = result.get("recommendations") or []
    if recs:
        lines += ["", "## Recommended input changes", "", "| change | parameters | reasons | re-solve |",
                  "|---|---|---|---|"]
        for r in recs:
            params = ", ".join("%s=%s" % kv for kv in sorted(r["parameters"].items()))
            lines.append("| %s | %s | %s | %s |" % (r["kind"], params, ", ".join(r["reason_codes"]),
                                                   "yes" if r["requires_resolve"] else "no"))
    for key in ("rounds", "proof", "measured", "issues"):
        if result.get(key):
            lines += ["", "## %s" % key.capitalize(), "", "```", str(result[key])[:4000], "```"]
    return atomic_write_text(ctx.directory / "report.md", "\n".join(lines) + "\n")


def publish_results(ctx, *, xml: str | None, sidecar: dict | None, model: dict | None, result: dict,
                    best: dict | None) -> dict:
    artifacts = []
    if xml is not None:
        atomic_write_text(ctx.directory / "schedule.xml", xml)
        artifacts.append("schedule.xml")
    if sidecar is not None:
        atomic_write_json(ctx.directory / "schedule.json", sidecar)
        artifacts.append("schedule.json")
    if model is not None:
        atomic_write_json(ctx.directory / "model.json", model)
        artifacts.append("model.json")
    write_report(ctx, result, best)
    artifacts.append("report.md")
    archive = ctx.directory / "details.zip"
    with zipfile.ZipFile(str(archive) + ".tmp", "w", zipfile.ZIP_DEFLATED) as z:
        for path in sorted(ctx.process.rglob("*")):
            if path.is_file():
                z.write(path, path.relative_to(ctx.directory))
    Path(str(archive) + ".tmp").replace(archive)
    artifacts.append("details.zip")
    from vericcl_b200.execution.transport import export_manifest
    export_manifest(ctx.directory)
    artifacts.append("manifest.json")
    ctx.update_run_json(artifacts=artifacts)
    ctx.emit("results_published", artifacts=artifacts)
    return {"artifacts": artifacts}
