"""Run context: case/run directory layout, input snapshot, run.json, events.

Layout (reference README "Results and troubleshooting" and
vericcl/artifacts/layout.py:23):

    <project>/examples/<case>/output/<run_id>/
        run.json  report.md  run.log  schedule.xml  schedule.json  model.json
        checkpoint.json  trace.json  details.zip
        process/{input_snapshot,models,candidates,jobs,checkpoints,statistics,live,reports,best,tmp}/
        process/events.jsonl
"""
from __future__ import annotations

import shutil
import sys
import time
import uuid
from dataclasses import dataclass, field
from datetime import datetime, timezone
from pathlib import Path

from vericcl_b200.execution.events import EventLog
from vericcl_b200.utils.jsonio import atomic_write_json, strict_load

PROCESS_DIRS = ("input_snapshot", "models", "candidates", "jobs", "checkpoints", "statistics", "live", "reports",
                "best", "tmp", "rebuildable-cache")


def new_run_id(prefix: str = "run") -> str:
    return "%s-%s-%s" % (prefix, datetime.now(timezone.utc).strftime("%Y%m%dT%H%M%S"), uuid.uuid4().hex[:6])


@dataclass
class RunContext:
    project_root: Path
    case: str
    run_id: str
    command: str
    directory: Path
    events: EventLog
    started_monotonic: float = field(default_factory=time.monotonic)

    @property
    def process(self) -> Path:
        return self.directory / "process"

    @classmethod
    def create(cls, project_root, case: str, command: str, *, run_id: str | None = None, input_files=None,
               extra_inputs=None):
        project_root = Path(project_root).resolve()
        run_id = run_id or new_run_id(command)
        directory = project_root / "examples" / case / "output" / run_id
        if directory.exists():
            raise FileExistsError("run directory already exists: %s (use a new --run-id)" % directory)
        for name in PROCESS_DIRS:
            (directory / "process" / name).mkdir(parents=True, exist_ok=True)
        events = EventLog(directory / "process")
        ctx = cls(project_root, case, run_id, command, directory, events)
        snapshot = {}
        for name, path in dict(input_files or {}, **(extra_inputs or {})).items():
            if path is None:
                continue
            target = ctx.process / "input_snapshot" / (name + Path(path).suffix)
            shutil.copyfile(path, target)
            snapshot[name] = {"source": str(Path(path).resolve()), "copy": str(target.relative_to(directory))}
        ctx.write_run_json({"run_id": run_id, "case": case, "command": command, "status": "running",
                            "invocation": sys.argv, "input_snapshot": snapshot,
                            "started_utc": datetime.now(timezone.utc).isoformat(), "best": None, "result": None})
        events.emit("run_started", run_id=run_id, command=command)
        return ctx

    @classmethod
    def open(cls, directory):
        directory = Path(directory).resolve()
        meta = strict_load(directory / "run.json")
        case_dir = directory.parent.parent
        ctx = cls(case_dir.parent.parent, meta["case"], meta["run_id"], meta["command"], directory,
                  EventLog(directory / "process"))
        return ctx

    def read_run_json(self) -> dict:
        path = self.directory / "run.json"
        return strict_load(path) if path.exists() else {}

    def write_run_json(self, doc: dict) -> None:
        atomic_write_json(self.directory / "run.json", doc)

    def update_run_json(self, **fields) -> dict:
        doc = self.read_run_json()
        doc.update(fields)
        self.write_run_json(doc)
        return doc

    def emit(self, kind: str, **payload):
        return self.events.emit(kind, **payload)

    def elapsed_s(self) -> float:
        return time.monotonic() - self.started_monotonic


def finalize_run(ctx: RunContext, result: dict) -> dict:
    doc = ctx.update_run_json(status="finished", result=result,
                              finished_utc=datetime.now(timezone.utc).isoformat())
    ctx.emit("run_finished", **{k: v for k, v in result.items() if k != "timing"})
    return doc
