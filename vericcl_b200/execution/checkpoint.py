"""Content-addressed checkpoints and resume.

A checkpoint is an immutable JSON document under
``process/checkpoints/<sha256>.json`` holding the phase, input references,
model reference, best candidate record, budget snapshot, search cursor and
extra state, with per-file sha256 of every referenced artifact and
monotonic / wall / boot-id stamps.  ``latest.json`` points at the newest one
with its checksum.  Restore verifies every checksum, the event log's
sequence, and unresolved GPU ownership, and reports the downtime to charge
to the budgets (reference: vericcl/workflow_state.py:68-204).
"""
from __future__ import annotations

import hashlib
import time
from datetime import datetime, timezone

from vericcl_b200.errors import RuntimeFailure
from vericcl_b200.execution.events import verify_sequence
from vericcl_b200.execution.processes import boot_id
from vericcl_b200.utils.hashing import digest
from vericcl_b200.utils.jsonio import atomic_write_json, canonical_dumps, strict_load

SCHEMA_VERSION = 5


def file_sha256(path) -> str:
    h = hashlib.sha256()
    with open(path, "rb") as handle:
        for block in iter(lambda: handle.read(1 << 20), b""):
            h.update(block)
    return h.hexdigest()


def save_checkpoint(ctx, *, phase: str, state: dict, files=(), budgets: dict | None = None) -> str:
    checksums = {}
    for rel in files:
        path = ctx.directory / rel
        if path.exists():
            checksums[str(rel)] = file_sha256(path)
    doc = {"schema_version": SCHEMA_VERSION, "phase": phase, "state": state, "files": checksums,
           "budgets": budgets or {}, "event_sequence": ctx.events.sequence,
           "stamps": {"monotonic": time.monotonic(), "wall_utc": datetime.now(timezone.utc).isoformat(),
                      "wall_epoch": time.time(), "boot_id": boot_id()}}
    key = digest(doc)
    path = ctx.process / "checkpoints" / (key + ".json")
    if not path.exists():
        atomic_write_json(path, doc, mode=0o444)
    text = canonical_dumps(doc)
    atomic_write_json(ctx.process / "checkpoints" / "latest.json",
                      {"checkpoint": path.name, "sha256": hashlib.sha256(text.encode()).hexdigest()})
    atomic_write_json(ctx.directory / "checkpoint.json", {"phase": phase, "checkpoint": path.name,
                                                          "elapsed_s": (budgets or {}).get("elapsed_s")})
    ctx.emit("checkpoint_saved", phase=phase, checkpoint=path.name)
    return path.name


def restore_checkpoint(ctx, *, registry=None, owner: str | None = None) -> dict:
    latest = ctx.process / "checkpoints" / "latest.json"
    if not latest.exists():
        raise RuntimeFailure("no checkpoint to resume from")
    pointer = strict_load(latest)
    doc = strict_load(ctx.process / "checkpoints" / pointer["checkpoint"])
    if hashlib.sha256(canonical_dumps(doc).encode()).hexdigest() != pointer["sha256"]:
        raise RuntimeFailure("checkpoint checksum mismatch")
    if doc.get("schema_version") != SCHEMA_VERSION:
        raise RuntimeFailure("unsupported checkpoint schema")
    for rel, want in doc["files"].items():
        path = ctx.directory / rel
        if not path.exists() or file_sha256(path) != want:
            raise RuntimeFailure("checkpointed file changed or vanished: " + rel)
    records = ctx.events.read()
    if not verify_sequence(records):
        raise RuntimeFailure("event log sequence is not strictly increasing")
    if registry is not None and owner is not None:
        pending = registry.unresolved(owner)
        if pending:
            raise RuntimeFailure("GPU ownership from the interrupted run is unresolved: %s" % pending)
    stamps = doc["stamps"]
    downtime = max(0.0, time.time() - stamps["wall_epoch"]) if stamps.get("boot_id") else 0.0
    doc["downtime_s"] = downtime
    ctx.emit("checkpoint_restored", checkpoint=pointer["checkpoint"], downtime_s=downtime)
    return doc
