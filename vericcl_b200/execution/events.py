"""Structured event log: fsync'd ``events.jsonl`` plus a human ``run.log``.

Each event carries schema version, a strictly increasing sequence number,
UTC time, monotonic nanoseconds, node, rank and kind; payloads are redacted
before they are written (reference: vericcl/execution/events.py:34-64).
"""
from __future__ import annotations

import json
import os
import socket
import threading
import time
from datetime import datetime, timezone
from pathlib import Path

from vericcl_b200.execution.security import Redactor

SCHEMA_VERSION = 1


class EventLog:
    def __init__(self, directory, *, rank: int = 0, redactor: Redactor | None = None):
        self.directory = Path(directory)
        self.directory.mkdir(parents=True, exist_ok=True)
        self.path = self.directory / "events.jsonl"
        self.log_path = self.directory / "run.log"
        self.rank = rank
        self.node = socket.gethostname()
        self.redactor = redactor or Redactor()
        self._lock = threading.Lock()
        self.sequence = self._last_sequence()

    def _last_sequence(self) -> int:
        if not self.path.exists():
            return 0
        last = 0
        valid = []
        with self.path.open() as handle:
            for line in handle:
                try:
                    record = json.loads(line)
                except json.JSONDecodeError:
                    break   # truncated tail (crash while writing): repaired below
                if record.get("sequence", 0) <= last:
                    break
                last = record["sequence"]
                valid.append(line if line.endswith("\n") else line + "\n")
        with self.path.open("w") as handle:
            handle.writelines(valid)
            handle.flush()
            os.fsync(handle.fileno())
        return last

    def emit(self, kind: str, **payload) -> dict:
        with self._lock:
            self.sequence += 1
            record = {"schema_version": SCHEMA_VERSION, "sequence": self.sequence,
                      "utc": datetime.now(timezone.utc).isoformat(), "monotonic_ns": time.monotonic_ns(),
                      "node": self.node, "rank": self.rank, "kind": kind,
                      "payload": self.redactor.redact(payload)}
            line = json.dumps(record, sort_keys=True, default=str)
            with self.path.open("a") as handle:
                handle.write(line + "\n")
                handle.flush()
                os.fsync(handle.fileno())
            with self.log_path.open("a") as handle:
                handle.write("%s [%s] %s %s\n" % (record["utc"], self.sequence, kind,
                                                  json.dumps(record["payload"], default=str)[:400]))
            return record

    def read(self):
        if not self.path.exists():
            return []
        return [json.loads(line) for line in self.path.read_text().splitlines() if line.strip()]


def verify_sequence(records) -> bool:
    last = 0
    for record in records:
        if record["sequence"] <= last:
            return False
        last = record["sequence"]
    return True
