"""Durable GPU ownership registry keyed by GPU UUID.

A run acquires the GPUs it launches on (``active``), releases them with a
receipt after the job's processes are gone (``released``), or quarantines them
when release cannot be confirmed (``quarantined``).  New jobs refuse GPUs that
are active or quarantined under another owner; resume refuses unresolved
ownership (reference: vericcl/execution/ownership.py:10-74).  The registry is a
JSON file updated under an exclusive ``flock``.
"""
from __future__ import annotations

import fcntl
import json
import os
import time
from contextlib import contextmanager
from pathlib import Path

from vericcl_b200.errors import RuntimeFailure


class GPUOwnershipRegistry:
    def __init__(self, path):
        self.path = Path(path)
        self.path.parent.mkdir(parents=True, exist_ok=True)

    @contextmanager
    def _locked(self):
        with open(str(self.path) + ".lock", "a+") as lock:
            fcntl.flock(lock.fileno(), fcntl.LOCK_EX)
            try:
                data = json.loads(self.path.read_text()) if self.path.exists() else {}
                yield data
                tmp = str(self.path) + ".tmp"
                with open(tmp, "w") as handle:
                    json.dump(data, handle, indent=2, sort_keys=True)
                    handle.flush()
                    os.fsync(handle.fileno())
                os.replace(tmp, self.path)
            finally:
                fcntl.flock(lock.fileno(), fcntl.LOCK_UN)

    def acquire(self, uuids, owner: str) -> None:
        with self._locked() as data:
            for uuid in uuids:
                entry = data.get(uuid)
                if entry and entry["state"] in ("active", "quarantined") and entry["owner"] != owner:
                    raise RuntimeFailure("GPU %s is %s by %s" % (uuid, entry["state"], entry["owner"]))
            for uuid in uuids:
                data[uuid] = {"state": "active", "owner": owner, "since": time.time()}

    def release(self, uuids, owner: str, receipt: dict | None = None) -> None:
        with self._locked() as data:
            for uuid in uuids:
                entry = data.get(uuid)
                if entry and entry["owner"] == owner:
                    data[uuid] = {"state": "released", "owner": owner, "since": time.time(), "receipt": receipt or {}}

    def quarantine(self, uuids, owner: str, reason: str) -> None:
        with self._locked() as data:
            for uuid in uuids:
                data[uuid] = {"state": "quarantined", "owner": owner, "since": time.time(), "reason": reason}

    def state(self, uuid: str):
        data = json.loads(self.path.read_text()) if self.path.exists() else {}
        return data.get(uuid)

    def unresolved(self, owner: str):
        data = json.loads(self.path.read_text()) if self.path.exists() else {}
        return sorted(u for u, e in data.items() if e["owner"] == owner and e["state"] != "released")


def local_gpu_uuids(count: int | None = None):
    """UUIDs of local GPUs via NVML (read-only); synthetic ids without NVML."""
    try:
        import pynvml
        pynvml.nvmlInit()
        try:
            n = pynvml.nvmlDeviceGetCount() if count is None else count
            return [pynvml.nvmlDeviceGetUUID(pynvml.nvmlDeviceGetHandleByIndex(i)) for i in range(n)]
        finally:
            pynvml.nvmlShutdown()
    except Exception:
        return ["GPU-local-%d" % i for i in range(count or 0)]
