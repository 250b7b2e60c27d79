"""Task-level significance budget as a hash-chained, file-locked JSONL ledger.

Every measured comparison draws its significance level from the task's total
``task_alpha`` (≤ 0.05): attempt k gets ``min(cap, remaining / 2)`` so the
total never exceeds the budget however many comparisons run.  Entries are
appended under ``flock`` and each carries the sha256 of the previous entry,
so tampering or truncation is detectable (reference:
vericcl/verification/online/statistical_ledger.py:44-80).
"""
from __future__ import annotations

import fcntl
import hashlib
import json
from pathlib import Path


class StatisticalLedger:
    def __init__(self, path, *, task_alpha: float = 0.05, single_cap: float = 0.05):
        if not 0 < task_alpha <= 0.05 or not 0 < single_cap <= 0.05:
            raise ValueError("alpha budgets must be in (0, 0.05]")
        self.path = Path(path)
        self.path.parent.mkdir(parents=True, exist_ok=True)
        self.task_alpha = task_alpha
        self.single_cap = single_cap

    def entries(self):
        if not self.path.exists():
            return []
        return [json.loads(line) for line in self.path.read_text().splitlines() if line.strip()]

    def verify(self) -> bool:
        prev = "0" * 64
        for entry in self.entries():
            if entry["prev"] != prev:
                return False
            body = json.dumps({k: v for k, v in entry.items() if k != "hash"}, sort_keys=True)
            if hashlib.sha256(body.encode()).hexdigest() != entry["hash"]:
                return False
            prev = entry["hash"]
        return True

    def spent(self) -> float:
        return sum(e["alpha"] for e in self.entries())

    def allocate(self, attempt_id: str) -> float:
        with open(str(self.path) + ".lock", "a+") as lock:
            fcntl.flock(lock.fileno(), fcntl.LOCK_EX)
            try:
                entries = self.entries()
                remaining = self.task_alpha - sum(e["alpha"] for e in entries)
                alpha = max(0.0, min(self.single_cap, remaining / 2.0))
                prev = entries[-1]["hash"] if entries else "0" * 64
                entry = {"attempt": attempt_id, "alpha": alpha, "prev": prev, "index": len(entries)}
                entry["hash"] = hashlib.sha256(json.dumps(entry, sort_keys=True).encode()).hexdigest()
                with self.path.open("a") as handle:
                    handle.write(json.dumps(entry, sort_keys=True) + "\n")
                return alpha
            finally:
                fcntl.flock(lock.fileno(), fcntl.LOCK_UN)
