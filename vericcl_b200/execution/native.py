"""Launch the native C-API driver (``vericcl-native``) for every rank and combine receipts.

Each rank runs as an owned process (own process group, deadline, TERM/KILL)
with a JSON configuration naming the schedule XML, the control address and
the workload; ranks agree through the native TCP control plane, not MPI.
Per invocation the slowest rank's device time counts, and the invocations
are averaged (reference: vericcl/execution/native.py:28-259 and
runtime/execution/driver.cc:26-150).
"""
from __future__ import annotations

import json
import os
import secrets
import statistics
import subprocess
import tempfile
import time
from pathlib import Path

from vericcl_b200.errors import RuntimeFailure
from vericcl_b200.execution.processes import ProcessIdentity, boot_id, start_time, terminate_group


def combine_schedule_results(receipts):
    """Max over ranks per invocation, then the mean over invocations (µs)."""
    times = [r["device_times_us"] for r in receipts]
    if not times or any(len(t) != len(times[0]) for t in times):
        raise RuntimeFailure("ranks reported different invocation counts")
    per_invocation = [max(ts) for ts in zip(*times)]
    return {"mean_us": statistics.fmean(per_invocation), "per_invocation_us": per_invocation,
            "bad": sum(r["bad"] for r in receipts)}


class NativeScheduleDriver:
    def __init__(self, xml: str, nranks: int, *, devices=None, binary=None, port: int | None = None):
        from vericcl_b200.ops.build import build_driver
        self.xml = xml
        self.nranks = nranks
        self.devices = list(devices) if devices is not None else list(range(nranks))
        self.binary = Path(binary) if binary else build_driver()
        self.port = port or (20000 + secrets.randbelow(20000))

    def measure(self, *, count: int, dtype: int = 0, redop: int = 0, scale: float = 1.0, nlanes: int = 32,
                niters: int = 1, warmup: int = 3, iters: int = 10, timeout_s: float = 60.0, trace_dir=None):
        """Device-timed invocations; with ``trace_dir`` every rank also writes
        ``trace-rank<r>.bin`` (per-step trace of its last invocation)."""
        with tempfile.TemporaryDirectory() as tmp:
            tmp = Path(tmp)
            (tmp / "schedule.xml").write_text(self.xml)
            session = secrets.token_hex(4)
            procs = []
            for rank in range(self.nranks):
                cfg = {"xml": str(tmp / "schedule.xml"), "rank": rank, "nranks": self.nranks,
                       "device": self.devices[rank], "control_address": "127.0.0.1", "control_port": self.port,
                       "session": session, "count": count, "dtype": dtype, "redop": redop, "scale": scale,
                       "nlanes": nlanes, "niters": niters, "warmup": warmup, "iters": iters,
                       "timeout_s": timeout_s, "receipt": str(tmp / ("receipt-%d.json" % rank))}
                if trace_dir is not None:
                    Path(trace_dir).mkdir(parents=True, exist_ok=True)
                    cfg["trace"] = str(Path(trace_dir) / ("trace-rank%d.bin" % rank))
                path = tmp / ("config-%d.json" % rank)
                path.write_text(json.dumps(cfg))
                p = subprocess.Popen([str(self.binary), str(path)], stdout=subprocess.PIPE, stderr=subprocess.PIPE,
                                     text=True, start_new_session=True)
                procs.append((p, ProcessIdentity(p.pid, os.getpgid(p.pid), start_time(p.pid), boot_id())))
            deadline = time.monotonic() + timeout_s * 3 + 30
            codes = []
            for p, ident in procs:
                try:
                    p.wait(max(1.0, deadline - time.monotonic()))
                except subprocess.TimeoutExpired:
                    terminate_group(ident)
                codes.append(p.returncode)
            errors = [p.stderr.read() if p.stderr else "" for p, _ in procs]
            if any(c != 0 for c in codes):
                raise RuntimeFailure("native driver failed: codes %s; %s" % (codes, " | ".join(e[-400:] for e in errors)))
            receipts = [json.loads((tmp / ("receipt-%d.json" % r)).read_text()) for r in range(self.nranks)]
        return combine_schedule_results(receipts)
