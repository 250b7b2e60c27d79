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
            "bad": sum(r["bad"] for r in receipts), "bad_input": sum(r.get("bad_input", 0) for r in receipts)}


class NativeScheduleDriver:
    """Run every rank of a schedule through the native driver and combine the receipts.

    ``hosts`` names each rank's host (default: all on this machine); ranks on
    other hosts are launched over ssh with the driver, its library, the
    schedule and the rank's configuration staged into a per-session
    directory (:class:`~vericcl_b200.execution.transport.HostRunner`), and
    rank 0's host serves the control plane.  With a ``registry`` the local
    GPUs of the job are held in the GPU ownership registry under ``owner``
    while it runs, released with a receipt afterwards, and quarantined when a
    rank's process group cannot be confirmed gone.
    """

    def __init__(self, xml: str, nranks: int, *, devices=None, binary=None, port: int | None = None, hosts=None,
                 registry=None, owner: str | None = None, runner_factory=None, environment=None):
        from vericcl_b200.execution.transport import HostRunner
        self.xml = xml
        self.nranks = nranks
        self.devices = list(devices) if devices is not None else list(range(nranks))
        if binary is None:
            from vericcl_b200.ops.build import build_driver
            binary = build_driver()
        self.binary = Path(binary)
        self.port = port or (20000 + secrets.randbelow(20000))
        self.hosts = list(hosts) if hosts is not None else ["localhost"] * nranks
        if len(self.hosts) != nranks or len(self.devices) != nranks:
            raise RuntimeFailure("hosts and devices need one entry per rank")
        factory = runner_factory or (lambda host: HostRunner(host))
        self.runners = [factory(h) for h in self.hosts]
        self.registry = registry
        self.owner = owner or "native-%s" % secrets.token_hex(4)
        # runtime.environment of the request: exported to every rank's process
        self.environment = {str(k): str(v) for k, v in (environment or {}).items()}

    def _local_uuids(self):
        from vericcl_b200.execution.ownership import local_gpu_uuids
        devices = sorted({d for d, r in zip(self.devices, self.runners) if r.local})
        if not devices:
            return []
        uuids = local_gpu_uuids(max(devices) + 1)
        return [uuids[d] for d in devices]

    def measure(self, *, count: int, dtype: int = 0, redop: int = 0, scale: float = 1.0, nlanes: int = 32,
                niters: int = 1, warmup: int = 3, iters: int = 10, timeout_s: float = 60.0, trace_dir=None,
                grace_s: float = 30.0, root: int = 0):
        """Device-timed invocations; with ``trace_dir`` every rank also writes
        ``trace-rank<r>.bin`` (per-step trace of its last invocation).  A rank
        still running ``3 · timeout_s + grace_s`` after the launch has its
        process group terminated and the measurement fails."""
        uuids = self._local_uuids() if self.registry is not None else []
        if uuids:
            self.registry.acquire(uuids, self.owner)
        session = secrets.token_hex(4)
        self.last_clean = True
        try:
            result = self._run(session, count, dtype, redop, scale, nlanes, niters, warmup, iters, timeout_s,
                               trace_dir, grace_s, root)
        except Exception:
            if uuids:
                if self.last_clean:
                    self.registry.release(uuids, self.owner, {"session": session, "result": "failed"})
                else:
                    self.registry.quarantine(uuids, self.owner, "a rank's process group outlived its deadline")
            raise
        finally:
            for runner in {r.host: r for r in self.runners}.values():
                runner.cleanup(session)
        if uuids:
            if self.last_clean:
                self.registry.release(uuids, self.owner, {"session": session, "mean_us": result["mean_us"]})
            else:
                self.registry.quarantine(uuids, self.owner, "a rank's process group outlived its deadline")
        return result

    def _run(self, session, count, dtype, redop, scale, nlanes, niters, warmup, iters, timeout_s, trace_dir,
             grace_s=30.0, root=0):
        from vericcl_b200.ops.build import OUT
        all_local = all(r.local for r in self.runners)
        control = "127.0.0.1" if all_local else self.hosts[0]
        lib = OUT / "libvericcl_b200.so"
        with tempfile.TemporaryDirectory() as tmp:
            tmp = Path(tmp)
            xml_path = tmp / "schedule.xml"
            xml_path.write_text(self.xml)
            staged = {}
            procs = []
            for rank, runner in enumerate(self.runners):
                if runner.local:
                    where = {"xml": str(xml_path), "binary": str(self.binary),
                             "receipt": str(tmp / ("receipt-%d.json" % rank)),
                             "trace": str(Path(trace_dir) / ("trace-rank%d.bin" % rank)) if trace_dir else None}
                else:
                    if runner.host not in staged:
                        files = [self.binary, xml_path] + ([lib] if lib.exists() else [])
                        staged[runner.host] = runner.stage(files, session)
                    stage = runner.stage_dir(session)
                    where = {"xml": staged[runner.host][xml_path], "binary": staged[runner.host][self.binary],
                             "receipt": "%s/receipt-%d.json" % (stage, rank),
                             "trace": "%s/trace-rank%d.bin" % (stage, rank) if trace_dir else None}
                cfg = {"xml": where["xml"], "rank": rank, "nranks": self.nranks, "device": self.devices[rank],
                       "control_address": control, "control_port": self.port, "session": session, "count": count,
                       "dtype": dtype, "redop": redop, "scale": scale, "nlanes": nlanes, "niters": niters,
                       "warmup": warmup, "iters": iters, "timeout_s": timeout_s, "receipt": where["receipt"],
                       "root": root}
                if trace_dir is not None:
                    Path(trace_dir).mkdir(parents=True, exist_ok=True)
                    cfg["trace"] = where["trace"]
                path = tmp / ("config-%d.json" % rank)
                path.write_text(json.dumps(cfg))
                cfg_arg = str(path) if runner.local else runner.stage([path], session)[path]
                if runner.local:
                    argv, env = runner.command([where["binary"], cfg_arg]), dict(os.environ, **self.environment)
                else:
                    exports = ["%s=%s" % kv for kv in sorted(self.environment.items())]
                    prefix = ["env"] + exports if exports else []
                    argv, env = runner.command(prefix + [where["binary"], cfg_arg]), None
                p = subprocess.Popen(argv, stdout=subprocess.PIPE, stderr=subprocess.PIPE, text=True,
                                     start_new_session=True, env=env)
                procs.append((p, ProcessIdentity(p.pid, os.getpgid(p.pid), start_time(p.pid), boot_id()), where))
            deadline = time.monotonic() + timeout_s * 3 + grace_s
            codes = []
            for p, ident, _ in procs:
                try:
                    p.wait(max(1.0, deadline - time.monotonic()))
                except subprocess.TimeoutExpired:
                    self.last_clean = terminate_group(ident) and self.last_clean
                    try:
                        p.wait(5.0)            # reap it, so its exit status is known
                    except subprocess.TimeoutExpired:
                        self.last_clean = False
                codes.append(p.returncode)
            errors = [p.stderr.read() if p.stderr else "" for p, _, _ in procs]
            if any(c != 0 for c in codes):
                raise RuntimeFailure("native driver failed: codes %s; %s"
                                     % (codes, " | ".join(e[-400:] for e in errors)))
            receipts = []
            for rank, (runner, (_, _, where)) in enumerate(zip(self.runners, procs)):
                local_receipt = tmp / ("receipt-%d.json" % rank)
                runner.fetch(where["receipt"], local_receipt)
                receipts.append(json.loads(local_receipt.read_text()))
                if trace_dir is not None and not runner.local:
                    runner.fetch(where["trace"], Path(trace_dir) / ("trace-rank%d.bin" % rank))
        return combine_schedule_results(receipts)
