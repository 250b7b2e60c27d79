"""Owned child processes with bounded termination.

A child runs in its own process group; its identity (pid, process-group id,
start time from /proc, boot id) is recorded so a later run can tell whether
a leftover process is still the same one.  On deadline the whole group gets
SIGTERM, then SIGKILL after a grace period; output is captured and redacted
(reference: vericcl/execution/processes.py:36-197).
"""
from __future__ import annotations

import os
import signal
import subprocess
import time
from dataclasses import asdict, dataclass
from pathlib import Path

from vericcl_b200.execution.security import Redactor


def boot_id() -> str:
    try:
        return Path("/proc/sys/kernel/random/boot_id").read_text().strip()
    except OSError:
        return "unknown"


def _stat(pid: int):
    try:
        return Path("/proc/%d/stat" % pid).read_text().rsplit(")", 1)[1].split()
    except (OSError, IndexError):
        return None


def start_time(pid: int) -> int | None:
    fields = _stat(pid)
    try:
        return int(fields[19]) if fields else None
    except (IndexError, ValueError):
        return None


def is_zombie(pid: int) -> bool:
    """True when the process has exited and only waits to be reaped by its parent."""
    fields = _stat(pid)
    return bool(fields) and fields[0] in ("Z", "X")


@dataclass(frozen=True)
class ProcessIdentity:
    pid: int
    pgid: int
    start_ticks: int | None
    boot_id: str

    def alive(self) -> bool:
        """The recorded process still runs (an exited process awaiting its reaper counts as gone)."""
        return (boot_id() == self.boot_id and self.start_ticks is not None and start_time(self.pid) == self.start_ticks
                and not is_zombie(self.pid))


@dataclass
class ProcessResult:
    identity: ProcessIdentity
    returncode: int | None
    stdout: str
    stderr: str
    timed_out: bool
    duration_s: float

    def as_json(self):
        d = asdict(self)
        d["identity"] = asdict(self.identity)
        return d


def run_owned_process(cmd, *, timeout_s: float, env=None, cwd=None, grace_s: float = 5.0, redactor=None,
                      record_dir=None) -> ProcessResult:
    redactor = redactor or Redactor()
    t0 = time.monotonic()
    proc = subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.PIPE, env=env, cwd=cwd, text=True,
                            start_new_session=True)
    ident = ProcessIdentity(proc.pid, os.getpgid(proc.pid), start_time(proc.pid), boot_id())
    if record_dir is not None:
        from vericcl_b200.utils.jsonio import atomic_write_json
        atomic_write_json(Path(record_dir) / "identity.json", asdict(ident))
    timed_out = False
    try:
        out, err = proc.communicate(timeout=timeout_s)
    except subprocess.TimeoutExpired:
        timed_out = True
        terminate_group(ident, grace_s)
        out, err = proc.communicate()
    result = ProcessResult(ident, proc.returncode, redactor.redact(out or ""), redactor.redact(err or ""),
                           timed_out, time.monotonic() - t0)
    if record_dir is not None:
        from vericcl_b200.utils.jsonio import atomic_write_json
        atomic_write_json(Path(record_dir) / "exit.json", result.as_json())
    return result


def terminate_group(ident: ProcessIdentity, grace_s: float = 5.0) -> bool:
    """SIGTERM then SIGKILL the identified process group; True when it is gone."""
    for sig, wait in ((signal.SIGTERM, grace_s), (signal.SIGKILL, 2.0)):
        try:
            os.killpg(ident.pgid, sig)
        except ProcessLookupError:
            return True
        deadline = time.monotonic() + wait
        while time.monotonic() < deadline:
            if not ident.alive():
                return True
            time.sleep(0.05)
    return not ident.alive()


def reconcile_owned_process(identity: dict) -> str:
    """State of a process recorded by an earlier run: ``gone`` or ``running``."""
    ident = ProcessIdentity(**identity)
    return "running" if ident.alive() else "gone"
