"""Job transport for native runs: local or ssh hosts, machine inventory, manifests.

A rank of a native job runs on the host that ``runtime.rank_map`` names.  A
host that resolves to this machine runs the command directly; any other host
is reached with ``ssh`` (batch mode, no password prompts) after its inputs
are staged with ``scp`` into a per-session directory under the remote home
(staging paths are home-relative; absolute or parent-escaping paths are
refused), and its outputs are fetched back the same way.  The machine
inventory (GPU UUIDs and names through read-only NVML, driver and library
versions, digests of this package's native artifacts) identifies where a
measurement came from; ``export_manifest`` writes it with the sha256 of every
artifact of a run directory (reference: vericcl/online/remote.py:122-240,442-520
and vericcl/execution/manifest.py:13).
"""
from __future__ import annotations

import hashlib
import shlex
import shutil
import socket
import subprocess
from dataclasses import dataclass
from pathlib import Path, PurePosixPath

from vericcl_b200.errors import RuntimeFailure

NATIVE_DIR = Path(__file__).resolve().parents[1] / "_native"


def _local_addresses() -> set:
    addrs = {"127.0.0.1", "::1", "localhost"}
    for name in (socket.gethostname(), socket.getfqdn()):
        addrs.add(name)
        try:
            for info in socket.getaddrinfo(name, None):
                addrs.add(info[4][0])
        except OSError:
            pass
    return addrs


def is_local(host: str | None) -> bool:
    """True when ``host`` names this machine (empty, loopback, own name or one of its addresses)."""
    if not host:
        return True
    local = _local_addresses()
    if host in local or host.startswith("127."):
        return True
    try:
        return any(info[4][0] in local or info[4][0].startswith("127.") for info in socket.getaddrinfo(host, None))
    except OSError:
        return False


def _home_relative(path: str) -> str:
    p = PurePosixPath(path)
    if p.is_absolute() or ".." in p.parts or not p.parts:
        raise RuntimeFailure("remote staging paths must stay inside the remote home: %r" % path)
    return str(p)


@dataclass
class HostRunner:
    """Runs commands and moves files for one host (directly when it is this machine)."""
    host: str = "localhost"
    ssh: str = "ssh"
    scp: str = "scp"
    stage_root: str = ".vericcl_b200/stage"
    timeout_s: float = 120.0

    @property
    def local(self) -> bool:
        return is_local(self.host)

    def stage_dir(self, session: str) -> str:
        return _home_relative(str(PurePosixPath(self.stage_root) / session))

    def command(self, argv) -> list:
        """The argv that runs ``argv`` on this host."""
        if self.local:
            return [str(a) for a in argv]
        return [self.ssh, "-o", "BatchMode=yes", self.host, "--", " ".join(shlex.quote(str(a)) for a in argv)]

    def _run(self, argv) -> None:
        res = subprocess.run(argv, capture_output=True, text=True, timeout=self.timeout_s)
        if res.returncode != 0:
            raise RuntimeFailure("%s failed on %s: %s" % (argv[0], self.host, res.stderr[-500:]))

    def stage(self, files, session: str) -> dict:
        """Copy ``files`` to the host's session directory; returns {local path: path on the host}."""
        files = [Path(f) for f in files]
        if self.local:
            return {f: str(f) for f in files}
        remote = self.stage_dir(session)
        self._run(self.command(["mkdir", "-p", remote]))
        out = {}
        for f in files:
            target = str(PurePosixPath(remote) / f.name)
            self._run([self.scp, "-q", "-B", str(f), "%s:%s" % (self.host, target)])
            out[f] = target
        return out

    def fetch(self, remote_path: str, local_path) -> None:
        local_path = Path(local_path)
        if self.local:
            if Path(remote_path).resolve() != local_path.resolve():
                shutil.copyfile(remote_path, local_path)
            return
        self._run([self.scp, "-q", "-B", "%s:%s" % (self.host, _home_relative(remote_path)), str(local_path)])

    def cleanup(self, session: str) -> None:
        if not self.local:
            subprocess.run(self.command(["rm", "-rf", self.stage_dir(session)]), capture_output=True,
                           timeout=self.timeout_s)


def _sha256(path: Path) -> str:
    h = hashlib.sha256()
    with open(path, "rb") as handle:
        for block in iter(lambda: handle.read(1 << 20), b""):
            h.update(block)
    return h.hexdigest()


def machine_inventory() -> dict:
    """Where a measurement ran: host, GPUs (read-only NVML), driver and library versions, native artifacts."""
    inv = {"host": socket.gethostname(), "gpus": [], "driver": None}
    try:
        import pynvml
        pynvml.nvmlInit()
        try:
            drv = pynvml.nvmlSystemGetDriverVersion()
            inv["driver"] = drv.decode() if isinstance(drv, bytes) else drv
            for i in range(pynvml.nvmlDeviceGetCount()):
                h = pynvml.nvmlDeviceGetHandleByIndex(i)
                name = pynvml.nvmlDeviceGetName(h)
                inv["gpus"].append({"index": i, "uuid": pynvml.nvmlDeviceGetUUID(h),
                                    "name": name.decode() if isinstance(name, bytes) else name,
                                    "memory_bytes": int(pynvml.nvmlDeviceGetMemoryInfo(h).total)})
        finally:
            pynvml.nvmlShutdown()
    except Exception as error:   # no NVML (CPU machine): record why
        inv["nvml"] = "unavailable: %s" % type(error).__name__
    try:
        import torch
        inv["torch"] = torch.__version__
        inv["cuda_runtime"] = torch.version.cuda
        nccl = torch.cuda.nccl.version() if torch.cuda.is_available() else None
        inv["nccl"] = ".".join(map(str, nccl)) if isinstance(nccl, tuple) else nccl
    except Exception:
        pass
    inv["native"] = {p.name: _sha256(p) for p in sorted(NATIVE_DIR.glob("*"))
                     if p.is_file() and not p.name.endswith(".stamp")} if NATIVE_DIR.exists() else {}
    return inv


def export_manifest(run_dir, inventory: dict | None = None) -> Path:
    """``manifest.json`` of a run directory: every artifact with size and sha256, plus the inventory.

    ``run.json`` (the run's mutable index, updated until the run finishes) is not listed.
    """
    from vericcl_b200.utils.jsonio import atomic_write_json
    run_dir = Path(run_dir)
    files = []
    for p in sorted(run_dir.rglob("*")):
        if p.is_file() and p.relative_to(run_dir).as_posix() not in ("manifest.json", "run.json"):
            files.append({"path": str(p.relative_to(run_dir)), "bytes": p.stat().st_size, "sha256": _sha256(p)})
    return atomic_write_json(run_dir / "manifest.json",
                             {"schema_version": 1, "files": files,
                              "inventory": inventory if inventory is not None else machine_inventory()})
