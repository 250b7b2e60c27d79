"""Job transport on the CPU: ranks on "remote" hosts through fake ssh/scp, ownership, inventory, manifests."""
import json
import stat
import sys
from pathlib import Path

import pytest

from vericcl_b200.errors import RuntimeFailure
from vericcl_b200.execution.native import NativeScheduleDriver
from vericcl_b200.execution.ownership import GPUOwnershipRegistry, local_gpu_uuids
from vericcl_b200.execution.transport import HostRunner, export_manifest, is_local, machine_inventory

FAKE_DRIVER = """#!{py}
import json, os, sys
cfg = json.load(open(sys.argv[1]))
rank = cfg["rank"]
with open(cfg["receipt"], "w") as f:
    json.dump({{"rank": rank, "nranks": cfg["nranks"], "bad": 0, "env": os.environ.get("VB_TEST_ENV"),
               "device_times_us": [10.0 + rank, 20.0 - rank, 30.0]}}, f)
if "trace" in cfg:
    open(cfg["trace"], "wb").write(b"trace-of-rank-%d" % rank)
"""

# ssh HOST -- CMD: run CMD in that host's fake home
FAKE_SSH = """#!/bin/sh
while [ "$1" = "-o" ]; do shift 2; done
host="$1"; shift; [ "$1" = "--" ] && shift
mkdir -p "$FAKE_ROOT/$host" && cd "$FAKE_ROOT/$host" && exec sh -c "$*"
"""

# scp -q -B SRC DST with one side HOST:PATH (relative to that host's fake home)
FAKE_SCP = """#!/bin/sh
shift 2
map() { case "$1" in *:*) h="${1%%:*}"; echo "$FAKE_ROOT/$h/${1#*:}";; *) echo "$1";; esac; }
src=$(map "$1"); dst=$(map "$2"); mkdir -p "$(dirname "$dst")"; cp "$src" "$dst"
"""


def _script(path: Path, text: str) -> Path:
    path.write_text(text)
    path.chmod(path.stat().st_mode | stat.S_IXUSR)
    return path


@pytest.fixture
def fakes(tmp_path, monkeypatch):
    root = tmp_path / "hosts"
    root.mkdir()
    monkeypatch.setenv("FAKE_ROOT", str(root))
    ssh = _script(tmp_path / "fake_ssh", FAKE_SSH)
    scp = _script(tmp_path / "fake_scp", FAKE_SCP)
    driver = _script(tmp_path / "fake_driver", FAKE_DRIVER.format(py=sys.executable))
    return root, ssh, scp, driver


def test_is_local():
    assert is_local("") and is_local("localhost") and is_local("127.0.0.1")
    assert not is_local("gpu-node-17.invalid")


def test_remote_command_and_home_confined_staging():
    r = HostRunner("gpu-node-17.invalid")
    assert r.command(["a b", "c"]) == ["ssh", "-o", "BatchMode=yes", "gpu-node-17.invalid", "--", "'a b' c"]
    assert r.stage_dir("s1") == ".vericcl_b200/stage/s1"
    with pytest.raises(RuntimeFailure):
        HostRunner("h.invalid", stage_root="/etc").stage_dir("x")
    with pytest.raises(RuntimeFailure):
        HostRunner("h.invalid", stage_root="../up").stage_dir("x")


def test_ranks_on_remote_hosts_through_ssh(fakes, tmp_path):
    root, ssh, scp, driver = fakes
    hosts = ["localhost", "node-a.invalid", "node-b.invalid"]
    reg = GPUOwnershipRegistry(tmp_path / "owners.json")
    drv = NativeScheduleDriver("<algo/>", 3, binary=driver, hosts=hosts, registry=reg, owner="job-1",
                               runner_factory=lambda h: HostRunner(h, ssh=str(ssh), scp=str(scp)))
    res = drv.measure(count=16, iters=3, timeout_s=20, trace_dir=tmp_path / "traces")
    assert res["per_invocation_us"] == [12.0, 20.0, 30.0] and res["bad"] == 0
    for rank in range(3):
        assert (tmp_path / "traces" / ("trace-rank%d.bin" % rank)).read_bytes() == b"trace-of-rank-%d" % rank
    # the remote hosts received the staged driver and schedule, and the session directory was cleaned up
    assert (root / "node-a.invalid" / ".vericcl_b200" / "stage").exists()
    assert not any((root / "node-a.invalid" / ".vericcl_b200" / "stage").iterdir())
    # the local GPU of rank 0 was held during the run and released with a receipt
    uuid = local_gpu_uuids(1)[0]
    assert reg.state(uuid)["state"] == "released" and reg.state(uuid)["receipt"]["mean_us"] > 0


def test_busy_gpu_is_refused(fakes, tmp_path):
    _, ssh, scp, driver = fakes
    reg = GPUOwnershipRegistry(tmp_path / "owners.json")
    reg.acquire([local_gpu_uuids(1)[0]], "someone-else")
    drv = NativeScheduleDriver("<algo/>", 1, binary=driver, registry=reg, owner="job-2")
    with pytest.raises(RuntimeFailure, match="active"):
        drv.measure(count=16, iters=1, timeout_s=10)


def test_failed_rank_releases_and_reports(fakes, tmp_path):
    _, _, _, driver = fakes
    bad = _script(tmp_path / "bad_driver", "#!/bin/sh\necho boom >&2\nexit 8\n")
    reg = GPUOwnershipRegistry(tmp_path / "owners.json")
    drv = NativeScheduleDriver("<algo/>", 2, binary=bad, registry=reg, owner="job-3")
    with pytest.raises(RuntimeFailure, match="boom"):
        drv.measure(count=16, iters=1, timeout_s=10)
    assert reg.unresolved("job-3") == []


def test_inventory_and_manifest(tmp_path):
    inv = machine_inventory()
    assert inv["host"] and isinstance(inv["gpus"], list)
    run = tmp_path / "run"
    (run / "process").mkdir(parents=True)
    (run / "schedule.xml").write_text("<algo/>")
    (run / "process" / "events.jsonl").write_text("{}\n")
    path = export_manifest(run, inventory={"host": "h"})
    doc = json.loads(Path(path).read_text())
    assert {f["path"] for f in doc["files"]} == {"schedule.xml", "process/events.jsonl"}
    assert all(len(f["sha256"]) == 64 for f in doc["files"]) and doc["inventory"] == {"host": "h"}


def test_runtime_environment_reaches_every_rank(fakes, tmp_path, monkeypatch):
    import json as _json
    from vericcl_b200.execution import native as native_mod
    root, ssh, scp, driver = fakes
    seen = []
    real = native_mod.combine_schedule_results

    def spy(receipts):
        seen.extend(r.get("env") for r in receipts)
        return real(receipts)
    monkeypatch.setattr(native_mod, "combine_schedule_results", spy)
    drv = NativeScheduleDriver("<algo/>", 2, binary=driver, hosts=["localhost", "node-c.invalid"],
                               environment={"VB_TEST_ENV": "x y"},
                               runner_factory=lambda h: HostRunner(h, ssh=str(ssh), scp=str(scp)))
    drv.measure(count=16, iters=1, timeout_s=20)
    assert seen == ["x y", "x y"]
    assert _json  # module used above


def test_hung_rank_is_terminated_and_reported(fakes, tmp_path):
    """A rank that never finishes is killed at the deadline; the others' results are not combined."""
    _, _, _, driver = fakes
    hang = _script(tmp_path / "hang_driver", "#!/bin/sh\n"
                   "case \"$(cat \"$1\")\" in *'\"rank\": 1'*) exec sleep 600;; esac\n"
                   "exec \"%s\" \"$1\"\n" % driver)
    reg = GPUOwnershipRegistry(tmp_path / "owners.json")
    drv = NativeScheduleDriver("<algo/>", 2, binary=hang, registry=reg, owner="job-4")
    import time
    t0 = time.monotonic()
    with pytest.raises(RuntimeFailure, match="codes"):
        drv.measure(count=16, iters=1, timeout_s=0.5, grace_s=1.0)
    assert time.monotonic() - t0 < 30
    # the hung rank's group was terminated, so its GPU is released rather than quarantined
    assert reg.unresolved("job-4") == []
