import json
import sys

import pytest

from vericcl_b200.errors import BudgetExhausted, RuntimeFailure
from vericcl_b200.execution.budget import BudgetManager, StandaloneLease
from vericcl_b200.execution.context import RunContext
from vericcl_b200.execution.checkpoint import restore_checkpoint, save_checkpoint
from vericcl_b200.execution.events import EventLog, verify_sequence
from vericcl_b200.execution.ownership import GPUOwnershipRegistry
from vericcl_b200.execution.processes import reconcile_owned_process, run_owned_process
from vericcl_b200.execution.security import Redactor


def test_events_sequence_and_truncated_tail(tmp_path):
    log = EventLog(tmp_path)
    for i in range(3):
        log.emit("k", i=i, password="hunter2")
    text = (tmp_path / "events.jsonl").read_text()
    assert "hunter2" not in text
    (tmp_path / "events.jsonl").write_text(text + '{"sequence": 4, "trunc')
    log2 = EventLog(tmp_path)
    assert log2.sequence == 3 and verify_sequence(log2.read())


def test_budget_manager_leases():
    clock = [0.0]
    mgr = BudgetManager({"max_repair_per_round_s": 10, "max_repair_total_s": 15}, clock=lambda: clock[0])
    lease = mgr.acquire("repair")
    clock[0] = 9.0
    lease.check()
    clock[0] = 10.5
    with pytest.raises(BudgetExhausted):
        lease.check()
    lease.release()
    mgr.new_round()
    assert mgr.remaining("repair") == pytest.approx(5.0)
    lease = StandaloneLease.after(6, clock=lambda: clock[0])
    clock[0] += 7
    with pytest.raises(BudgetExhausted):
        lease.check()


def test_owned_process_timeout_kills_group(tmp_path):
    res = run_owned_process([sys.executable, "-c", "import time; time.sleep(30)"], timeout_s=0.5, grace_s=0.5,
                            record_dir=tmp_path)
    assert res.timed_out and reconcile_owned_process(res.identity.__dict__) == "gone"
    assert json.loads((tmp_path / "exit.json").read_text())["timed_out"]
    ok = run_owned_process([sys.executable, "-c", "print('token=abc')"], timeout_s=30, redactor=Redactor(["abc"]))
    assert ok.returncode == 0 and "abc" not in ok.stdout


def test_gpu_ownership(tmp_path):
    reg = GPUOwnershipRegistry(tmp_path / "own.json")
    reg.acquire(["GPU-a"], "run1")
    with pytest.raises(RuntimeFailure):
        reg.acquire(["GPU-a"], "run2")
    assert reg.unresolved("run1") == ["GPU-a"]
    reg.release(["GPU-a"], "run1", {"exit": 0})
    reg.acquire(["GPU-a"], "run2")
    reg.quarantine(["GPU-a"], "run2", "no release receipt")
    with pytest.raises(RuntimeFailure):
        reg.acquire(["GPU-a"], "run3")


def test_checkpoint_tamper_detection(tmp_path):
    ctx = RunContext.create(tmp_path, "c", "solve", run_id="x")
    (ctx.directory / "art.txt").write_text("v1")
    save_checkpoint(ctx, phase="p", state={"a": 1}, files=["art.txt"], budgets={"elapsed_s": 1.0})
    doc = restore_checkpoint(ctx)
    assert doc["state"] == {"a": 1} and doc["downtime_s"] >= 0
    (ctx.directory / "art.txt").write_text("v2")
    with pytest.raises(RuntimeFailure):
        restore_checkpoint(ctx)
    reg = GPUOwnershipRegistry(tmp_path / "own.json")
    reg.acquire(["GPU-z"], "x")
    (ctx.directory / "art.txt").write_text("v1")
    with pytest.raises(RuntimeFailure, match="ownership"):
        restore_checkpoint(ctx, registry=reg, owner="x")
