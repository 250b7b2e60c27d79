"""Concurrent builds of the in-tree native modules: one process builds at a time, every process ends with a
module that loads (several ranks of a multi-GPU job import the extension at the same moment)."""
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_two_processes_rebuilding_at_once_both_succeed():
    code = ("import time; from vericcl_b200.ops import build; t = time.monotonic(); "
            "build.build_plan_module(force=True); print(round(time.monotonic() - t, 2))")
    procs = [subprocess.Popen([sys.executable, "-c", code], cwd=ROOT, stdout=subprocess.PIPE,
                              stderr=subprocess.PIPE, text=True) for _ in range(2)]
    outs = [p.communicate(timeout=600) for p in procs]
    assert all(p.returncode == 0 for p in procs), [o[1][-2000:] for o in outs]
    load = subprocess.run([sys.executable, "-c", "from vericcl_b200.ops import native; "
                           "m = native.plan(); print(m.__file__)"], cwd=ROOT, capture_output=True, text=True,
                          timeout=300)
    assert load.returncode == 0, load.stderr[-2000:]
    assert "_vbplan" in load.stdout
