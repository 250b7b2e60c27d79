"""Clean-checkout check: every source the native build and the entry points need is tracked by git."""
import shutil
import subprocess
from pathlib import Path

import pytest

from vericcl_b200.ops import build

ROOT = Path(__file__).resolve().parents[1]


def _tracked():
    if shutil.which("git") is None or not (ROOT / ".git").exists():
        pytest.skip("not a git checkout")
    out = subprocess.run(["git", "ls-files"], cwd=ROOT, capture_output=True, text=True, check=True).stdout
    return set(out.split())


def test_build_sources_are_tracked():
    tracked = _tracked()
    rel = []
    for name in ("RUNTIME_SOURCES", "CUDA_SOURCES", "PLAN_SOURCES", "CAPI_SOURCES"):
        rel += ["csrc/" + s for s in getattr(build, name, [])]
    rel += ["csrc/cuda/noalloc.cu", "csrc/runtime/driver.cc", "tests/native/test_control_and_contract.cc",
            "tests/native/test_capi_cpu.cc", "tests/native/cpu_stubs/stubs.cc", "tests/native/cpu_stubs/cuda.h",
            "tests/native/cpu_stubs/cuda_runtime.h", "tests/requirements.json"]
    headers = [str(p.relative_to(ROOT)) for p in (ROOT / "csrc" / "include").rglob("*.h")]
    missing = [p for p in rel + headers if p not in tracked]
    assert not missing, missing


def test_entry_points_and_no_build_outputs_tracked():
    tracked = _tracked()
    for path in ("__graft_entry__.py", "bench.py", "sweep.py", "README.md", "pytest.ini"):
        assert path in tracked
    built = [p for p in tracked if p.endswith((".so", ".o", ".stamp", ".ncu-rep")) or p.startswith("_work/")]
    assert not built, built
