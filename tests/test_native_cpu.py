"""Production C++ (contract utilities, TCP control plane) compiled with g++ and run on the CPU."""
import subprocess

from vericcl_b200.execution.native import combine_schedule_results
from vericcl_b200.ops.build import build_native_tests


def test_native_contract_and_control_plane():
    binary = build_native_tests()
    proc = subprocess.run([str(binary)], capture_output=True, text=True, timeout=120)
    assert proc.returncode == 0, proc.stdout + proc.stderr
    assert "native cpu tests passed" in proc.stdout


def test_combine_takes_slowest_rank_per_invocation():
    out = combine_schedule_results([{"device_times_us": [1, 5, 3], "bad": 0}, {"device_times_us": [2, 4, 3], "bad": 0}])
    assert out["per_invocation_us"] == [2, 5, 3] and out["mean_us"] == 10 / 3
