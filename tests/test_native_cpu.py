"""Production C++ (contract utilities, TCP control plane) compiled with g++ and run on the CPU."""
import subprocess

from vericcl_b200.execution.native import combine_schedule_results
from vericcl_b200.ops.build import build_native_tests


def test_native_contract_and_control_plane(tmp_path):
    binary = build_native_tests()
    trace = tmp_path / "trace-rank3.bin"
    proc = subprocess.run([str(binary), str(trace)], capture_output=True, text=True, timeout=120)
    assert proc.returncode == 0, proc.stdout + proc.stderr
    assert "native cpu tests passed" in proc.stdout
    # the C++ trace writer and the Python reader agree on the file layout
    from vericcl_b200.online.trace import parse_trace
    doc = parse_trace(trace.read_bytes(), partial_ok=False)
    assert doc["rank"] == 3 and doc["ctas"] == 4 and doc["steps"] == 3 and doc["complete"]
    recs = doc["records"]
    assert len(recs) == 16
    ops = {0: [1, 2, 0], 1: [4]}
    for r in recs:
        assert r.start_ns == 1000 * r.cta + 100 * r.iteration + 10 * r.step + 1
        assert r.end_ns == r.start_ns + 4 and r.wait_ns == 2
        assert r.block == r.cta // 2 and r.lane == r.cta % 2 and r.op == ops[r.block][r.step]


def test_combine_takes_slowest_rank_per_invocation():
    out = combine_schedule_results([{"device_times_us": [1, 5, 3], "bad": 0}, {"device_times_us": [2, 4, 3], "bad": 0}])
    assert out["per_invocation_us"] == [2, 5, 3] and out["mean_us"] == 10 / 3
    assert out["bad"] == 0 and out["bad_input"] == 0
    changed = combine_schedule_results([{"device_times_us": [1], "bad": 0, "bad_input": 3},
                                        {"device_times_us": [1], "bad": 2, "bad_input": 0}])
    assert changed["bad"] == 2 and changed["bad_input"] == 3


def test_capi_execute_path_on_cpu_stand_ins(tmp_path):
    """vb_execute staging symmetry and unresolved-execution ownership, two ranks as threads (no GPU)."""
    from vericcl_b200.ops.build import build_capi_cpu_tests
    from vericcl_b200.synthesis import schedule_xml
    binary = build_capi_cpu_tests()
    ar, rd = tmp_path / "allreduce.xml", tmp_path / "reduce.xml"
    ar.write_text(schedule_xml("allreduce", 2, 2))
    rd.write_text(schedule_xml("reduce", 2, 2, root=1))
    proc = subprocess.run([str(binary), str(ar), str(rd)], capture_output=True, text=True, timeout=120)
    assert proc.returncode == 0, proc.stdout + proc.stderr
    assert "capi cpu tests passed" in proc.stdout
