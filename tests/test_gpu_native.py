"""The C API driver (vericcl-native) on two GPUs: analytic device check of an AllReduce."""
import pytest

from vericcl_b200.synthesis import schedule_xml


def _gpus():
    try:
        import torch
        return torch.cuda.device_count()
    except Exception:
        return 0


@pytest.mark.gpu
@pytest.mark.multigpu
def test_native_driver_allreduce_two_gpus():
    if _gpus() < 2:
        pytest.skip("needs two GPUs")
    from vericcl_b200.execution.native import NativeScheduleDriver
    xml = schedule_xml("allreduce", 2, 2)
    res = NativeScheduleDriver(xml, 2).measure(count=1 << 16, nlanes=16, iters=5, timeout_s=20)
    assert res["bad"] == 0
    assert len(res["per_invocation_us"]) == 5 and res["mean_us"] > 0


@pytest.mark.gpu
@pytest.mark.multigpu
def test_native_driver_writes_step_traces(tmp_path):
    if _gpus() < 2:
        pytest.skip("needs two GPUs")
    from vericcl_b200.execution.native import NativeScheduleDriver
    from vericcl_b200.online.trace import parse_trace
    xml = schedule_xml("allreduce", 2, 2)
    res = NativeScheduleDriver(xml, 2).measure(count=1 << 16, nlanes=4, iters=3, timeout_s=20, trace_dir=tmp_path)
    assert res["bad"] == 0
    for rank in range(2):
        doc = parse_trace((tmp_path / ("trace-rank%d.bin" % rank)).read_bytes(), partial_ok=False)
        assert doc["rank"] == rank and doc["complete"] and doc["records"]
        assert all(r.end_ns >= r.start_ns > 0 for r in doc["records"])


@pytest.mark.gpu
@pytest.mark.multigpu
@pytest.mark.parametrize("coll,root", [("reduce_scatter", 0), ("alltoall", 0), ("broadcast", 1), ("reduce", 1),
                                       ("allgather", 0)])
def test_native_driver_checks_every_collective(coll, root):
    """The driver's analytic check and read-only input re-check cover each collective kind."""
    if _gpus() < 2:
        pytest.skip("needs two GPUs")
    from vericcl_b200.execution.native import NativeScheduleDriver
    slices = 2
    xml = schedule_xml(coll, 2, slices, root=root if coll in ("broadcast", "reduce") else 0)
    res = NativeScheduleDriver(xml, 2).measure(count=1 << 14, nlanes=4, iters=2, timeout_s=20, root=root)
    assert res["bad"] == 0 and res["bad_input"] == 0
