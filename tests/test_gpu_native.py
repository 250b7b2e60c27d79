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
