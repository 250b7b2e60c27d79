"""Multi-GPU correctness of the interpreter (torchrun over the visible GPUs)."""
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _gpus():
    try:
        import torch
        return torch.cuda.device_count()
    except Exception:
        return 0


@pytest.mark.gpu
@pytest.mark.multigpu
def test_collectives_two_gpus():
    if _gpus() < 2:
        pytest.skip("needs two GPUs")
    env = dict(os.environ, VB_QUICK="1", NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr", "127.0.0.1", "--master-port", "29533",
           os.path.join(ROOT, "tests", "mp_collectives.py")]
    proc = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=700)
    assert proc.returncode == 0, proc.stdout[-4000:] + proc.stderr[-4000:]
    assert '"failures": 0' in proc.stdout
