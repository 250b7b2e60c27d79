"""The reference arm's contract on the host: one JSON line with ``impl: reference``, and the multi-GPU runs
report why they are unavailable instead of starting the reference library."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "baseline"))


def test_multi_gpu_runs_print_the_unavailable_line():
    env = dict(os.environ, WORLD_SIZE="2", RANK="0", LOCAL_RANK="0", MASTER_ADDR="127.0.0.1", MASTER_PORT="29999")
    proc = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--gpus", "2",
                           "--steps", "3", "--warmup", "3"], cwd=ROOT, env=env, capture_output=True, text=True,
                          timeout=120)
    assert proc.returncode == 0, proc.stderr[-2000:]
    line = json.loads(proc.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference" and "hung" in line["unavailable"]


def test_other_ranks_print_nothing():
    env = dict(os.environ, WORLD_SIZE="2", RANK="1", LOCAL_RANK="1", MASTER_ADDR="127.0.0.1", MASTER_PORT="29999")
    proc = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--gpus", "2"],
                          cwd=ROOT, env=env, capture_output=True, text=True, timeout=120)
    assert proc.returncode == 0 and proc.stdout.strip() == ""


def test_unavailable_reason_by_world_size():
    import reference_arm
    assert reference_arm.unavailable_reason(2) == reference_arm.MULTI_GPU_HANG
    assert reference_arm.unavailable_reason(8) == reference_arm.MULTI_GPU_HANG
    one = reference_arm.unavailable_reason(1)
    # one GPU: runnable when the library is built, else the build outcome
    assert one is None or "reference" in one


def test_bf16_round_trip_matches_torch():
    import numpy as np
    import torch
    import reference_arm
    x = np.random.default_rng(3).standard_normal(4096).astype(np.float32)
    bits = reference_arm.bf16_bits(x)
    ref = torch.from_numpy(x).to(torch.bfloat16).view(torch.int16).numpy().astype(np.uint16)
    assert np.array_equal(bits, ref)
    assert np.array_equal(reference_arm.bf16_to_f32(bits), torch.from_numpy(x).to(torch.bfloat16).float().numpy())


def test_bench_and_sweep_command_lines():
    """The driver's contract flags exist (bench: --gpus --steps --warmup --impl; sweep: sizes and variants)."""
    out = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--help"], cwd=ROOT, capture_output=True,
                         text=True, timeout=120)
    assert out.returncode == 0
    for flag in ("--gpus", "--steps", "--warmup", "--impl", "--cta-budgets", "--e2e-steps", "--per-bucket"):
        assert flag in out.stdout, flag
    out = subprocess.run([sys.executable, os.path.join(ROOT, "sweep.py"), "--help"], cwd=ROOT, capture_output=True,
                         text=True, timeout=120)
    assert out.returncode == 0 and "--variants" in out.stdout and "--graph" in out.stdout
