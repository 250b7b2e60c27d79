"""Probe executor that runs calibration jobs on the local GPUs.

All jobs of a campaign run in one ``torchrun`` job (one process per GPU of
``runtime.rank_map``) through the same compiler and interpreter as real
schedules: every job's probe XML is compiled and launched for each payload
size, for ``launches`` rounds of ``timed_iterations`` device-timed
iterations after ``warmup_iterations``; the time of an iteration is the max
over ranks.  The child runs as an owned process group with the calibration
job deadline.  Returns ``None`` when no GPU is visible, so the workflow
records calibration as skipped (reference counterpart:
vericcl/verification/online/remote.py:442, ``NativeProbeDriver``).
"""
from __future__ import annotations

import json
import os
import sys
import tempfile
from pathlib import Path

from vericcl_b200.errors import RuntimeFailure
from vericcl_b200.execution.processes import run_owned_process
from vericcl_b200.online.fitting import Sample
from vericcl_b200.online.probe_jobs import plan_probes


def native_probe_executor(request):
    try:
        import torch
        gpus = torch.cuda.device_count()
    except Exception:
        gpus = 0
    if gpus < request.rank_count:
        return None
    cache = {}

    def run(job):
        if not cache:
            cache.update(_run_all(request))
        if job.job_id not in cache:
            raise RuntimeFailure("probe %s produced no samples" % job.job_id)
        return cache[job.job_id]
    return run


def _run_all(request):
    from vericcl_b200.topology import load_topology
    cfg = request.request_config["sketch"]["calibration"]
    jobs = plan_probes(request, load_topology(request))
    with tempfile.TemporaryDirectory() as tmp:
        spec = Path(tmp) / "jobs.json"
        out = Path(tmp) / "samples.json"
        spec.write_text(json.dumps({"jobs": [j.as_json() for j in jobs], "warmup": cfg["warmup_iterations"],
                                    "timed": cfg["timed_iterations"], "launches": min(cfg["launches"], 4),
                                    "datatype": request.collective.datatype, "output": str(out)}))
        root = Path(__file__).resolve().parents[2]
        cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
               "--nproc-per-node=%d" % request.rank_count, "--master-addr", "127.0.0.1", "--master-port", "29621",
               "-m", "vericcl_b200.online.probe_worker", str(spec)]
        extra = {str(k): str(v) for k, v in (request.request_config["runtime"].get("environment") or {}).items()}
        env = dict(os.environ, **extra, PYTHONPATH=str(root) + os.pathsep + os.environ.get("PYTHONPATH", ""))
        res = run_owned_process(cmd, timeout_s=float(cfg["job_timeout_s"]), env=env, cwd=str(root))
        if res.returncode != 0 or not out.exists():
            raise RuntimeFailure("probe job failed (%s): %s" % (res.returncode, res.stderr[-2000:]))
        data = json.loads(out.read_text())
    samples = {}
    for job_id, items in data.items():
        samples[job_id] = [Sample(i["component"], i["bytes"], i["time_us"], "native_interpreter", i["launch"],
                                  i["correct"]) for i in items]
    return samples
