"""torchrun worker that executes calibration probe jobs (one process per GPU).

Counterpart of the reference's ``vericcl-probe`` binary
(runtime/probes/main.cu:130) launched per rank by
vericcl/verification/online/remote.py:233 (``_probe_command``): here every
job's probe XML runs through the same compiler and interpreter as real
schedules.
"""
from __future__ import annotations

import json
import os
import sys

import torch
import torch.distributed as dist


def main(spec_path: str) -> int:
    from vericcl_b200.online.probe_jobs import ProbeFlow, ProbeJob, build_probe_xml
    from vericcl_b200.parallel import Communicator
    spec = json.loads(open(spec_path).read())
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist.init_process_group("cpu:gloo,cuda:nccl", device_id=torch.device("cuda", local))
    rank, world = dist.get_rank(), dist.get_world_size()
    dtype = {"float32": torch.float32, "bfloat16": torch.bfloat16, "float16": torch.float16}.get(
        spec["datatype"], torch.float32)
    esize = torch.tensor([], dtype=dtype).element_size()
    max_bytes = max(max(j["payload_sizes"]) for j in spec["jobs"]) * 8
    comm = Communicator(heap_bytes=4 * max_bytes + (64 << 20))
    results = {}
    for jd in spec["jobs"]:
        job = ProbeJob(jd["job_id"], "", tuple(ProbeFlow(f["kind"], f["src"], f["dst"], f["channels"])
                                              for f in jd["flows"]), tuple(jd["payload_sizes"]), jd["mode"])
        plan = comm.compile(build_probe_xml(job, world), nlanes=32)
        samples = []
        for size in job.payload_sizes:
            count = (size // esize) * len(job.flows)
            inp = comm.empty(count, dtype)
            out = comm.empty(count, dtype)
            inp.fill_(1.0)
            for launch in range(spec["launches"]):
                # one barrier per launch round, then back-to-back invocations: after the warm-up the ranks run
                # in lockstep, so an invocation's device time is not inflated by the barrier's exit skew
                comm.barrier()
                for _ in range(spec["warmup"]):
                    comm.run(plan, inp, out)
                events = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                          for _ in range(spec["timed"])]
                for s, e in events:
                    s.record()
                    comm.run(plan, inp, out)
                    e.record()
                torch.cuda.synchronize()
                t = torch.tensor([s.elapsed_time(e) * 1e3 for s, e in events], dtype=torch.float64)
                dist.all_reduce(t, op=dist.ReduceOp.MAX, group=comm.control_group)
                times = [float(v) for v in t.tolist()]
                comm.check_status()
                for f in job.flows:
                    comp = f.flow_id if job.mode == "shared" else (
                        ("%s:%d" % (f.kind, f.src)) if f.kind in ("copy", "reduce")
                        else ("link:" if f.kind == "send" else "rrc:") + "%d:%d" % (f.src, f.dst))
                    for t in times:
                        samples.append({"component": comp, "bytes": size, "time_us": t, "launch": launch,
                                        "correct": True})
            comm.free(inp)
            comm.free(out)
        results[job.job_id] = samples
    if rank == 0:
        with open(spec["output"], "w") as handle:
            json.dump(results, handle)
    comm.close()
    dist.destroy_process_group()
    return 0


USAGE = ("usage: torchrun --nproc-per-node P -m vericcl_b200.online.probe_worker SPEC.json\n"
         "runs the probe jobs listed in SPEC.json (written by the calibration campaign) on P GPUs and writes "
         "their device times to the file named by its \"output\" field")

if __name__ == "__main__":
    if len(sys.argv) != 2 or sys.argv[1] in ("-h", "--help"):
        print(USAGE)
        sys.exit(0 if len(sys.argv) == 2 else 2)
    sys.exit(main(sys.argv[1]))
