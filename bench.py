"""Gradient-bucket AllReduce benchmark (the flagship data-parallel step).

Workload: an 8B-parameter model's bf16 gradients (16 GB per rank) in 25 MiB
buckets with a fused 1/8 scale, one synthesized AllReduce schedule replayed
for every bucket by the sm_100a interpreter over NVLink/NVSwitch.  Data is
synthetic N(0, 0.02).  One step = one full gradient sync.

Launch: ``python bench.py`` (1 GPU) or ``torchrun --nproc-per-node N bench.py
--gpus N``.  Timing: W untimed warm-up steps, then K steps bracketed by a
barrier and a device synchronize, measured with CUDA events on the launching
stream; the reported time is the max over ranks.  The 16 GB buffer is larger
than the 126 MB L2, so no flush is needed between steps.

Units.  ``busbw_per_gpu_gbs`` is the nccl-tests bus bandwidth of one GPU
(2(P-1)/P × bytes / time).  ``value`` is the whole-job aggregate: that figure
summed over the N GPUs.  With one GPU an AllReduce moves nothing between GPUs;
the bytes are then counted once and the figure is the rate of the in-place
scale pass (an HBM read and write), labelled as such.  ``nvlink`` gives the
bytes each GPU really sends per direction on the path the plan takes and
their fraction of 900 GB/s (nominal) and 770 GB/s (measured peer copy).

``cta_budget`` times the same sync on 16, 32, 64 and 148 CTAs per GPU
(``--cta-budgets``) beside the default (32 CTAs on an NVLS plan, every SM
otherwise): in data-parallel training the SMs the sync leaves free are what
the overlapping backward pass gets.

``--impl reference`` runs the reference's own MSCCL/NCCL 2.12.12 build instead
(``baseline/reference_arm.py``), without PyTorch or this package.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "AllGather/AllReduce bus GB/s vs size at 2/4/8 B200 vs ref MSCCL/NCCL; % of 900GB/s"
MODEL = "gradient-bucket AllReduce: 8B-param bf16 gradients (16 GB/rank), 25 MiB buckets, fused scale 1/8"


def parse():
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=("vericcl", "reference"), default="vericcl")
    ap.add_argument("--params", type=int, default=8_000_000_000)
    ap.add_argument("--bucket-bytes", type=int, default=25 * 1024 * 1024)
    ap.add_argument("--scale", type=float, default=0.125)
    ap.add_argument("--e2e-steps", type=int, default=2)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-nccl", action="store_true")
    ap.add_argument("--per-bucket", action="store_true", help="one launch per bucket instead of one batched launch")
    ap.add_argument("--slices", type=int, default=None, help="slices per rank of the synthesized schedule")
    ap.add_argument("--cta-budgets", default="16,32,64,148",
                    help="also time the sync restricted to these CTAs per GPU (comma list; empty: skip)")
    return ap.parse_args()


class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, devices, enabled=True):
        self.enabled = enabled
        # nvidia-smi numbers GPUs physically; map CUDA ordinals through CUDA_VISIBLE_DEVICES when it lists indices
        visible = [v.strip() for v in os.environ.get("CUDA_VISIBLE_DEVICES", "").split(",") if v.strip()]
        if visible and all(v.isdigit() for v in visible):
            devices = [int(visible[d]) for d in devices if d < len(visible)]
        self.devices = devices
        self.proc = None
        self.path = os.path.join("/tmp", "vb_clocks_%d.csv" % os.getpid())

    def __enter__(self):
        if not self.enabled:
            return self
        try:
            self.out = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", "--query-gpu=" + self.FIELDS, "--format=csv,noheader,nounits",
                                          "-i", ",".join(str(d) for d in self.devices), "-lms", "100"],
                                         stdout=self.out, stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
            return self
        # start timing only once the sampler is producing lines, so the samples cover the timed region
        deadline = time.monotonic() + 10.0
        while time.monotonic() < deadline and self.proc.poll() is None:
            self.out.flush()
            if os.path.getsize(self.path) > 0:
                break
            time.sleep(0.05)
        self.started = time.monotonic()
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            # keep sampling until at least 0.3 s have passed so short timed regions still get samples
            while time.monotonic() - getattr(self, "started", 0.0) < 0.3:
                time.sleep(0.05)
            self.proc.terminate()
            try:
                self.proc.wait(5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.out.close()

    def summary(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        sm, mx, reasons = [], [], set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        with open(self.path) as f:
            for line in f:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) < 9 or not parts[0].isdigit() or int(parts[0]) not in self.devices:
                    continue
                try:
                    sm.append(float(parts[1]))
                    mx.append(float(parts[2]))
                except ValueError:
                    continue
                for name, value in zip(names, parts[5:9]):
                    if value.lower() == "active":
                        reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm)}


def timed(fn, steps, stream, barrier):
    """Device time of ``steps`` calls of ``fn`` on ``stream`` (ms per call), bracketed by barriers."""
    import torch
    barrier()
    torch.cuda.synchronize()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for _ in range(steps):
        fn()
    t1.record(stream)
    torch.cuda.synchronize()
    barrier()
    return t0.elapsed_time(t1) / steps


def main():
    args = parse()
    if args.impl == "reference":
        sys.path.insert(0, os.path.join(ROOT, "baseline"))
        import reference_arm
        return reference_arm.run(args, ClockSampler, METRIC, MODEL)
    import torch
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world != args.gpus:
        raise SystemExit("--gpus %d but WORLD_SIZE=%d (launch N>1 with torchrun)" % (args.gpus, world))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    import torch.distributed as dist
    from datetime import timedelta
    if world > 1:
        dist.init_process_group("cpu:gloo,cuda:nccl", timeout=timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    rank = dist.get_rank() if world > 1 else 0
    from vericcl_b200.models import GradBucketAllReduce
    from vericcl_b200.parallel import Communicator
    dtype = torch.bfloat16
    esize = 2
    total_bytes = args.params * esize
    heap = total_bytes + 2 * args.bucket_bytes + (256 << 20)
    nvls = os.environ.get("VERICCL_NVLS")
    multicast = (world >= 4) if nvls is None else nvls not in ("0", "")
    comm = Communicator(heap_bytes=heap, timeout_s=20.0, multicast=multicast)
    ar = GradBucketAllReduce(comm, args.params, dtype=dtype, bucket_bytes=args.bucket_bytes, scale=args.scale,
                             slices_per_rank=args.slices)
    gen = torch.Generator(device="cuda").manual_seed(1234 + rank)
    flat = ar.flat
    step = 1 << 28
    for lo in range(0, flat.numel(), step):
        part = flat[lo:lo + step]
        part.copy_(torch.randn(part.numel(), generator=gen, device="cuda", dtype=torch.float32).mul_(0.02))
    stream = torch.cuda.current_stream()
    batched = not args.per_bucket

    def barrier():
        if world > 1:
            comm.barrier()

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=comm.control_group)
        return float(t.item())

    # correctness of the first and last bucket of one full sync against an fp32 sum of every rank's data, untimed
    first, last = ar.bucket(0), ar.bucket(ar.buckets - 1)
    saved = [first.clone(), last.clone()]
    ar.sync(stream, batched=batched)
    torch.cuda.synchronize()
    comm.check_status()
    err, tol_fail = 0.0, False
    for got, ref in zip((first, last), saved):
        ref = ref.float()
        if world > 1:
            dist.all_reduce(ref)
        ref.mul_(args.scale)
        e = (got.float() - ref).abs().max().item()
        err = max(err, e)
        tol_fail |= e > 2e-2 * max(1e-6, ref.abs().max().item())
    check_ok = max_over_ranks(1.0 if tol_fail else 0.0) == 0.0
    del saved

    for _ in range(args.warmup):
        ar.sync(stream, batched=batched)
    torch.cuda.synchronize()
    comm.check_status()
    with ClockSampler([local] if world == 1 else list(range(world)), enabled=rank == 0) as clocks:
        ms = timed(lambda: ar.sync(stream, batched=batched), args.steps, stream, barrier)
    ms = max_over_ranks(ms)
    comm.check_status()
    clock_info = clocks.summary() if rank == 0 else None
    bus = ar.bus_bytes_per_rank()
    busbw = bus / (ms * 1e-3) / 1e9
    value = busbw * world
    launches = args.steps * (ar.buckets if args.per_bucket else ar.launches_per_sync)
    link_bytes = ar.nvlink_bytes_per_rank()
    link_gbs = link_bytes / (ms * 1e-3) / 1e9
    nvlink = {"bytes_per_gpu_per_direction": int(link_bytes), "gbs_per_direction": round(link_gbs, 2),
              "pct_of_900_nominal": round(100 * link_gbs / 900.0, 2),
              "pct_of_770_measured_peer_copy": round(100 * link_gbs / 770.0, 2),
              "path": ("none (one GPU)" if world == 1 else
                       "NVLS multimem.ld_reduce + multimem.st: (1+1/P) x bytes each way" if ar.plan.multicast else
                       "peer pulls (reduce-scatter + all-gather): 2(P-1)/P x bytes each way")}

    # the same product API with one launch per bucket (how data-parallel training fires buckets as they fill)
    other = None
    if world > 1 and not args.no_nccl:
        alt = not batched
        for _ in range(2):
            ar.sync(stream, batched=alt)
        oms = max_over_ranks(timed(lambda: ar.sync(stream, batched=alt), max(2, args.steps // 4), stream, barrier))
        comm.check_status()
        other = {"mode": "batched" if alt else "per-bucket", "ms_per_step": round(oms, 4),
                 "busbw_per_gpu_gbs": round(bus / (oms * 1e-3) / 1e9, 2),
                 "launches_per_step": ar.launches_per_sync if alt else ar.buckets}

    # the same sync on a CTA budget: the SMs left over are what overlapping backward compute gets
    budgets = None
    if args.cta_budgets:
        budgets = {"default": {"ctas": ar.ctas_of(ar.plan), "ms_per_step": round(ms, 4),
                            "busbw_per_gpu_gbs": round(busbw, 2)}}
        for want in [int(v) for v in args.cta_budgets.split(",") if v.strip()]:
            bplan = ar.plan_with_budget(want)
            for _ in range(2):
                ar.sync(stream, batched=batched, plan=bplan)
            bms = max_over_ranks(timed(lambda: ar.sync(stream, batched=batched, plan=bplan),
                                       max(2, args.steps // 4), stream, barrier))
            comm.check_status()
            budgets[str(want)] = {"ctas": ar.ctas_of(bplan), "sms_free": max(0, 148 - ar.ctas_of(bplan)),
                                  "ms_per_step": round(bms, 4), "busbw_per_gpu_gbs": round(bus / (bms * 1e-3) / 1e9, 2)}
            del bplan

    nccl = None
    if world > 1 and not args.no_nccl:
        premul = dist._make_nccl_premul_sum(args.scale)
        bufs = [ar.bucket(i) for i in range(ar.buckets)]
        flat_all = ar.grads

        def per_bucket():
            for b in bufs:
                dist.all_reduce(b, op=premul)

        def grouped():
            with dist._coalescing_manager(device=torch.device("cuda", local)):
                for b in bufs:
                    dist.all_reduce(b, op=premul)

        def flat_call():
            dist.all_reduce(flat_all, op=premul)

        nccl = {"library": "torch %s, NCCL %s" % (torch.__version__, ".".join(map(str, torch.cuda.nccl.version()))),
                "op": "ncclAllReduce PREMUL_SUM (scale fused)"}
        for name, fn in (("per_bucket", per_bucket), ("per_bucket_grouped", grouped), ("flat_16GB", flat_call)):
            try:
                for _ in range(max(1, min(2, args.warmup))):
                    fn()
                torch.cuda.synchronize()
                nms = max_over_ranks(timed(fn, max(2, args.steps // 4), stream, barrier))
                nccl[name] = {"ms_per_step": round(nms, 4), "busbw_per_gpu_gbs": round(bus / (nms * 1e-3) / 1e9, 2)}
            except Exception as e:     # a comparator that fails does not void the product's line
                nccl[name] = {"error": str(e)[:200]}

    e2e = None
    if not args.no_e2e:
        host = None
        try:
            host = torch.empty(flat.numel(), dtype=dtype, pin_memory=True)
            host.copy_(flat)
        except RuntimeError:
            host = None
        if host is not None:
            out_host = torch.empty(32768, dtype=dtype, pin_memory=True)

            def e2e_step():
                # host->device copies of bucket groups overlapped with the AllReduce of the groups already in
                ar.sync_from_host(host, stream)
                out_host.copy_(ar.grads[:32768], non_blocking=True)
                stream.synchronize()
                _ = float(out_host[0])

            def e2e_serial():
                flat.copy_(host, non_blocking=True)
                ar.sync(stream, batched=batched)
                out_host.copy_(ar.grads[:32768], non_blocking=True)
                stream.synchronize()
                _ = float(out_host[0])

            e2e_step()
            ems = max_over_ranks(timed(e2e_step, args.e2e_steps, stream, barrier))
            e2e_serial()
            sms = max_over_ranks(timed(e2e_serial, args.e2e_steps, stream, barrier))
            e2e = {"value": round(bus / (ems * 1e-3) / 1e9 * world, 2),
                   "unit": "GB/s (sum over GPUs of per-GPU bus bandwidth)",
                   "ms_per_step": round(ems, 3), "h2d_bytes_per_step": int(total_bytes),
                   "d2h_bytes_per_step": int(out_host.numel() * esize),
                   "api": "GradBucketAllReduce.sync_from_host: pinned host->device copies of 8 bucket groups "
                          "overlapped with the AllReduce of the groups already copied, then a device->host read",
                   "serial": {"ms_per_step": round(sms, 3), "value": round(bus / (sms * 1e-3) / 1e9 * world, 2),
                              "api": "one host->device copy of all gradients, then GradBucketAllReduce.sync"}}
            del host
    if rank == 0:
        line = {"metric": METRIC, "value": round(value, 2), "unit": "GB/s (sum over GPUs of per-GPU bus bandwidth)",
                "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "bf16", "data": "synthetic N(0,0.02) gradients, random init",
                "impl": "vericcl_b200",
                "config": {"model": MODEL, "global_batch": None, "seq_len": None,
                           "parallelism": "dp%d" % world, "bucket_bytes": args.bucket_bytes,
                           "buckets": ar.buckets, "bytes_per_rank": total_bytes, "scale": args.scale,
                           "schedule": "synthesized AllReduce (hierarchy/direct) replayed per bucket",
                           "launch": "per-bucket" if args.per_bucket else "all buckets in one persistent launch",
                           "plan": {"lanes": ar.plan.nlanes, "iters": ar.plan.niters,
                                    "nvls": bool(ar.plan.multicast), "heap_multicast": comm.multicast,
                                    "instance": ("one-shot" if ar.plan.kind == "oneshot" else
                                                 {0: "register-lean vector loads (L2 prefetch hint)" if comm.lean
                                                  else "vector loads", 1: "TMA-staged loads",
                                                  3: "TMA loads + stores"}[
                                                     comm.bulk_for(ar.plan, ar.bucket_elems * esize)]),
                                    "stats": ar.plan.device_plan.stats() if ar.plan.device_plan is not None
                                    else {"path": ar.plan.kind}},
                           "l2": "inputs (16 GB) larger than the 126 MB L2; no flush needed"},
                "busbw_per_gpu_gbs": round(busbw, 2),
                "busbw_note": ("one GPU: no inter-GPU traffic; bytes counted once, i.e. the in-place scale pass "
                               "rate (HBM read + write)") if world == 1 else "nccl-tests bus bandwidth, 2(P-1)/P",
                "nvlink": nvlink, "other_launch_mode": other, "cta_budget": budgets,
                "check": {"first_last_bucket_max_err": err, "ok": bool(check_ok),
                          "reference": "fp32 sum over ranks (torch) x scale"},
                "clocks": clock_info, "e2e": e2e, "gpu_launches": launches, "nccl": nccl}
        print(json.dumps(line), flush=True)
    comm.close()
    if world > 1:
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
