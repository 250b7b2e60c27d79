"""AllReduce / AllGather bus-bandwidth sweep, 1 KiB … 1 GiB per rank (powers of 4), vs stock NCCL.

    torchrun --nproc-per-node N --master-addr 127.0.0.1 sweep.py [--colls allreduce,allgather]
             [--dtype bfloat16] [--min-bytes 1024] [--max-bytes 1073741824] [--iters 20] [--warmup 5]
             [--method hierarchy|constructive_trees] [--slices S] [--nvls auto|on|off] [--graph]
             [--check-max-bytes B] [--oneshot-max B] [--timeline]

Each point: the synthesized schedule through the sm_100a interpreter (heap
buffers, CUDA-event device time, max over ranks) and torch.distributed NCCL
on the same buffers.  ``--slices`` sets the slices per rank (S = M/slices);
``--nvls`` forces the NVLink-SHARP mapping on or off.  Up to
``--check-max-bytes`` per rank, each point first runs once on seeded inputs
and compares against an fp64 host reference.  busbw follows nccl-tests: AllReduce algbw·2(P−1)/P
with size M; AllGather algbw·(P−1)/P with size P·M.  Rank 0 prints one JSON
line per point and a final summary line.
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import time

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--colls", default="allreduce,allgather")
    ap.add_argument("--dtype", default="bfloat16")
    ap.add_argument("--min-bytes", type=int, default=1024)
    ap.add_argument("--max-bytes", type=int, default=1 << 30)
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--no-nccl", action="store_true")
    ap.add_argument("--graph", action="store_true", help="capture the timed launches in CUDA graphs (both impls)")
    ap.add_argument("--method", default="hierarchy", choices=("hierarchy", "constructive_trees"))
    ap.add_argument("--slices", type=int, default=None, help="slices per rank (default: P for AR, 1 for AG)")
    ap.add_argument("--nvls", default="auto", choices=("auto", "on", "off"))
    ap.add_argument("--check-max-bytes", type=int, default=1 << 24)
    ap.add_argument("--timeline", action="store_true",
                    help="record kernel entry/exit per interpreter launch and report durations and gaps")
    ap.add_argument("--oneshot-max", type=int, default=None,
                    help="largest per-rank payload of the one-shot path (0: always the interpreter)")
    ap.add_argument("--variants", default="",
                    help="';'-separated engine settings to compare in one run, each a ','-separated list of "
                         "NAME=VALUE (VERICCL_ prefix implied), e.g. 'MERGE=1;MERGE=0;MERGE=0,LANES=21'")
    args = ap.parse_args()
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world > 1:
        dist.init_process_group("cpu:gloo,cuda:nccl", device_id=torch.device("cuda", local))
    from vericcl_b200.models import CollectiveEngine
    from vericcl_b200.parallel import Communicator
    dtype = {"bfloat16": torch.bfloat16, "float32": torch.float32, "float16": torch.float16}[args.dtype]
    esize = torch.tensor([], dtype=dtype).element_size()
    heap = args.max_bytes * (world + 2) + (256 << 20)
    multicast = {"auto": world >= 4, "on": True, "off": False}[args.nvls]
    comm = Communicator(heap_bytes=heap, multicast=multicast)
    eng = CollectiveEngine(comm, method=args.method, slices_per_rank=args.slices, oneshot_max_bytes=args.oneshot_max)
    rank = comm.rank
    stream = torch.cuda.current_stream()

    host_us = [0.0]

    def timed(fn):
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize()
        graph = None
        if args.graph:
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                for _ in range(args.iters):
                    fn()
            graph.replay()
            torch.cuda.synchronize()
        comm.barrier()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record(stream)
        h0 = time.perf_counter()
        if graph is not None:
            graph.replay()
        else:
            for _ in range(args.iters):
                fn()
        host_us[0] = (time.perf_counter() - h0) / args.iters * 1e6
        e.record(stream)
        torch.cuda.synchronize()
        t = torch.tensor([s.elapsed_time(e) / args.iters * 1e3], dtype=torch.float64)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX, group=comm.control_group)
        return float(t.item())

    def seeded(r, count):
        g = torch.Generator().manual_seed(1234 + r)
        return torch.randn(count, generator=g, dtype=torch.float64)

    def check(coll, plan, count, inp, out, run=None):
        """One run on seeded N(0,1) inputs against an fp64 host reference; returns the max relative error."""
        mine = seeded(rank, count)
        inp.copy_(mine.to(dtype))
        torch.cuda.synchronize()
        comm.barrier()
        if run is None:
            comm.run(plan, inp, out)
        else:
            run()
        torch.cuda.synchronize()
        comm.check_status()
        if coll == "allreduce":
            want = sum(seeded(r, count).to(dtype).double() for r in range(world))
        else:
            want = torch.cat([seeded(r, count).to(dtype).double() for r in range(world)])
        got = out.double().cpu()
        return float((got - want).abs().max() / max(1e-12, float(want.abs().max())))

    results = []
    variants = [v for v in args.variants.split(";") if v.strip()] or [""]
    for variant in variants:
        settings = dict(kv.split("=", 1) for kv in variant.split(",") if kv.strip())
        for k, v in settings.items():
            os.environ["VERICCL_" + k.strip()] = v.strip()
        saved = (comm.lean, comm.bulk)
        if "LEAN" in settings:
            comm.lean = settings["LEAN"] not in ("0", "")
        if "BULK" in settings:
            from vericcl_b200.parallel.comm import _bulk_mode
            comm.bulk = _bulk_mode(settings["BULK"])
        run_sizes(args, variant, comm, eng, world, rank, dtype, esize, timed, check, host_us, results)
        comm.lean, comm.bulk = saved
        for k in settings:
            os.environ.pop("VERICCL_" + k.strip(), None)
    if rank == 0:
        print(json.dumps({"summary": True, "points": len(results)}), flush=True)
    comm.close()
    if world > 1:
        dist.destroy_process_group()


def run_sizes(args, variant, comm, eng, world, rank, dtype, esize, timed, check, host_us, results):
    size = args.min_bytes
    while size <= args.max_bytes:
        count = size // esize
        for coll in args.colls.split(","):
            if coll == "allreduce":
                buf = comm.empty(count, dtype)
                plan = eng.plan("allreduce", count, dtype, inplace=True)
                err = check(coll, plan, count, buf, buf) if size <= args.check_max_bytes else None
                buf.normal_()
                tl = comm.timeline_buffer() if args.timeline and plan.kind == "interp" else None
                ours = timed(lambda: comm.run(plan, buf, buf, timeline=tl))
                ours_host = host_us[0]
                gaps = comm.launch_gaps(tl, args.iters) if tl is not None else None
                comm.check_status()
                nccl = None if (args.no_nccl or world == 1) else timed(lambda: dist.all_reduce(buf))
                factor = 2.0 * (world - 1) / world if world > 1 else 1.0
                nbytes = size
                comm.free(buf)
            elif coll == "allgather_fp8":
                # the fused block-scaled fp8 AllGather; busbw counts the logical (input dtype) bytes
                inp = comm.empty(count, dtype)
                out = comm.empty(count * world, dtype)
                inp.normal_()
                err = None
                tl, gaps = None, None

                class _Fused:
                    kind, nlanes, niters, multicast = "fp8_fused", 0, 1, False
                plan = _Fused()
                ours = timed(lambda: eng.all_gather_fp8(inp, out))
                ours_host = host_us[0]
                comm.check_status()
                nccl = None if (args.no_nccl or world == 1) else timed(
                    lambda: dist.all_gather_into_tensor(out, inp))
                factor = (world - 1) / world if world > 1 else 1.0
                nbytes = size * world
                comm.free(inp)
                comm.free(out)
            else:
                inp = comm.empty(count, dtype)
                out = comm.empty(count * world, dtype)
                plan = eng.plan("allgather", count, dtype, inplace=False)
                push = eng.use_push(size)
                if push:
                    class _Push:
                        kind, nlanes, niters, multicast = "push", 0, 1, False
                    plan = _Push()
                    run = lambda: eng.all_gather(inp, out)          # noqa: E731
                else:
                    run = None
                err = check(coll, plan, count, inp, out, run) if size <= args.check_max_bytes else None
                inp.normal_()
                tl = comm.timeline_buffer() if args.timeline and plan.kind == "interp" else None
                ours = timed(run if push else (lambda: comm.run(plan, inp, out, timeline=tl)))
                ours_host = host_us[0]
                gaps = comm.launch_gaps(tl, args.iters) if tl is not None else None
                comm.check_status()
                nccl = None if (args.no_nccl or world == 1) else timed(
                    lambda: dist.all_gather_into_tensor(out, inp))
                factor = (world - 1) / world if world > 1 else 1.0
                nbytes = size * world
                comm.free(inp)
                comm.free(out)
            point = {"coll": coll, "n_gpus": world, "bytes_per_rank": size, "dtype": args.dtype, "graph": args.graph,
                     "time_us": round(ours, 3), "host_enqueue_us": round(ours_host, 2),
                     "busbw_gbs": round(nbytes / ours / 1e3 * factor, 2),
                     "path": plan.kind, "lanes": plan.nlanes, "iters": plan.niters, "nvls": plan.multicast,
                     "method": args.method,
                     "slices": eng.slices_per_rank or (1 if coll == "allgather" else world)}
            if err is not None:
                point["max_rel_err_vs_fp64"] = err
            if gaps is not None:
                point["kernel_us_median"] = gaps["kernel_us_median"]
                point["launch_gap_us_median"] = gaps["gap_us_median"]
            if nccl is not None:
                point.update({"nccl_time_us": round(nccl, 3),
                              "nccl_busbw_gbs": round(nbytes / nccl / 1e3 * factor, 2),
                              "speedup_vs_nccl": round(nccl / ours, 3)})
            if variant:
                point["variant"] = variant
            results.append(point)
            if rank == 0:
                print(json.dumps(point), flush=True)
        size *= 4


if __name__ == "__main__":
    main()
