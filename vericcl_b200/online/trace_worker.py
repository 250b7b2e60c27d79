"""Capture one traced invocation of a schedule on every rank and write the traces.

    torchrun --nproc-per-node P --master-addr 127.0.0.1 -m vericcl_b200.online.trace_worker \\
        --out DIR (--xml schedule.xml | --coll allreduce [--method hierarchy] [--slices S]) \\
        --bytes-per-rank B [--dtype bfloat16] [--nvls auto|on|off] [--lanes L] [--iters I]

Every rank warms the schedule up, brackets one traced launch with
host/%globaltimer clock samples and writes ``DIR/trace-rank<r>.bin`` (the
binary trace format of :mod:`vericcl_b200.online.trace`).  Rank 0 gathers the
records and clock maps and writes ``DIR/trace.json``: the causality report
(per-rank spans, slowest steps, dominant waits, cross-rank orders that the
clock uncertainty cannot resolve) plus a per-step timeline averaged over
lanes and iterations (start offset from the earliest step on any rank, wait
and duration), which is where a small message's latency goes.  The
reference captures the same per-step times from its patched MSCCL
(runtime/msccl-trace/include/vericcl_trace_format.h) and analyses them in
vericcl/verification/online/causality.py.
"""
from __future__ import annotations

import argparse
import json
import os
import sys
from collections import defaultdict
from pathlib import Path

import torch

OP_NAMES = {0: "nop", 1: "copy", 2: "reduce", 3: "mc_reduce", 4: "mc_store", 5: "mc_allreduce"}


def timeline(traces, clock_maps, origins=None):
    """Mean step times per (rank, step) in µs.

    A step "starts" when its waits are satisfied.  ``start_us`` is on the
    aligned host clock, from the earliest step start of any rank (its
    accuracy is the clock maps' uncertainty); ``local_start_us`` is on the
    rank's own GPU timer, from that rank's earliest step start (exact).
    ``wait_us`` is the time the step spent in its waits and ``duration_us``
    the time of its data work.
    """
    first = None
    local_first = {}
    for rank, recs in traces.items():
        for r in recs:
            t = clock_maps[rank].to_host(r.start_ns)
            first = t if first is None else min(first, t)
            local_first[rank] = min(local_first.get(rank, r.start_ns), r.start_ns)
    acc = defaultdict(lambda: [0.0, 0.0, 0.0, 0.0, 0, -1])
    for rank, recs in traces.items():
        cmap = clock_maps[rank]
        for r in recs:
            a = acc[(rank, r.block, r.step)]
            start = cmap.to_host(r.start_ns)
            a[0] += start - first
            a[1] += r.start_ns - local_first[rank]
            a[2] += r.wait_ns
            a[3] += cmap.to_host(r.end_ns) - start
            a[4] += 1
            a[5] = r.op
    rows = []
    for (rank, block, step), (s, ls, w, d, n, op) in sorted(acc.items()):
        row = {"rank": rank, "block": block, "step": step, "op": OP_NAMES.get(op, str(op)), "records": n,
               "start_us": round(s / n / 1e3, 3), "local_start_us": round(ls / n / 1e3, 3),
               "wait_us": round(w / n / 1e3, 3), "duration_us": round(d / n / 1e3, 3)}
        if origins is not None:
            tb, xml_step = origins[rank][block][step]
            row["xml_tb"], row["xml_step"] = tb, xml_step
        rows.append(row)
    return rows


def capture_schedule_trace(xml_path, ranks: int, bytes_per_rank: int, datatype: str, out_dir, *, lanes: int = 32,
                           port: int = 29633, timeout_s: float = 600.0) -> dict:
    """Run this worker under torchrun on ``ranks`` local GPUs for one schedule; summary of ``trace.json``."""
    import subprocess
    out_dir = Path(out_dir)
    root = Path(__file__).resolve().parents[2]
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=%d" % ranks,
           "--master-addr", "127.0.0.1", "--master-port", str(port), "-m", "vericcl_b200.online.trace_worker",
           "--out", str(out_dir), "--xml", str(xml_path), "--bytes-per-rank", str(bytes_per_rank),
           "--dtype", datatype, "--nvls", "off", "--lanes", str(lanes)]
    env = dict(os.environ, PYTHONPATH=str(root) + os.pathsep + os.environ.get("PYTHONPATH", ""))
    res = subprocess.run(cmd, env=env, cwd=str(root), capture_output=True, text=True, timeout=timeout_s)
    if res.returncode != 0 or not (out_dir / "trace.json").exists():
        return {"error": "trace capture failed (%d): %s" % (res.returncode, res.stderr[-500:])}
    report = json.loads((out_dir / "trace.json").read_text())
    return {"path": str(out_dir / "trace.json"), "global_span_us": report["global_span_us"],
            "tails": report["tails"][:3]}


def trace_report_for_xml(xml: str, request, out_dir, *, port: int = 29641) -> dict | None:
    """Trace one invocation of ``xml`` on the request's local GPUs; the ``trace.json`` report (None on failure)."""
    out_dir = Path(out_dir)
    out_dir.mkdir(parents=True, exist_ok=True)
    path = out_dir / "schedule.xml"
    path.write_text(xml)
    summary = capture_schedule_trace(path, request.rank_count, request.hyperparameters.total_size_bytes,
                                     request.collective.datatype, out_dir, port=port)
    if "error" in summary:
        return None
    return json.loads((out_dir / "trace.json").read_text())


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="vericcl_b200.online.trace_worker")
    ap.add_argument("--out", required=True)
    ap.add_argument("--xml", default=None)
    ap.add_argument("--coll", default="allreduce")
    ap.add_argument("--method", default="hierarchy")
    ap.add_argument("--slices", type=int, default=None)
    ap.add_argument("--bytes-per-rank", type=int, default=1 << 20)
    ap.add_argument("--dtype", default="bfloat16", choices=("bfloat16", "float32", "float16"))
    ap.add_argument("--nvls", default="auto", choices=("auto", "on", "off"))
    ap.add_argument("--lanes", type=int, default=None)
    ap.add_argument("--iters", type=int, default=None)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--steady", action="store_true",
                    help="trace a launch enqueued right behind the warm-up launches (no barrier before it)")
    ap.add_argument("--repeat", type=int, default=1,
                    help="captured launches; per-step counters accumulate over all of them")
    args = ap.parse_args(argv)

    import torch.distributed as dist
    from vericcl_b200.models import CollectiveEngine
    from vericcl_b200.online.trace import analyze_trace_causality, capture_once, step_counters, write_trace
    from vericcl_b200.parallel import Communicator
    local = int(os.environ.get("LOCAL_RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("cpu:gloo,cuda:nccl", device_id=torch.device("cuda", local))
    dtype = getattr(torch, args.dtype)
    esize = torch.tensor([], dtype=dtype).element_size()
    count = args.bytes_per_rank // esize
    multicast = {"auto": world >= 4, "on": True, "off": False}[args.nvls]
    coll = args.coll
    if args.xml:
        xml = Path(args.xml).read_text()
        import re
        found = re.search(r'coll="([a-z_]+)"', xml)
        coll = found.group(1) if found else coll
    out_count = count * world if coll == "allgather" else count
    comm = Communicator(heap_bytes=(count + out_count) * esize * 4 + (64 << 20), multicast=multicast)
    # traces record the interpreter's steps, so the one-shot path is off here
    eng = CollectiveEngine(comm, method=args.method, slices_per_rank=args.slices, oneshot_max_bytes=0)
    inplace = coll == "allreduce"
    if args.xml:
        lanes, iters = args.lanes or 1, args.iters or 1
        plan = comm.compile(xml, nlanes=lanes, niters=iters,
                            multicast=comm.multicast and coll in ("allreduce", "allgather"))
    else:
        plan = eng.plan(coll, count, dtype, inplace=inplace)
        if args.lanes or args.iters:
            plan = comm.compile(plan.xml, nlanes=args.lanes or plan.nlanes, niters=args.iters or plan.niters,
                                multicast=plan.multicast)
    inp = comm.empty(count, dtype)
    inp.normal_()
    out = inp if inplace else comm.empty(out_count, dtype)
    got = capture_once(comm, plan, inp, out, warmup=args.warmup, steady=args.steady)
    counted = list(got["records"])
    for _ in range(max(0, args.repeat - 1)):
        counted += capture_once(comm, plan, inp, out, warmup=0, steady=args.steady)["records"]
    outdir = Path(args.out)
    outdir.mkdir(parents=True, exist_ok=True)
    write_trace(outdir / ("trace-rank%d.bin" % comm.rank), comm.rank, plan.device_plan.nblocks * plan.nlanes,
                plan.device_plan.max_steps(), got["records"])
    origins = [[tuple(o) for o in blk] for blk in plan.device_plan.step_origins()]
    counters = [dict(rank=k[0], block=k[1], step=k[2], **v) for k, v in sorted(step_counters(counted).items())]
    gathered = comm.all_gather_object({"rank": comm.rank, "records": got["records"], "clock": got["clock"],
                                       "origins": origins, "counters": counters})
    if comm.rank == 0:
        traces = {g["rank"]: g["records"] for g in gathered}
        clocks = {g["rank"]: g["clock"] for g in gathered}
        step_origins = {g["rank"]: g["origins"] for g in gathered}
        report = analyze_trace_causality(traces, clocks)
        report.update({"collective": coll, "ranks": world, "bytes_per_rank": args.bytes_per_rank,
                       "steady": args.steady,
                       "dtype": args.dtype, "lanes": plan.nlanes, "iters": plan.niters, "nvls": plan.multicast,
                       "clock_uncertainty_us": {r: round(c.uncertainty_ns / 1e3, 3) for r, c in clocks.items()},
                       "timeline": timeline(traces, clocks, step_origins),
                       "launches_counted": max(1, args.repeat),
                       "counters": [c for g in gathered for c in g["counters"]]})
        (outdir / "trace.json").write_text(json.dumps(report, indent=1, default=str))
        print(json.dumps({"trace": str(outdir / "trace.json"), "global_span_us": report["global_span_us"],
                          "records": sum(len(v) for v in traces.values())}))
    comm.close()
    if world > 1:
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
