"""Experiment matrix and report tables for size sweeps.

    python -m vericcl_b200.experiments matrix --gpus 2,4,8 [--colls allreduce,allgather] [--graph]
    python -m vericcl_b200.experiments report SWEEP_OUTPUT [SWEEP_OUTPUT ...] [--markdown]
    python -m vericcl_b200.experiments overhead {solve,replay} --inputs DIR ... --out FILE

``matrix`` prints the ``torchrun … sweep.py`` command of every (GPU count,
mode) cell of a message-size experiment (1 KiB … 1 GiB per rank, powers of
4, against NCCL on the same buffers).  ``report`` reads the JSON lines those
runs print (other lines are ignored) and tabulates, per collective, GPU
count and size: time, bus bandwidth, the path that ran (one-shot or
interpreter, NVLS or peer pulls), NCCL's time and the speedup, and the fp64
check error (reference counterpart: vericcl/experiments/v100.py:929 and
vericcl/experiments/report.py).  ``overhead`` attributes the synthesis
pipeline's wall clock to its phases (``vericcl_b200/overhead.py``).
"""
from __future__ import annotations

import argparse
import json
import sys
from pathlib import Path


def matrix_commands(gpus, *, colls: str = "allreduce,allgather", graph: bool = False, max_bytes: int = 1 << 30,
                    port: int = 29500) -> list:
    out = []
    for i, n in enumerate(gpus):
        cmd = ["python", "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=%d" % n,
               "--master-addr", "127.0.0.1", "--master-port", str(port + i), "sweep.py", "--colls", colls,
               "--max-bytes", str(max_bytes)]
        if graph:
            cmd.append("--graph")
        out.append(cmd)
    return out


def load_points(paths) -> list:
    points = []
    for path in paths:
        for line in Path(path).read_text().splitlines():
            line = line.strip()
            if not line.startswith("{"):
                continue
            try:
                doc = json.loads(line)
            except json.JSONDecodeError:
                continue
            if "coll" in doc and "bytes_per_rank" in doc and "time_us" in doc:
                points.append(doc)
    return points


def human_bytes(n: int) -> str:
    for unit, name in ((1 << 30, "GiB"), (1 << 20, "MiB"), (1 << 10, "KiB")):
        if n >= unit and n % unit == 0:
            return "%d %s" % (n // unit, name)
    return "%d B" % n


def _path(p) -> str:
    kind = p.get("path", "interp")
    if kind == "oneshot":
        return "one-shot" + (" NVLS" if p.get("nvls") else "")
    return ("NVLS" if p.get("nvls") else "P2P") + (" %s" % p["method"] if p.get("method") not in (None, "hierarchy")
                                                   else "")


def report_rows(points) -> list:
    rows = []
    for p in sorted(points, key=lambda d: (d["coll"], d["n_gpus"], bool(d.get("graph")), d["bytes_per_rank"])):
        rows.append({"coll": p["coll"], "gpus": p["n_gpus"], "mode": "graph" if p.get("graph") else "eager",
                     "size": human_bytes(p["bytes_per_rank"]), "path": _path(p), "time_us": p["time_us"],
                     "busbw_gbs": p.get("busbw_gbs"), "nccl_us": p.get("nccl_time_us"),
                     "x_nccl": p.get("speedup_vs_nccl"), "err": p.get("max_rel_err_vs_fp64")})
    return rows


def markdown(rows) -> str:
    head = ["coll", "GPUs", "mode", "bytes/rank", "path", "µs", "busbw GB/s", "NCCL µs", "× NCCL", "fp64 rel err"]
    lines = ["| " + " | ".join(head) + " |", "|" + "---|" * len(head)]
    for r in rows:
        vals = [r["coll"], r["gpus"], r["mode"], r["size"], r["path"], r["time_us"], r["busbw_gbs"], r["nccl_us"],
                r["x_nccl"], "" if r["err"] is None else "%.1e" % r["err"]]
        lines.append("| " + " | ".join("" if v is None else str(v) for v in vals) + " |")
    return "\n".join(lines) + "\n"


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="vericcl_b200.experiments")
    sub = ap.add_subparsers(dest="command", required=True)
    m = sub.add_parser("matrix")
    m.add_argument("--gpus", default="2,4,8")
    m.add_argument("--colls", default="allreduce,allgather")
    m.add_argument("--graph", action="store_true")
    m.add_argument("--max-bytes", type=int, default=1 << 30)
    r = sub.add_parser("report")
    r.add_argument("files", nargs="+")
    r.add_argument("--markdown", action="store_true")
    from vericcl_b200 import overhead
    overhead.add_arguments(sub.add_parser("overhead", help="pipeline wall-clock attribution or schedule replay"))
    args = ap.parse_args(argv)
    if args.command == "overhead":
        return overhead.run(args)
    if args.command == "matrix":
        for cmd in matrix_commands([int(g) for g in args.gpus.split(",")], colls=args.colls, graph=args.graph,
                                   max_bytes=args.max_bytes):
            print(" ".join(cmd))
        return 0
    rows = report_rows(load_points(args.files))
    if args.markdown:
        sys.stdout.write(markdown(rows))
    else:
        for row in rows:
            print(json.dumps(row))
    return 0


if __name__ == "__main__":
    sys.exit(main())
