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


NVLINK_MEASURED_GBS = 770.0      # peer copy per direction per GPU measured on B200s (900 nominal)


def nvlink_bytes(point) -> int | None:
    """Bytes the busier direction of one GPU's NVLink ports carries for this point's path."""
    p, m = point["n_gpus"], point["bytes_per_rank"]
    if p < 2:
        return None
    coll, kind, nvls = point["coll"], point.get("path", "interp"), bool(point.get("nvls"))
    if coll == "allreduce":
        if kind == "oneshot":
            return 2 * m * p if nvls else 2 * m * (p - 1)          # 16-byte lines carry 8 payload bytes
        return int(m * (1 + 1 / p)) if nvls else int(2 * m * (p - 1) / p)
    if coll == "allgather_fp8":
        esize = 4 if point.get("dtype") == "float32" else 2
        return int((p - 1) * (m // esize) * (1 + 4 / 128))
    if kind == "oneshot":
        return 2 * m * p if nvls else 2 * m * (p - 1)
    return m * p if nvls else m * (p - 1)                           # multicast stores also land on the sender


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
            elif doc.get("impl") == "reference" and "coll" in doc and "us" in doc:
                points.append(dict(doc, reference=True))
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
    if kind in ("push", "fp8_fused"):
        return {"push": "push", "fp8_fused": "fp8 fused"}[kind]
    return ("NVLS" if p.get("nvls") else "P2P") + (" %s" % p["method"] if p.get("method") not in (None, "hierarchy")
                                                   else "")


def report_rows(points) -> list:
    """One row per product point, with the reference library's time of the same (collective, GPUs, size)."""
    ref = {(p["coll"], p["ranks"], p["bytes_per_rank"]): p["us"] for p in points if p.get("reference")}
    rows = []
    mine = [p for p in points if not p.get("reference")]
    for p in sorted(mine, key=lambda d: (d["coll"], d["n_gpus"], bool(d.get("graph")), d.get("variant", ""),
                                         d["bytes_per_rank"])):
        link = nvlink_bytes(p)
        link_gbs = None if link is None else link / (p["time_us"] * 1e-6) / 1e9
        ref_us = ref.get((p["coll"], p["n_gpus"], p["bytes_per_rank"]))
        rows.append({"coll": p["coll"], "gpus": p["n_gpus"], "mode": "graph" if p.get("graph") else "eager",
                     "size": human_bytes(p["bytes_per_rank"]), "path": _path(p), "variant": p.get("variant", ""),
                     "time_us": p["time_us"], "busbw_gbs": p.get("busbw_gbs"), "nccl_us": p.get("nccl_time_us"),
                     "x_nccl": p.get("speedup_vs_nccl"), "ref_us": ref_us,
                     "x_ref": None if ref_us is None else round(ref_us / p["time_us"], 3),
                     "nvlink_gbs": None if link_gbs is None else round(link_gbs, 1),
                     "frac_770": None if link_gbs is None else round(link_gbs / NVLINK_MEASURED_GBS, 3),
                     "err": p.get("max_rel_err_vs_fp64")})
    return rows


def markdown(rows) -> str:
    head = ["coll", "GPUs", "mode", "bytes/rank", "path", "variant", "µs", "busbw GB/s", "NCCL 2.28 µs", "× NCCL",
            "ref 2.12 µs", "× ref", "NVLink GB/s/dir", "of 770", "fp64 rel err"]
    lines = ["| " + " | ".join(head) + " |", "|" + "---|" * len(head)]
    for r in rows:
        vals = [r["coll"], r["gpus"], r["mode"], r["size"], r["path"], r["variant"], r["time_us"], r["busbw_gbs"],
                r["nccl_us"], r["x_nccl"], r["ref_us"], r["x_ref"], r["nvlink_gbs"], r["frac_770"],
                "" if r["err"] is None else "%.1e" % r["err"]]
        lines.append("| " + " | ".join("" if v is None else str(v) for v in vals) + " |")
    return "\n".join(lines) + "\n"


def pivot(rows, *, variant: str = "") -> str:
    """× NCCL per (collective, GPUs, mode) row and message-size column, for one variant (default: the engine's
    default path, i.e. rows without a variant); cells below 1.0 are marked with an asterisk."""
    picked = [r for r in rows if r["variant"] == variant and r["x_nccl"] is not None]
    sizes = sorted({r["size"] for r in picked}, key=_size_bytes)
    keys = sorted({(r["coll"], r["gpus"], r["mode"]) for r in picked})
    cell = {(r["coll"], r["gpus"], r["mode"], r["size"]): r for r in picked}
    lines = ["| coll | GPUs | mode | " + " | ".join(sizes) + " |", "|" + "---|" * (3 + len(sizes))]
    behind = 0
    for key in keys:
        vals = []
        for size in sizes:
            r = cell.get(key + (size,))
            if r is None:
                vals.append("")
                continue
            x = r["x_nccl"]
            behind += x < 1.0
            vals.append(("%.2f" % x) + ("*" if x < 1.0 else ""))
        lines.append("| %s | %d | %s | " % key + " | ".join(vals) + " |")
    lines.append("")
    lines.append("%d of %d cells below 1.0 (marked *)" % (behind, len(cell)))
    return "\n".join(lines) + "\n"


def _size_bytes(text: str) -> int:
    number, unit = text.split()
    return int(number) * {"B": 1, "KiB": 1 << 10, "MiB": 1 << 20, "GiB": 1 << 30}[unit]


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
    r.add_argument("--pivot", action="store_true", help="× NCCL as a size × (collective, GPUs, mode) table")
    r.add_argument("--variant", default="", help="with --pivot: the variant to tabulate (default: none)")
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
    if args.pivot:
        sys.stdout.write(pivot(rows, variant=args.variant))
    elif args.markdown:
        sys.stdout.write(markdown(rows))
    else:
        for row in rows:
            print(json.dumps(row))
    return 0


if __name__ == "__main__":
    sys.exit(main())
