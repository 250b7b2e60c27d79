"""Schedule experiment matrix: plan, solve, benchmark and summarize, resumable.

    python -m vericcl_b200.experiment_matrix plan --out exp --groups 1,2 --per-group 4 \\
        --colls allgather,allreduce --sizes 4m,16m,64m [--inter-gbps 25]
    python -m vericcl_b200.experiment_matrix solve --manifest exp/manifest.json [--resume] [--case ID ...]
    python -m vericcl_b200.experiment_matrix benchmark --manifest exp/manifest.json [--resume]
    python -m vericcl_b200.experiment_matrix summarize --manifest exp/manifest.json [--markdown]

``plan`` writes a manifest of cases (collective × topology × size per rank)
and each case's four request documents: one NVSwitch group of ``per-group``
ranks, or ``groups`` of them joined by an emulated slow link.  ``solve``
synthesizes every case through the CLI (``python -m vericcl_b200 solve``)
into ``<exp>/runs``; ``benchmark`` measures each solved schedule on the
local GPUs through the native driver (device time, slowest rank per
invocation; multi-group cases with the inter-group link emulated).  Every
task records its status, the sha256 of its inputs and of its output in
``state.json``; ``--resume`` skips a task whose record passed and whose
input and output digests still match (reference:
vericcl/experiments/v100.py:929-1420, whose stages and resumable task
records this follows for one B200 node instead of two V100 nodes).
"""
from __future__ import annotations

import argparse
import hashlib
import json
import os
import sys
import time
from pathlib import Path

from vericcl_b200.utils.jsonio import atomic_write_json, strict_load

UNITS = {"k": 1 << 10, "m": 1 << 20, "g": 1 << 30}


def parse_size(text: str) -> int:
    text = text.strip().lower()
    if text[-1:] in UNITS:
        return int(float(text[:-1]) * UNITS[text[-1]])
    return int(text)


def _sha(path) -> str:
    return hashlib.sha256(Path(path).read_bytes()).hexdigest()


def _inputs_sha(case_dir: Path) -> str:
    h = hashlib.sha256()
    for name in ("topology", "sketch", "atom", "runtime"):
        h.update((case_dir / (name + ".json")).read_bytes())
    return h.hexdigest()


class StateStore:
    """Task records keyed by task id, written atomically after every task."""

    def __init__(self, path):
        self.path = Path(path)

    def load(self) -> dict:
        return strict_load(self.path) if self.path.exists() else {}

    def put(self, task_id: str, record: dict) -> None:
        state = self.load()
        state[task_id] = record
        atomic_write_json(self.path, state)


def plan_matrix(out, *, groups=(1, 2), per_group: int = 4, colls=("allgather", "allreduce"), sizes=(4 << 20,),
                inter_gbps: float = 25.0, datatype: str = "float32", slices: int = 4) -> dict:
    from vericcl_b200.examples import example_documents, write_documents
    from vericcl_b200.topology.nvswitch import multinode_topology, nvswitch_topology
    out = Path(out)
    cases = []
    for g in groups:
        ranks = g * per_group
        topo_name = "nvswitch-x%d" % ranks if g == 1 else "emulated-%dx%d-%ggbps" % (g, per_group, inter_gbps)
        for coll in colls:
            for size in sizes:
                topo = nvswitch_topology(ranks) if g == 1 else multinode_topology(g, per_group,
                                                                                 inter_gbps=inter_gbps)
                unit = slices * (ranks if coll in ("reduce_scatter", "alltoall") else 1)
                slice_bytes = size // unit
                docs = example_documents(coll, "hierarchy", ranks, total_size_bytes=size,
                                         slice_size_bytes=slice_bytes, datatype=datatype, topology=topo,
                                         calibration=False, scratch_bytes=max(1 << 30, 4 * size))
                case_id = "%s-%s-%d" % (coll, topo_name, size)
                case_dir = out / "cases" / case_id
                write_documents(case_dir, docs)
                cases.append({"id": case_id, "collective": coll, "groups": g, "per_group": per_group,
                              "ranks": ranks, "bytes_per_rank": size, "datatype": datatype,
                              "inter_gbps": inter_gbps if g > 1 else None,
                              "documents": str(case_dir.relative_to(out))})
    manifest = {"version": 1, "created_utc": time.strftime("%Y-%m-%dT%H:%M:%SZ", time.gmtime()), "cases": cases}
    atomic_write_json(out / "manifest.json", manifest)
    return manifest


def _load(manifest_path):
    manifest_path = Path(manifest_path)
    return manifest_path.parent, strict_load(manifest_path)


def _select(manifest, ids):
    cases = manifest["cases"]
    if ids:
        known = {c["id"] for c in cases}
        unknown = sorted(set(ids) - known)
        if unknown:
            raise ValueError("unknown case ids: %s" % unknown)
        cases = [c for c in cases if c["id"] in ids]
    return cases


def _reusable(record, inputs_sha, output) -> bool:
    return bool(record) and record.get("status") == "passed" and record.get("input_sha256") == inputs_sha \
        and Path(output).is_file() and record.get("output_sha256") == _sha(output)


def solve_matrix(manifest_path, *, case_ids=(), resume: bool = False) -> list:
    from vericcl_b200.cli.main import main as cli
    root, manifest = _load(manifest_path)
    store = StateStore(root / "state.json")
    previous = store.load()
    records = []
    for case in _select(manifest, case_ids):
        task = "solve:" + case["id"]
        case_dir = root / case["documents"]
        inputs_sha = _inputs_sha(case_dir)
        outputs = root / "runs" / "examples" / "matrix" / "output"
        last = previous.get(task) or {}
        if resume and last.get("run") and _reusable(last, inputs_sha, root / last["run"] / "schedule.xml"):
            records.append(last)
            continue
        run_id = "solve-%s-%d" % (inputs_sha[:12], len(list(outputs.glob("solve-%s-*" % inputs_sha[:12])))
                                  if outputs.exists() else 0)
        argv = ["solve", "--project-root", str(root / "runs"), "--case", "matrix", "--run-id", run_id]
        for k in ("topology", "sketch", "atom", "runtime"):
            argv += ["--" + k, str(case_dir / (k + ".json"))]
        start = time.monotonic()
        code = cli(argv)
        actual = outputs / run_id
        meta = strict_load(actual / "run.json") if (actual / "run.json").exists() else {}
        best = meta.get("best") or {}
        ok = code == 0 and (actual / "schedule.xml").is_file() and best.get("t_pred_us") is not None
        record = {"task": task, "case": case["id"], "status": "passed" if ok else "failed", "exit_code": code,
                  "run": str(actual.relative_to(root)), "input_sha256": inputs_sha,
                  "output_sha256": _sha(actual / "schedule.xml") if ok else None,
                  "t_pred_us": best.get("t_pred_us"), "wall_s": round(time.monotonic() - start, 3)}
        store.put(task, record)
        records.append(record)
    return records


def benchmark_matrix(manifest_path, *, case_ids=(), resume: bool = False, measure=None, iters: int = 10) -> list:
    """Measure every solved schedule; ``measure(xml, request) -> µs`` defaults to the native driver."""
    from vericcl_b200.input.loader import load_request
    root, manifest = _load(manifest_path)
    store = StateStore(root / "state.json")
    previous = store.load()
    if measure is None:
        from vericcl_b200.online.measure import native_measure

        def measure(xml, request):
            return native_measure(xml, request, iters=iters)
    records = []
    for case in _select(manifest, case_ids):
        solved = previous.get("solve:" + case["id"])
        task = "benchmark:" + case["id"]
        if not solved or solved.get("status") != "passed":
            record = {"task": task, "case": case["id"], "status": "skipped", "reason": "not solved"}
            store.put(task, record)
            records.append(record)
            continue
        xml_path = root / solved["run"] / "schedule.xml"
        if resume and _reusable(previous.get(task), solved["output_sha256"], xml_path):
            records.append(previous[task])
            continue
        case_dir = root / case["documents"]
        files = {k: case_dir / (k + ".json") for k in ("topology", "sketch", "atom", "runtime")}
        request = load_request(files, purpose="verify")
        env = {}
        if case.get("groups", 1) > 1:
            # the slow inter-group link is paced by the interpreter on one NVSwitch node
            env["VERICCL_EMULATE"] = "group=%d,gbps=%g" % (case["per_group"], case["inter_gbps"])
        saved = {k: os.environ.get(k) for k in env}
        os.environ.update(env)
        try:
            us = float(measure(xml_path.read_text(), request))
            status, error = "passed", None
        except Exception as exc:   # a failed measurement is recorded, the matrix goes on
            us, status, error = None, "failed", "%s: %s" % (type(exc).__name__, exc)
        finally:
            for k, v in saved.items():
                if v is None:
                    os.environ.pop(k, None)
                else:
                    os.environ[k] = v
        size = case["bytes_per_rank"]
        record = {"task": task, "case": case["id"], "status": status, "measured_us": us, "error": error,
                  "input_sha256": solved["output_sha256"],
                  "output_sha256": _sha(xml_path) if status == "passed" else None,
                  "algbw_gbs": (size / us / 1e3) if us else None, "emulation": env.get("VERICCL_EMULATE")}
        store.put(task, record)
        records.append(record)
    return records


def summarize(manifest_path) -> list:
    root, manifest = _load(manifest_path)
    state = StateStore(root / "state.json").load()
    rows = []
    for case in manifest["cases"]:
        s = state.get("solve:" + case["id"], {})
        b = state.get("benchmark:" + case["id"], {})
        rows.append({"case": case["id"], "collective": case["collective"], "ranks": case["ranks"],
                     "groups": case["groups"], "bytes_per_rank": case["bytes_per_rank"],
                     "solve": s.get("status", "pending"), "t_pred_us": s.get("t_pred_us"),
                     "solve_wall_s": s.get("wall_s"), "benchmark": b.get("status", "pending"),
                     "measured_us": b.get("measured_us"),
                     "measured_over_predicted": (b["measured_us"] / s["t_pred_us"])
                     if b.get("measured_us") and s.get("t_pred_us") else None})
    return rows


def markdown(rows) -> str:
    head = "| case | P | groups | bytes/rank | solve | T_pred µs | benchmark | measured µs | measured/pred |"
    lines = [head, "|---|---|---|---|---|---|---|---|---|"]

    def f(v, fmt="%.3f"):
        return "—" if v is None else fmt % v

    for r in rows:
        lines.append("| %s | %d | %d | %d | %s | %s | %s | %s | %s |" % (
            r["case"], r["ranks"], r["groups"], r["bytes_per_rank"], r["solve"], f(r["t_pred_us"]),
            r["benchmark"], f(r["measured_us"]), f(r["measured_over_predicted"], "%.3f")))
    return "\n".join(lines) + "\n"


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="vericcl_b200.experiment_matrix")
    sub = ap.add_subparsers(dest="stage", required=True)
    p = sub.add_parser("plan")
    p.add_argument("--out", required=True)
    p.add_argument("--groups", default="1,2")
    p.add_argument("--per-group", type=int, default=4)
    p.add_argument("--colls", default="allgather,allreduce")
    p.add_argument("--sizes", default="4m,16m,64m")
    p.add_argument("--inter-gbps", type=float, default=25.0)
    p.add_argument("--datatype", default="float32")
    for name in ("solve", "benchmark"):
        s = sub.add_parser(name)
        s.add_argument("--manifest", required=True)
        s.add_argument("--case", action="append", default=[])
        s.add_argument("--resume", action="store_true")
    m = sub.add_parser("summarize")
    m.add_argument("--manifest", required=True)
    m.add_argument("--markdown", action="store_true")
    args = ap.parse_args(argv)
    if args.stage == "plan":
        manifest = plan_matrix(args.out, groups=[int(g) for g in args.groups.split(",")], per_group=args.per_group,
                               colls=args.colls.split(","), sizes=[parse_size(s) for s in args.sizes.split(",")],
                               inter_gbps=args.inter_gbps, datatype=args.datatype)
        print(json.dumps({"cases": len(manifest["cases"])}))
        return 0
    if args.stage == "solve":
        records = solve_matrix(args.manifest, case_ids=args.case, resume=args.resume)
    elif args.stage == "benchmark":
        records = benchmark_matrix(args.manifest, case_ids=args.case, resume=args.resume)
    else:
        rows = summarize(args.manifest)
        sys.stdout.write(markdown(rows) if args.markdown else "".join(json.dumps(r) + "\n" for r in rows))
        return 0
    print(json.dumps({"tasks": len(records), "passed": sum(r["status"] == "passed" for r in records)}))
    return 0 if all(r["status"] in ("passed", "skipped") for r in records) else 1


if __name__ == "__main__":
    sys.exit(main())
