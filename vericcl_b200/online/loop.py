"""Online tuning loop on an emulated two-group topology.

    python -m vericcl_b200.online.loop --project-root runs [--groups 2] [--per-group 4]
        [--inter-gbps 25] [--size-bytes 134217728] [--rounds 3] [--pairs 6] [--datatype float32]
        [--no-final-measure] [--no-rank-shares]

Builds the request for an AllReduce over ``groups`` NVSwitch groups joined by
a slow shared inter-group link (each group's traffic to the other groups
shares one ``inter_gbps`` resource, split evenly over the group's ranks as the
emulator enforces it), emulates that link on one box by pacing
the interpreter's inter-group steps (``VERICCL_EMULATE``), and runs the
primary workflow with calibration and measured acceptance enabled:
probe campaign → cost-model refit → verification against the refitted model
→ repair / resynthesis per round, where a candidate is adopted only when the
paired device-timed comparison accepts it.  The workflow's run directory
keeps the events, reports and checkpoints; this module prints one JSON line
with the per-round outcome and the device time of the first and the final
schedule (reference: vericcl/workflow_v5.py:553-666 for the loop,
vericcl/online/acceptance.py for the paired comparison).
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import time
from pathlib import Path

from vericcl_b200.examples import example_documents, write_documents
from vericcl_b200.topology.nvswitch import multinode_topology


def loop_documents(*, groups: int, per_group: int, inter_gbps: float, size_bytes: int, rounds: int,
                   datatype: str, pairs: int, slice_bytes: int | None = None, rank_shares: bool = True) -> dict:
    ranks = groups * per_group
    docs = example_documents("allreduce", "hierarchy", ranks, total_size_bytes=size_bytes,
                             slice_size_bytes=slice_bytes or size_bytes // ranks, datatype=datatype,
                             topology=multinode_topology(groups, per_group, inter_gbps=inter_gbps,
                                                         rank_shares=rank_shares),
                             tuning_rounds=rounds, calibration=True, scratch_bytes=4 * size_bytes)
    docs["sketch"]["trace_and_measure"].update({"enabled": True, "pairs": pairs, "max_rounds": 2,
                                                "max_cv": 0.05, "warmup_iterations": 2, "timed_iterations": 5})
    docs["sketch"]["calibration"].update({"warmup_iterations": 2, "timed_iterations": 5, "launches": 2,
                                          "payload_sizes": [2 << 20, 8 << 20, 32 << 20],
                                          "probe_scope": "link_classes"})
    return docs


def run_loop(project_root, *, groups: int = 2, per_group: int = 4, inter_gbps: float = 25.0,
             size_bytes: int = 128 << 20, rounds: int = 3, datatype: str = "float32", pairs: int = 6,
             case: str = "online-loop", measure_final: bool = True, rank_shares: bool = True) -> dict:
    emulate = "group=%d,gbps=%g" % (per_group, inter_gbps)
    previous = os.environ.get("VERICCL_EMULATE")
    os.environ["VERICCL_EMULATE"] = emulate
    try:
        return _run_loop(Path(project_root), emulate, groups=groups, per_group=per_group, inter_gbps=inter_gbps,
                         size_bytes=size_bytes, rounds=rounds, datatype=datatype, pairs=pairs, case=case,
                         measure_final=measure_final, rank_shares=rank_shares)
    finally:
        if previous is None:
            os.environ.pop("VERICCL_EMULATE", None)
        else:
            os.environ["VERICCL_EMULATE"] = previous


def _run_loop(root: Path, emulate: str, *, groups, per_group, inter_gbps, size_bytes, rounds, datatype, pairs, case,
              measure_final, rank_shares=True) -> dict:
    from vericcl_b200.cli.main import main as cli_main
    from vericcl_b200.utils.jsonio import strict_load
    docs = loop_documents(groups=groups, per_group=per_group, inter_gbps=inter_gbps, size_bytes=size_bytes,
                          rounds=rounds, datatype=datatype, pairs=pairs, rank_shares=rank_shares)
    files = write_documents(root / "inputs" / case, docs)
    run_id = "loop-%s" % time.strftime("%Y%m%d-%H%M%S")
    argv = ["solve", "--project-root", str(root), "--case", case, "--run-id", run_id]
    for name in ("topology", "sketch", "atom", "runtime"):
        argv += ["--" + name, str(files[name])]
    code = cli_main(argv)
    run_dir = root / "examples" / case / "output" / run_id
    if not (run_dir / "run.json").exists():
        return {"exit_code": code, "error": "no run directory written"}
    meta = strict_load(run_dir / "run.json")
    result = meta.get("result") or {}
    summary = {"exit_code": code, "run": str(run_dir), "emulate": emulate,
               "ranks": groups * per_group, "size_bytes": size_bytes, "datatype": datatype,
               "stop_reason": result.get("stop_reason"), "best": meta.get("best"),
               "rounds": [{k: r.get(k) for k in ("round", "start_t_pred_us", "cut_lower_bound_us", "result",
                                                 "t_pred_us", "measured")} for r in result.get("rounds", [])]}
    calibration = run_dir / "process" / "reports" / "calibration.json"
    if calibration.exists():
        report = strict_load(calibration)
        summary["calibration"] = {k: report.get(k) for k in ("qualified", "rejected", "fit_errors")
                                  if k in report}
    if measure_final and code == 0:
        import torch
        if torch.cuda.device_count() >= groups * per_group:
            summary["device_us"] = _measure_first_and_final(run_dir, files)
            summary["trace"] = _capture_trace(run_dir, groups * per_group, size_bytes, datatype)
        else:
            summary["device_us"] = "skipped: fewer GPUs than ranks"
    return summary


def _measure_first_and_final(run_dir: Path, files: dict) -> dict:
    from vericcl_b200.input.loader import load_request
    from vericcl_b200.online.measure import native_measure
    request = load_request(files, [], purpose="solve")
    out = {}
    final = run_dir / "schedule.xml"
    baseline = sorted((run_dir / "process" / "candidates").glob("*/schedule.xml"), key=lambda p: p.stat().st_mtime)
    if baseline:
        out["first_candidate"] = native_measure(baseline[0].read_text(), request, iters=10, warmup=3)
    if final.exists():
        out["final"] = native_measure(final.read_text(), request, iters=10, warmup=3)
    return out


def _capture_trace(run_dir: Path, ranks: int, size_bytes: int, datatype: str) -> dict:
    """The run's trace of the final schedule (the CLI captures it when measurement is on), else capture one."""
    from vericcl_b200.online.trace_worker import capture_schedule_trace
    path = run_dir / "trace.json"
    if path.exists():
        report = json.loads(path.read_text())
        return {"path": str(path), "global_span_us": report["global_span_us"], "tails": report["tails"][:3]}
    return capture_schedule_trace(run_dir / "schedule.xml", ranks, size_bytes, datatype,
                                  run_dir / "process" / "traces")


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="vericcl_b200.online.loop")
    ap.add_argument("--project-root", required=True)
    ap.add_argument("--case", default="online-loop")
    ap.add_argument("--groups", type=int, default=2)
    ap.add_argument("--per-group", type=int, default=4)
    ap.add_argument("--inter-gbps", type=float, default=25.0)
    ap.add_argument("--size-bytes", type=int, default=128 << 20)
    ap.add_argument("--rounds", type=int, default=3)
    ap.add_argument("--pairs", type=int, default=6)
    ap.add_argument("--datatype", default="float32")
    ap.add_argument("--no-final-measure", action="store_true")
    ap.add_argument("--no-rank-shares", action="store_true",
                    help="describe only the group-shared link, not the emulator's per-rank shares of it")
    args = ap.parse_args(argv)
    summary = run_loop(args.project_root, groups=args.groups, per_group=args.per_group, inter_gbps=args.inter_gbps,
                       size_bytes=args.size_bytes, rounds=args.rounds, datatype=args.datatype, pairs=args.pairs,
                       case=args.case, measure_final=not args.no_final_measure,
                       rank_shares=not args.no_rank_shares)
    print(json.dumps(summary, default=str))
    return 0 if summary.get("exit_code") == 0 else 1


if __name__ == "__main__":
    sys.exit(main())
