"""Command line: ``python -m vericcl_b200 {solve,verify,calibrate,inspect,resume,manual-generate}``.

Arguments mirror the reference CLI (vericcl/cli/main.py:22-80): the four
input files, ``--project-root``, ``--case``, ``--run-id``, repeated
``--set FIELD=JSON`` overrides and ``--override-input``; ``verify`` adds
``--xml --sidecar --model [--tune]``; ``inspect`` and ``resume`` take
``--run``; ``manual-generate`` writes an editable manual-stage input folder
(``--out``) from the four inputs.  Exit codes: 0 ok, 2 invalid input, 5 semantic failure, 7 budget,
8 runtime failure, 130 interrupted.
"""
from __future__ import annotations

import argparse
import json
import sys
from pathlib import Path

from vericcl_b200 import __version__
from vericcl_b200.errors import VericclError


def _inputs(p):
    p.add_argument("--project-root", default=".")
    p.add_argument("--case", required=True)
    p.add_argument("--run-id", default=None)
    for name in ("topology", "sketch", "atom", "runtime"):
        p.add_argument("--" + name, required=True)
    p.add_argument("--set", dest="overrides", action="append", default=[], metavar="FIELD=JSON")
    p.add_argument("--override-input", action="store_true")


def build_parser():
    parser = argparse.ArgumentParser(prog="vericcl_b200", description="B200 collective schedule synthesizer")
    parser.add_argument("--version", action="version", version="vericcl_b200 " + __version__)
    sub = parser.add_subparsers(dest="command", required=True)
    _inputs(sub.add_parser("solve", help="synthesize, verify and tune a schedule"))
    v = sub.add_parser("verify", help="check an existing schedule (optionally tune it)")
    _inputs(v)
    v.add_argument("--xml", required=True)
    v.add_argument("--sidecar", required=True)
    v.add_argument("--model", required=True)
    v.add_argument("--tune", action="store_true")
    _inputs(sub.add_parser("calibrate", help="measure the cost model on the GPUs"))
    i = sub.add_parser("inspect", help="print a run's status as JSON")
    i.add_argument("--run", required=True)
    r = sub.add_parser("resume", help="continue a run from its checkpoint")
    r.add_argument("--run", required=True)
    m = sub.add_parser("manual-generate", help="write an editable manual-stage plan as a new input folder")
    for name in ("topology", "sketch", "atom", "runtime"):
        m.add_argument("--" + name, required=True)
    m.add_argument("--out", required=True, help="folder for the four documents with atom.manual enabled")
    m.add_argument("--from", dest="source", choices=("direct", "hierarchy"), default="direct",
                   help="the plan whose stages become manual nodes")
    return parser


def _files(args):
    return {name: getattr(args, name) for name in ("topology", "sketch", "atom", "runtime")}


def _probe_executor(request):
    from vericcl_b200.online.native_probe import native_probe_executor
    return native_probe_executor(request)


def new_run(args) -> int:
    from vericcl_b200.execution.context import RunContext
    from vericcl_b200.input.loader import load_request
    from vericcl_b200.performance.model import CostModel
    from vericcl_b200.utils.jsonio import strict_load
    from vericcl_b200.workflow import PrimaryWorkflow
    purpose = args.command
    request = load_request(_files(args), args.overrides, override_input=args.override_input, purpose=purpose)
    extra = {}
    verify_inputs = None
    model = None
    if purpose == "verify":
        extra = {"schedule_xml": args.xml, "schedule_sidecar": args.sidecar, "model": args.model}
        verify_inputs = {"xml": Path(args.xml).read_text(), "sidecar": strict_load(args.sidecar)}
        model = CostModel.from_json(strict_load(args.model))
    ctx = RunContext.create(args.project_root, args.case, purpose, run_id=args.run_id, input_files=_files(args),
                            extra_inputs=extra)
    ctx.update_run_json(effective_request=dict(request.request_config), value_sources=dict(request.value_sources),
                        size_accounting=dict(request.size_accounting), overrides=list(args.overrides))
    executor = _probe_executor(request) if (purpose == "calibrate" or
                                            request.request_config["sketch"]["calibration"]["enabled"]) else None
    measure = trace_provider = None
    if request.request_config["sketch"]["trace_and_measure"]["enabled"] and executor is not None:
        from vericcl_b200.online.measure import measured_acceptance
        from vericcl_b200.online.trace_worker import trace_report_for_xml
        measure = measured_acceptance(request, ctx.process / "statistics" / "ledger.jsonl")
        counter = iter(range(1 << 30))
        trace_provider = (lambda bundle: trace_report_for_xml(
            bundle.xml, request, ctx.process / "traces" / ("round-%d" % next(counter))))
    wf = PrimaryWorkflow(request, ctx, purpose=purpose, tune=getattr(args, "tune", False), model=model,
                         verify_inputs=verify_inputs, probe_executor=executor, measure=measure,
                         trace_provider=trace_provider)
    result = wf.run()
    if measure is not None and result.status == "ok" and (ctx.directory / "schedule.xml").exists():
        _trace_best(request, ctx)
    print(json.dumps({"run": str(ctx.directory), "status": result.status, "stop_reason": result.stop_reason,
                      "t_pred_us": None if result.best is None else result.best["t_pred_us"]}))
    return 0 if result.status == "ok" else 5


def _trace_best(request, ctx) -> None:
    """With trace_and_measure on GPUs: one traced invocation of the published schedule → ``trace.json``."""
    import shutil
    from vericcl_b200.online.trace_worker import capture_schedule_trace
    summary = capture_schedule_trace(ctx.directory / "schedule.xml", request.rank_count,
                                     request.hyperparameters.total_size_bytes, request.collective.datatype,
                                     ctx.process / "traces")
    if "error" in summary:
        ctx.emit("trace_failed", reason=summary["error"])
        return
    shutil.copyfile(summary["path"], ctx.directory / "trace.json")
    ctx.emit("trace_captured", global_span_us=summary["global_span_us"])


def inspect_run(args) -> int:
    from vericcl_b200.utils.jsonio import strict_load
    run = Path(args.run)
    meta = strict_load(run / "run.json")
    checkpoints = sorted(p.name for p in (run / "process" / "checkpoints").glob("*.json"))
    print(json.dumps({"run_id": meta.get("run_id"), "status": meta.get("status"), "best": meta.get("best"),
                      "result": meta.get("result"), "checkpoints": checkpoints}, indent=2, default=str))
    return 0


def resume_run(args) -> int:
    from vericcl_b200.execution.checkpoint import restore_checkpoint
    from vericcl_b200.execution.context import RunContext
    from vericcl_b200.input.loader import resolve_documents
    from vericcl_b200.performance.model import CostModel
    from vericcl_b200.utils.jsonio import strict_load
    from vericcl_b200.workflow import PrimaryWorkflow
    ctx = RunContext.open(args.run)
    meta = ctx.read_run_json()
    if meta.get("status") == "finished":
        print(json.dumps({"run": str(ctx.directory), "status": "already finished"}))
        return 0
    state = restore_checkpoint(ctx)
    request = resolve_documents(meta["effective_request"], purpose=meta["command"] if meta["command"] in (
        "solve", "verify", "calibrate") else "solve")
    model_path = ctx.process / "models" / (state["state"]["model_version"] + ".json")
    model = CostModel.from_json(strict_load(model_path)) if model_path.exists() else None
    wf = PrimaryWorkflow(request, ctx, purpose=state["state"].get("purpose", "solve"),
                         tune=state["state"].get("tune", False), model=model, restored=state)
    result = wf.run()
    print(json.dumps({"run": str(ctx.directory), "status": result.status, "stop_reason": result.stop_reason,
                      "resumed_from": state["phase"]}))
    return 0 if result.status == "ok" else 5


def manual_generate(args) -> int:
    """Manual nodes (stages, groups, roots, dependencies, input/output states) from the direct or hierarchy plan
    of the given inputs, written with the other three documents into ``--out``; the result is re-planned once
    to check it (reference: README.md "manual-generate")."""
    from vericcl_b200.examples import write_documents
    from vericcl_b200.input.loader import load_request
    from vericcl_b200.planner.direct import build_direct_plan
    from vericcl_b200.planner.manual import manual_nodes_from_plan, plan_manual
    from vericcl_b200.topology import load_topology
    from vericcl_b200.utils.jsonio import strict_load
    files = _files(args)
    docs = {name: strict_load(path) for name, path in files.items()}
    request = load_request(files)
    topology = load_topology(request)
    if args.source == "hierarchy":
        from vericcl_b200.planner.hierarchy import plan_hierarchy
        plan = plan_hierarchy(request, topology)
    else:
        plan = build_direct_plan(request, topology)
    nodes = manual_nodes_from_plan(plan)
    atom = dict(docs["atom"])
    manual = dict(atom.get("manual") or {})
    manual.update(enabled=True, nodes=nodes)
    atom["manual"] = manual
    docs["atom"] = atom
    paths = write_documents(Path(args.out), docs)
    checked = plan_manual(load_request(paths), topology)
    print(json.dumps({"out": str(Path(args.out)), "nodes": len(nodes),
                      "stages": len({n["stage_id"] for n in nodes}), "planned_nodes": len(checked.nodes)}))
    return 0


def main(argv=None) -> int:
    parser = build_parser()
    args = parser.parse_args(argv)
    try:
        if args.command in ("solve", "verify", "calibrate"):
            return new_run(args)
        if args.command == "inspect":
            return inspect_run(args)
        if args.command == "manual-generate":
            return manual_generate(args)
        return resume_run(args)
    except KeyboardInterrupt:
        return 130
    except VericclError as error:
        print("error: %s" % error, file=sys.stderr)
        return error.exit_code
