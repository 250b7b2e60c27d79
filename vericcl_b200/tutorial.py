"""Repair tutorial: local repair, history reuse and a resynthesis with another slice size.

    python -m vericcl_b200.tutorial --project-root DIR --run-id ID

A three-rank broadcast from rank 0 on a topology whose link 0→1 is ten times
slower than the others.  The starting schedule sends every slice straight
from the root; the tutorial then

1. analyses it (critical-path causes → repair strategies) and runs local
   repair, which moves the slices bound for rank 1 onto the path 0→2→1;
2. stores the repaired schedule in a history index and finds it again for
   the same topology with its ranks relabelled (isomorphic reuse);
3. resynthesizes with the slice size halved and doubled and keeps the best
   candidate by exact T_pred.

Every schedule it adopts passes the eight admission checks.  The run
directory holds each step's XML, ``tutorial.json`` (T_pred per step, the
repaired routes) and the usual ``run.json`` / events (reference:
tools/repair_example.py, which walks the same three steps on its own
tutorial model).
"""
from __future__ import annotations

import argparse
import json
import sys

SLOW_LINK = (0, 1)
SLOW_BETA = 0.1          # µs per byte on 0→1
FAST_BETA = 0.01         # µs per byte elsewhere


def tutorial_documents(total_size_bytes: int = 4096, slice_size_bytes: int = 1024) -> dict:
    from vericcl_b200.examples import example_documents
    docs = example_documents("broadcast", "hierarchy", 3, total_size_bytes=total_size_bytes,
                             slice_size_bytes=slice_size_bytes, calibration=False, root=0)
    for link in docs["topology"]["directed_links"]:
        link["beta_us_per_byte"] = SLOW_BETA if (link["src"], link["dst"]) == SLOW_LINK else FAST_BETA
        link["alpha_us"] = 1.0
    docs["topology"]["multicast_groups"] = []
    return docs


def direct_broadcast(request):
    """Every slice sent straight from the root to every other rank, one channel."""
    from vericcl_b200.composer.compose import NetworkCandidate, NetworkOperation
    n, p, root = request.hyperparameters.slice_count, request.rank_count, request.collective.root
    ops = []
    for index in range(n):
        sid = frozenset({root * n + index})
        for dst in range(p):
            if dst != root:
                ops.append(NetworkOperation("direct:%d:%d" % (index, dst), "send", root, dst, 0, 0, sid, sid,
                                            frozenset(), float(index), index))
    return NetworkCandidate(p, n, request.hyperparameters.slice_size_bytes, tuple(ops), "tutorial-direct")


def _routes(bundle) -> list:
    return sorted({(op.src_rank, op.dst_rank) for op in bundle.network.operations})


def run(project_root, run_id: str, case: str = "repair-tutorial") -> dict:
    from vericcl_b200.examples import write_documents
    from vericcl_b200.execution.context import RunContext, finalize_run
    from vericcl_b200.input.loader import load_request
    from vericcl_b200.performance.initial import initial_cost_model
    from vericcl_b200.solver.history import find_schedules, save_schedule
    from vericcl_b200.synthesis import Lowerer
    from vericcl_b200.topology import load_topology
    from vericcl_b200.tuning.resynthesis import ResynthesisRequest, resynthesize_branch
    from vericcl_b200.tuning.strategies import solve_repair
    from vericcl_b200.utils.jsonio import atomic_write_json, atomic_write_text
    from vericcl_b200.verification.bottlenecks import analyze
    from pathlib import Path

    docs = tutorial_documents()
    inputs = Path(project_root).resolve() / "examples" / case / "input" / run_id
    files = write_documents(inputs, docs)
    ctx = RunContext.create(project_root, case, "tutorial", run_id=run_id, input_files=files)
    request = load_request(files)
    topology = load_topology(request)
    model = initial_cost_model(request)
    lower = Lowerer(request, topology, model)
    steps = {}

    start = lower(direct_broadcast(request))
    if not start.can_execute:
        raise RuntimeError("the direct schedule failed its checks: %s" % start.checks)
    steps["direct"] = {"t_pred_us": start.t_pred_us, "routes": _routes(start)}
    atomic_write_text(ctx.process / "direct.xml", start.xml)
    ctx.emit("tutorial_step", step="direct", t_pred_us=start.t_pred_us)

    # 1. local repair on the critical path
    analysis = analyze(start, model, batch_size=8)
    outcome = solve_repair(start, analysis.strategies, lower=lower)
    repaired = outcome.best if outcome.improved else start
    steps["repair"] = {"t_pred_us": repaired.t_pred_us, "improved": bool(outcome.improved),
                       "causes": [c.kind for c in analysis.causes][:10], "routes": _routes(repaired)}
    atomic_write_text(ctx.process / "repaired.xml", repaired.xml)
    ctx.emit("tutorial_step", step="repair", t_pred_us=repaired.t_pred_us)

    # 2. history: store, then find it again for the same topology
    index = ctx.process / "history" / "index.json"
    save_schedule(index, request, topology, repaired.xml, repaired.t_pred_us)
    found = find_schedules(index, request, topology, tolerance=0.01, limit=4)
    steps["history"] = {"stored": 1, "found": len(found),
                        "t_pred_us": [f["t_pred_us"] for f in found]}

    # 3. resynthesis with other slice sizes
    best = repaired
    tried = []
    for factor in (0.5, 2):
        size = int(request.hyperparameters.slice_size_bytes * factor)
        alt = resynthesize_branch(request, ResynthesisRequest("partition", slice_size_bytes=size), model)
        if alt is None or not alt.can_execute:
            tried.append({"slice_size_bytes": size, "t_pred_us": None})
            continue
        tried.append({"slice_size_bytes": size, "t_pred_us": alt.t_pred_us})
        if alt.t_pred_us < best.t_pred_us:
            best = alt
    steps["resynthesis"] = {"branches": tried, "best_t_pred_us": best.t_pred_us,
                            "best_slice_size_bytes": best.request.hyperparameters.slice_size_bytes}
    atomic_write_text(ctx.directory / "schedule.xml", best.xml)
    atomic_write_json(ctx.directory / "tutorial.json", steps)
    finalize_run(ctx, {"status": "ok", "stop_reason": "tutorial", "best": {"t_pred_us": best.t_pred_us}})
    return steps


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="vericcl_b200.tutorial", description=__doc__.splitlines()[0])
    ap.add_argument("--project-root", required=True)
    ap.add_argument("--run-id", required=True)
    ap.add_argument("--case", default="repair-tutorial")
    args = ap.parse_args(argv)
    steps = run(args.project_root, args.run_id, args.case)
    print(json.dumps({k: v.get("t_pred_us", v.get("best_t_pred_us")) for k, v in steps.items()}))
    return 0


if __name__ == "__main__":
    sys.exit(main())
