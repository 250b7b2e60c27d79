"""Generate complete request documents for common cases.

``example_documents`` returns the four JSON documents (topology, sketch,
atom, runtime) for one collective on an NVSwitch B200 domain, with every
budget and tolerance the resolver requires filled in (reference:
tools/generate_examples.py, used by its README).  ``write_documents`` stores
them as ``<dir>/<name>.json``.  ``example_cases`` names a catalog of cases
(every collective kind, both synthesis methods, an emulated two-group
topology) and ``python -m vericcl_b200.examples run`` solves them through
the CLI, writing an index run with each case's exit code, T_pred and checks
(reference: tools/run_examples.py).
"""
from __future__ import annotations

from pathlib import Path

from vericcl_b200.topology.nvswitch import nvswitch_topology
from vericcl_b200.utils.jsonio import atomic_write_json


def example_documents(operator: str = "allreduce", method: str = "hierarchy", ranks: int = 8, *,
                      total_size_bytes: int = 1 << 20, slice_size_bytes: int | None = 1 << 18,
                      datatype: str = "float32", inplace: bool = False, topology: dict | None = None,
                      alpha_us: float | None = None, link_gbps: float | None = None, max_channels: int = 1,
                      tuning_rounds: int = 0, scratch_bytes: int = 1 << 30, calibration: bool = False,
                      per_model_timeout_s: float = 60.0, reduction_op: str | None = None,
                      scale: float | None = None, root: int = 0) -> dict:
    kw = {}
    if alpha_us is not None:
        kw["alpha_us"] = alpha_us
    if link_gbps is not None:
        kw["link_gbps"] = link_gbps
    topo = topology if topology is not None else nvswitch_topology(ranks, **kw)
    collective = {"operator": operator, "datatype": datatype, "inplace": inplace}
    if operator in ("allreduce", "reduce", "reduce_scatter"):
        collective["reduction_op"] = reduction_op or "sum"
        if scale is not None:
            collective["scale"] = scale
    if operator in ("broadcast", "reduce"):
        collective["root"] = root
    sketch = {
        "collective": collective,
        "hyperparameters": {"total_size_bytes": total_size_bytes, "slice_size_bytes": slice_size_bytes},
        "solver": {"backend": "highs", "per_model_timeout_s": per_model_timeout_s, "cpu_budget": 4,
                   "max_threads_per_model": 1, "max_parallel_models": 1, "max_channels": max_channels},
        "budgets": {"max_initial_synthesis_s": 600, "max_offline_validation_per_round_s": 300,
                    "max_offline_validation_total_s": 900, "max_repair_per_round_s": 300,
                    "max_repair_total_s": 900, "max_tuning_rounds": tuning_rounds, "cleanup_reserve_s": 5,
                    "max_online_validation_per_round_s": 600, "max_online_validation_total_s": 1800,
                    "max_run_wall_s": 3600},
        "tolerances": {"absolute": 1e-3, "relative": 1e-3},
        "calibration": {"enabled": calibration, "max_relative_fit_error": 0.1, "job_timeout_s": 300},
        "trace_and_measure": {"enabled": False, "job_timeout_s": 300, "trace_capacity_bytes": 1 << 24},
    }
    atom = {"synthesis_method": method, "M_switch": 1 << 24}
    # eight GPUs per host: ranks beyond the first eight go to further (named) hosts
    hosts = ["localhost" if topo["ranks"] <= 8 else "node-%d" % (r // 8) for r in range(topo["ranks"])]
    runtime = {"rank_map": [{"rank": r, "host": hosts[r], "device": r % 8} for r in range(topo["ranks"])],
               "environment": {"NCCL_BUFFSIZE": str(1 << 26)},
               "scratch_bytes_per_rank": scratch_bytes,
               "control": {"bind_address": "127.0.0.1", "port": 24950}}
    return {"topology": topo, "sketch": sketch, "atom": atom, "runtime": runtime}


def write_documents(directory, documents: dict) -> dict:
    directory = Path(directory)
    files = {}
    for name in ("topology", "sketch", "atom", "runtime"):
        files[name] = atomic_write_json(directory / (name + ".json"), documents[name])
    return files


def example_cases() -> dict:
    """Named example cases: documents for every collective kind and both synthesis methods."""
    from vericcl_b200.topology.nvswitch import multinode_topology
    kib = 1 << 10
    cases = {
        "allreduce-p4": example_documents("allreduce", "hierarchy", 4, total_size_bytes=64 * kib,
                                          slice_size_bytes=16 * kib),
        "allreduce-p8-scale": example_documents("allreduce", "hierarchy", 8, total_size_bytes=64 * kib,
                                                slice_size_bytes=8 * kib, scale=0.125),
        "allgather-p8": example_documents("allgather", "hierarchy", 8, total_size_bytes=64 * kib,
                                          slice_size_bytes=16 * kib),
        "allgather-p4-trees": example_documents("allgather", "constructive_trees", 4, total_size_bytes=64 * kib,
                                                slice_size_bytes=16 * kib),
        "reduce-scatter-p4": example_documents("reduce_scatter", "hierarchy", 4, total_size_bytes=64 * kib,
                                               slice_size_bytes=4 * kib),
        "broadcast-p4-root2": example_documents("broadcast", "hierarchy", 4, total_size_bytes=64 * kib,
                                                slice_size_bytes=16 * kib, root=2),
        "reduce-p4": example_documents("reduce", "hierarchy", 4, total_size_bytes=64 * kib,
                                       slice_size_bytes=16 * kib),
        "alltoall-p4": example_documents("alltoall", "hierarchy", 4, total_size_bytes=64 * kib,
                                         slice_size_bytes=4 * kib),
        "allreduce-2x4-emulated": example_documents("allreduce", "hierarchy", 8, total_size_bytes=64 * kib,
                                                    slice_size_bytes=8 * kib,
                                                    topology=multinode_topology(2, 4, inter_gbps=25.0)),
    }
    for docs in cases.values():
        docs["sketch"]["calibration"]["enabled"] = False
    return cases


def run_examples(project_root, run_prefix: str, names=None, *, case: str = "examples") -> dict:
    """Solve each named case through the public CLI; write an index run with every case's outcome."""
    from vericcl_b200.cli.main import main as cli
    from vericcl_b200.execution.context import RunContext, finalize_run
    from vericcl_b200.utils.jsonio import strict_load
    cases = example_cases()
    selected = list(names or cases)
    unknown = sorted(set(selected) - set(cases))
    if unknown or len(selected) != len(set(selected)):
        raise ValueError("unknown or duplicate example names: %s" % (unknown or selected))
    root = Path(project_root).resolve()
    index = RunContext.create(root, case, "examples", run_id=run_prefix + "-index")
    results = {}
    for name in selected:
        inputs = root / "examples" / case / "input" / name
        files = write_documents(inputs, cases[name])
        run_id = "%s-%s" % (run_prefix, name)
        argv = ["solve", "--project-root", str(root), "--case", case, "--run-id", run_id]
        for key in ("topology", "sketch", "atom", "runtime"):
            argv += ["--" + key, str(files[key])]
        code = cli(argv)
        run = root / "examples" / case / "output" / run_id
        meta = strict_load(run / "run.json") if (run / "run.json").exists() else {}
        best = meta.get("best") or {}
        results[name] = {"exit_code": code, "run": str(run.relative_to(root)), "t_pred_us": best.get("t_pred_us"),
                         "checks": {k: v.get("status") for k, v in (best.get("checks") or {}).items()},
                         "command": "python -m vericcl_b200 " + " ".join(argv)}
        index.emit("example_finished", name=name, exit_code=code, t_pred_us=best.get("t_pred_us"))
    atomic_write_json(index.directory / "examples.json", results)
    failed = sorted(n for n, r in results.items() if r["exit_code"] != 0)
    finalize_run(index, {"status": "ok" if not failed else "failed", "stop_reason": "examples", "best": None,
                         "failed": failed})
    return results


def main(argv=None) -> int:
    import argparse
    import json
    ap = argparse.ArgumentParser(prog="vericcl_b200.examples")
    sub = ap.add_subparsers(dest="verb", required=True)
    w = sub.add_parser("write", help="write one case's four documents")
    w.add_argument("name")
    w.add_argument("--out", required=True)
    r = sub.add_parser("run", help="solve cases through the CLI")
    r.add_argument("--project-root", required=True)
    r.add_argument("--run-prefix", required=True)
    r.add_argument("--names", nargs="+")
    sub.add_parser("list", help="list the case names")
    args = ap.parse_args(argv)
    if args.verb == "list":
        print("\n".join(example_cases()))
        return 0
    if args.verb == "write":
        write_documents(args.out, example_cases()[args.name])
        return 0
    results = run_examples(args.project_root, args.run_prefix, args.names)
    print(json.dumps({n: {"exit_code": r["exit_code"], "t_pred_us": r["t_pred_us"]} for n, r in results.items()}))
    return 0 if all(r["exit_code"] == 0 for r in results.values()) else 1


if __name__ == "__main__":
    import sys
    sys.exit(main())
