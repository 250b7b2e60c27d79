"""Device-timed schedule measurement and the workflow's measured-acceptance hook.

    python -m vericcl_b200.online.measure --inputs DIR --xml schedule.xml [--sidecar schedule.json]
        [--emulate group=2,gbps=25] [--no-measure] [--iters 10] [--warmup 3]

prints, for one solved schedule and the request documents in ``DIR``
(topology/sketch/atom/runtime.json), its predicted time under that topology
(with ``--sidecar``: the initial cost model of the request, exact event
simulation) and its device time on the local GPUs (C-API driver, slowest rank
per invocation, mean over ``--iters``), optionally on an emulated slow link.

``native_measure`` runs one XML schedule on the local GPUs through the C-API
driver and returns the mean per-invocation device time (slowest rank per
invocation).  ``measured_acceptance`` builds the workflow hook: for an
(incumbent, candidate) pair it runs the pre-planned AB/BA pairs, draws the
significance level from the task ledger and returns the comparison verdict.
With ``VERICCL_EMULATE`` set, the interpreter paces inter-group steps, which
is how the two-group online configuration is emulated on one NVSwitch box
(reference: vericcl/online/acceptance.py:110-168 for the paired comparison).
"""
from __future__ import annotations

from vericcl_b200.execution.native import NativeScheduleDriver
from vericcl_b200.online.acceptance import compare_measured
from vericcl_b200.online.statistical_ledger import StatisticalLedger

DTYPE_CODES = {"float32": 0, "bfloat16": 1, "float16": 2}


def native_measure(xml: str, request, *, iters: int = 5, warmup: int = 2, nlanes: int = 32) -> float:
    elem = request.element_bytes
    count = request.hyperparameters.total_size_bytes // elem
    runtime = request.request_config["runtime"]
    ranks = sorted(runtime["rank_map"], key=lambda e: e["rank"])
    paths = runtime.get("paths") or {}
    driver = NativeScheduleDriver(xml, request.rank_count, hosts=[e.get("host", "localhost") for e in ranks],
                                  devices=[e.get("device", e["rank"]) for e in ranks],
                                  binary=paths.get("vericcl_native") or None,
                                  environment=runtime.get("environment") or {})
    res = driver.measure(count=count, dtype=DTYPE_CODES.get(request.collective.datatype, 0), nlanes=nlanes,
                         warmup=warmup, iters=iters, timeout_s=60.0, root=request.collective.root or 0)
    if res["bad"] or res.get("bad_input"):
        raise RuntimeError("measured schedule produced wrong results (%d outputs, %d inputs changed)"
                           % (res["bad"], res.get("bad_input", 0)))
    return res["mean_us"]


def measured_acceptance(request, ledger_path, *, measure=None):
    cfg = request.request_config["sketch"]["trace_and_measure"]
    ledger = StatisticalLedger(ledger_path, task_alpha=cfg["task_alpha"], single_cap=cfg["single_attempt_alpha_cap"])
    measure = measure or native_measure

    def hook(incumbent, candidate):
        alpha = ledger.allocate("%s-vs-%s" % (getattr(incumbent, "candidate_id", "inc"),
                                              getattr(candidate, "candidate_id", "cand")))
        xmls = {"A": incumbent.xml, "B": candidate.xml}
        return compare_measured(lambda label: measure(xmls[label], request), pairs=cfg["pairs"], seed=cfg["seed"],
                                alpha=alpha, max_cv=cfg["max_cv"], max_rounds=cfg["max_rounds"],
                                min_relative_gain=cfg["min_relative_gain"])
    return hook


def main(argv=None) -> int:
    import argparse
    import json
    import os
    from pathlib import Path

    ap = argparse.ArgumentParser(prog="vericcl_b200.online.measure")
    ap.add_argument("--inputs", required=True, help="folder with topology/sketch/atom/runtime.json")
    ap.add_argument("--xml", required=True)
    ap.add_argument("--sidecar", default=None, help="the schedule's sidecar (schedule.json): also predict")
    ap.add_argument("--emulate", default=None, help="VERICCL_EMULATE for the measurement, e.g. group=2,gbps=25")
    ap.add_argument("--no-measure", action="store_true")
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    args = ap.parse_args(argv)
    from vericcl_b200.input.loader import load_request
    inputs = Path(args.inputs)
    files = {k: inputs / (k + ".json") for k in ("topology", "sketch", "atom", "runtime")}
    xml = Path(args.xml).read_text()
    out = {"xml": args.xml, "inputs": args.inputs}
    if args.sidecar:
        from vericcl_b200.program.sidecar import bundle_from_sidecar
        from vericcl_b200.topology import load_topology
        from vericcl_b200.utils.jsonio import strict_load
        request = load_request(files, purpose="verify")
        bundle = bundle_from_sidecar(request, load_topology(request), xml, strict_load(args.sidecar))
        out["t_pred_us"] = bundle.t_pred_us
    if not args.no_measure:
        if args.emulate:
            os.environ["VERICCL_EMULATE"] = args.emulate
        out["emulate"] = os.environ.get("VERICCL_EMULATE")
        out["device_us"] = native_measure(xml, load_request(files, [], purpose="solve"), iters=args.iters,
                                          warmup=args.warmup)
    print(json.dumps(out))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
