"""Device-timed schedule measurement and the workflow's measured-acceptance hook.

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
