"""Wall-clock attribution of the synthesis pipeline and timing of schedule replay.

    python -m vericcl_b200.experiments overhead solve --inputs DIR [--repeats 5] --out overhead.json
    python -m vericcl_b200.experiments overhead replay --inputs DIR --xml S.xml --sidecar S.json --out replay.json

``solve`` runs :func:`vericcl_b200.synthesis.synthesize` on the request in
``DIR`` (``topology.json``, ``sketch.json``, ``atom.json``,
``runtime.json``) ``repeats`` times, after one untimed warm-up, with every
pipeline phase wrapped in a timer: plan, demands, route MILP, composition,
timing MILP, constructive trees, storage plan, lowering, XML emission,
executable, exact prediction, admission checks and the native compile inside
them.  ``replay`` times the re-check of an immutable schedule (sidecar load,
the eight checks and the exact prediction).  The output holds every span
(inclusive, with its nesting depth), per-phase medians, the time no phase
claims, the outcome (T_pred, checks), the input digest and the machine
(reference: vericcl/experiments/overhead.py:23-374, which attributes its
own pipeline the same way).
"""
from __future__ import annotations

import hashlib
import importlib
import json
import os
import platform
import statistics
import sys
import time
from contextlib import contextmanager
from pathlib import Path

# (module, attribute, phase); each is looked up through its module at call time
PHASES = (
    ("vericcl_b200.synthesis", "plan_for", "plan"),
    ("vericcl_b200.synthesis", "build_demands", "demands"),
    ("vericcl_b200.synthesis", "choose_trees", "route_milp"),
    ("vericcl_b200.synthesis", "compose_routes", "compose"),
    ("vericcl_b200.solver.timing", "optimize_fixed_routes", "timing_milp"),
    ("vericcl_b200.solver.trees.construct", "construct_network", "constructive_trees"),
    ("vericcl_b200.synthesis", "build_storage_plan", "storage"),
    ("vericcl_b200.synthesis", "lower_program", "lowering"),
    ("vericcl_b200.synthesis", "emit_xml", "xml"),
    ("vericcl_b200.synthesis", "build_executable", "executable"),
    ("vericcl_b200.performance.simulation", "predict", "prediction"),
    ("vericcl_b200.program.checks", "evaluate_program", "checks"),
    ("vericcl_b200.program.device", "compile_xml", "native_compile"),
)


class PhaseTimer:
    """Nested wall-clock spans."""

    def __init__(self, clock=time.perf_counter_ns):
        self.clock = clock
        self.spans = []
        self._depth = 0

    @contextmanager
    def span(self, name: str):
        start = self.clock()
        self._depth += 1
        error = None
        try:
            yield
        except BaseException as exc:
            error = type(exc).__name__
            raise
        finally:
            self._depth -= 1
            self.spans.append({"name": name, "start_ns": start, "end_ns": self.clock(), "depth": self._depth,
                               "error": error})

    def totals(self) -> dict:
        out = {}
        for s in self.spans:
            out[s["name"]] = out.get(s["name"], 0) + s["end_ns"] - s["start_ns"]
        return out

    def top_level_ns(self) -> int:
        return sum(s["end_ns"] - s["start_ns"] for s in self.spans if s["depth"] == 0)


@contextmanager
def instrument(timer: PhaseTimer, phases=PHASES):
    """Wrap each phase function in a timer span for the duration of the block, then restore it."""
    saved = []
    try:
        for module_name, attr, phase in phases:
            module = importlib.import_module(module_name)
            original = getattr(module, attr)

            def wrapper(*args, __fn=original, __phase=phase, **kwargs):
                with timer.span(__phase):
                    return __fn(*args, **kwargs)

            setattr(module, attr, wrapper)
            saved.append((module, attr, original))
        yield timer
    finally:
        for module, attr, original in reversed(saved):
            setattr(module, attr, original)


def environment() -> dict:
    import numpy
    import scipy
    return {"python": platform.python_version(), "platform": platform.platform(), "machine": platform.machine(),
            "cpus": os.cpu_count(), "numpy": numpy.__version__, "scipy": scipy.__version__}


def input_digest(files: dict) -> str:
    h = hashlib.sha256()
    for name in sorted(files):
        h.update(name.encode())
        h.update(Path(files[name]).read_bytes())
    return h.hexdigest()


def _files(inputs) -> dict:
    d = Path(inputs)
    files = {k: d / (k + ".json") for k in ("topology", "sketch", "atom", "runtime")}
    missing = [str(p) for p in files.values() if not p.exists()]
    if missing:
        raise FileNotFoundError("missing input documents: %s" % ", ".join(missing))
    return files


def _summary(runs: list) -> dict:
    phases = sorted({name for r in runs for name in r["totals_ns"]})
    out = {name: statistics.median(r["totals_ns"].get(name, 0) for r in runs) / 1e6 for name in phases}
    return {"median_ms": out, "median_total_ms": statistics.median(r["total_ns"] for r in runs) / 1e6,
            "median_unattributed_ms": statistics.median(r["unattributed_ns"] for r in runs) / 1e6}


def _timed(fn, repeats: int, warmups: int = 1):
    result = None
    for _ in range(warmups):
        result = fn()
    runs = []
    for _ in range(repeats):
        timer = PhaseTimer()
        with instrument(timer):
            start = time.perf_counter_ns()
            result = fn()
            total = time.perf_counter_ns() - start
        runs.append({"total_ns": total, "totals_ns": timer.totals(), "spans": timer.spans,
                     "unattributed_ns": max(0, total - timer.top_level_ns())})
    return result, runs


def run_solve(inputs, *, repeats: int = 5, channels: int = 1) -> dict:
    from vericcl_b200.input.loader import load_request
    from vericcl_b200.synthesis import synthesize
    files = _files(inputs)
    request = load_request(files)
    if request.hyperparameters.slice_size_bytes is None:
        from vericcl_b200.planner.parameters import initial_parameter_domain
        request = request.with_slice(initial_parameter_domain(request)[0].slice_size_bytes)
    bundle, runs = _timed(lambda: synthesize(request, channels=channels), repeats)
    return {"mode": "solve", "inputs": {k: str(v) for k, v in files.items()}, "input_sha256": input_digest(files),
            "environment": environment(), "repeats": repeats, "runs": runs, "summary": _summary(runs),
            "outcome": {"t_pred_us": bundle.t_pred_us, "can_execute": bundle.can_execute,
                        "checks": {k: v.get("status") for k, v in bundle.checks.items()},
                        "slice_size_bytes": request.hyperparameters.slice_size_bytes}}


def run_replay(inputs, xml_path, sidecar_path, *, repeats: int = 5) -> dict:
    from vericcl_b200.input.loader import load_request
    from vericcl_b200.program.sidecar import bundle_from_sidecar
    from vericcl_b200.topology import load_topology
    from vericcl_b200.utils.jsonio import strict_load
    files = _files(inputs)
    request = load_request(files, purpose="verify")
    topology = load_topology(request)
    xml = Path(xml_path).read_text()
    sidecar = strict_load(sidecar_path)
    bundle, runs = _timed(lambda: bundle_from_sidecar(request, topology, xml, sidecar), repeats)
    return {"mode": "replay", "inputs": {k: str(v) for k, v in files.items()}, "input_sha256": input_digest(files),
            "schedule_sha256": hashlib.sha256(xml.encode()).hexdigest(), "environment": environment(),
            "repeats": repeats, "runs": runs, "summary": _summary(runs),
            "outcome": {"t_pred_us": bundle.t_pred_us, "can_execute": bundle.can_execute,
                        "checks": {k: v.get("status") for k, v in bundle.checks.items()}}}


def add_arguments(parser) -> None:
    parser.add_argument("mode", choices=("solve", "replay"))
    parser.add_argument("--inputs", required=True, help="directory with the four request documents")
    parser.add_argument("--xml")
    parser.add_argument("--sidecar")
    parser.add_argument("--repeats", type=int, default=5)
    parser.add_argument("--channels", type=int, default=1)
    parser.add_argument("--out", required=True)


def run(args) -> int:
    from vericcl_b200.utils.jsonio import atomic_write_json
    if args.mode == "replay":
        if not (args.xml and args.sidecar):
            raise SystemExit("replay needs --xml and --sidecar")
        doc = run_replay(args.inputs, args.xml, args.sidecar, repeats=args.repeats)
    else:
        doc = run_solve(args.inputs, repeats=args.repeats, channels=args.channels)
    atomic_write_json(args.out, doc)
    summary = doc["summary"]
    print(json.dumps({"mode": doc["mode"], "median_total_ms": round(summary["median_total_ms"], 3),
                      "phases_ms": {k: round(v, 3) for k, v in summary["median_ms"].items()},
                      "t_pred_us": doc["outcome"]["t_pred_us"]}))
    return 0


if __name__ == "__main__":
    import argparse
    ap = argparse.ArgumentParser(prog="vericcl_b200.overhead")
    add_arguments(ap)
    sys.exit(run(ap.parse_args()))
