"""The main loop: initial synthesis → baseline → calibration → tuning rounds.

Stages (reference: vericcl/workflow_v5.py:61-790):

1. **initial candidates** — for each legal (S, C) choice, synthesize with the
   selected method (hierarchy / constructive_trees / manual) plus the other
   method as a second stream; every candidate is lowered, checked (eight
   dimensions) and predicted exactly, and persisted under
   ``process/candidates/<id>/``.
2. **baseline** — executable candidates sorted by exact T_pred under the
   current model; the best is adopted.
3. **calibration** (optional) — probes refit the cost model; the incumbent
   and the stored candidates are re-evaluated under the new model version
   before any comparison.
4. **tuning rounds** — a directed-cut certificate can end the search; else a
   bottleneck analysis yields a batch of strategies, local repair and
   resynthesis branches produce candidates, each is compared with the
   incumbent under the same model, and only a strictly better one (and, when
   measurement is enabled, a measured improvement) is adopted.
5. **finish** — results are published (schedule.xml/json, model.json,
   report.md, details.zip) and the run is finalised.

A checkpoint is written at every stage boundary and after every stored
candidate; ``resume`` restores it.
"""
from __future__ import annotations

import time
from dataclasses import dataclass, field, replace

from vericcl_b200.errors import (BudgetExhausted, InputValidationError, ScratchBudgetError, SemanticError,
                                 SolverError)
from vericcl_b200.execution.budget import BudgetManager
from vericcl_b200.execution.checkpoint import save_checkpoint
from vericcl_b200.execution.context import finalize_run
from vericcl_b200.execution.publication import publish_results
from vericcl_b200.performance.initial import initial_cost_model, model_context
from vericcl_b200.performance.model import CostModel
from vericcl_b200.performance.simulation import predict
from vericcl_b200.planner.parameters import initial_parameter_domain
from vericcl_b200.program.sidecar import to_sidecar
from vericcl_b200.solver.bounds import dependency_lower_bound
from vericcl_b200.synthesis import (Lowerer, synthesize, synthesize_allreduce_rs_ag,
                                    synthesize_reduce_scatter_dual)
from vericcl_b200.topology import load_topology
from vericcl_b200.utils.jsonio import atomic_write_json, atomic_write_text


@dataclass
class RunResult:
    status: str
    stop_reason: str
    best: dict | None
    rounds: list = field(default_factory=list)
    proof: dict | None = None
    timing: dict = field(default_factory=dict)
    issues: list = field(default_factory=list)
    recommendations: list = field(default_factory=list)

    def as_json(self):
        return {"status": self.status, "stop_reason": self.stop_reason, "best": self.best, "rounds": self.rounds,
                "proof": self.proof, "timing": self.timing, "issues": self.issues,
                "recommendations": self.recommendations}


def accept_candidate(incumbent, candidate, *, tolerance: float = 1e-9) -> bool:
    """Strictly better exact T_pred under the same model version, all required checks valid."""
    if candidate is None or not candidate.can_execute or candidate.t_pred_us is None:
        return False
    if incumbent is None:
        return True
    if candidate.prediction.model_version != incumbent.prediction.model_version:
        return False
    return candidate.t_pred_us < incumbent.t_pred_us * (1 - tolerance)


class PrimaryWorkflow:
    def __init__(self, request, ctx, *, purpose: str = "solve", tune: bool = False, model: CostModel | None = None,
                 verify_inputs: dict | None = None, probe_executor=None, measure=None, restored: dict | None = None,
                 trace_provider=None):
        self.request = request
        self.ctx = ctx
        self.purpose = purpose
        self.tune = tune
        self.topology = load_topology(request)
        self.model = model or initial_cost_model(request)
        self.verify_inputs = verify_inputs or {}
        self.probe_executor = probe_executor
        self.measure = measure
        self.trace_provider = trace_provider   # bundle -> measured trace report (timeline with XML origins) or None
        self.measured_rejects: set = set()
        self.failure_recommendations: list = []    # input changes derived from candidates that failed to lower
        budgets = dict(request.request_config["sketch"]["budgets"])
        self.budgets = BudgetManager(budgets, cpu_budget=request.solver.cpu_budget)
        self.candidates = []
        self.incumbent = None
        self.rounds = []
        self.proof = None
        self.stage_times = {}
        self.restored = restored
        if restored:
            snap = restored.get("budgets", {})
            self.budgets.consumed.update(snap.get("consumed", {}))
            self.budgets.restore_elapsed(snap.get("elapsed_s", 0.0) + restored.get("downtime_s", 0.0))

    # -- persistence ------------------------------------------------------------
    def store(self, bundle, tag: str) -> str:
        cid = "%s-%03d" % (tag, len(self.candidates))
        d = self.ctx.process / "candidates" / cid
        d.mkdir(parents=True, exist_ok=True)
        atomic_write_text(d / "schedule.xml", bundle.xml)
        atomic_write_json(d / "schedule.json", to_sidecar(bundle))
        atomic_write_json(d / "candidate.json", {"id": cid, "origin": bundle.origin, "t_pred_us": bundle.t_pred_us,
                                                 "model_version": bundle.prediction.model_version,
                                                 "slice_size_bytes": bundle.request.hyperparameters.slice_size_bytes,
                                                 "method": bundle.request.selected_synthesis_method,
                                                 "can_execute": bundle.can_execute})
        atomic_write_json(d / "checks.json", bundle.checks)
        bundle.candidate_id = cid
        self.candidates.append(bundle)
        self.ctx.emit("candidate_stored", id=cid, t_pred_us=bundle.t_pred_us, can_execute=bundle.can_execute)
        return cid

    def checkpoint(self, phase: str):
        state = {"incumbent": getattr(self.incumbent, "candidate_id", None),
                 "candidates": [getattr(b, "candidate_id", None) for b in self.candidates],
                 "rounds": self.rounds, "model_version": self.model.version, "purpose": self.purpose,
                 "tune": self.tune}
        files = []
        if self.incumbent is not None and getattr(self.incumbent, "candidate_id", None):
            cid = self.incumbent.candidate_id
            files = ["process/candidates/%s/schedule.xml" % cid, "process/candidates/%s/schedule.json" % cid]
        atomic_write_json(self.ctx.process / "models" / (self.model.version + ".json"), self.model.as_json())
        save_checkpoint(self.ctx, phase=phase, state=state, files=files, budgets=self.budgets.snapshot())

    # -- stages -------------------------------------------------------------------
    def history_candidates(self):
        """Isomorphic schedules from earlier runs, revalidated under the current request and model."""
        hist = self.request.request_config["sketch"]["history"]
        if not hist["schedule_reuse"]:
            return
        from pathlib import Path
        from vericcl_b200.solver.history import find_schedules
        index = Path(hist["schedule_index"])
        if not index.is_absolute():
            index = self.ctx.project_root / "examples" / self.ctx.case / index
        for entry in find_schedules(index, self.request, self.topology, tolerance=hist["relative_bandwidth_tolerance"],
                                    limit=hist["max_schedule_candidates"]):
            self.ctx.emit("history_candidate", t_pred_us=entry["t_pred_us"])
            # a reused XML has no sidecar: it is checked by the compiler and the chunk simulator
            from vericcl_b200.program.device import compile_xml
            try:
                compile_xml(entry["xml"])
            except SemanticError:
                continue
            atomic_write_text(self.ctx.process / "candidates" / ("history-%03d.xml" % len(self.candidates)),
                              entry["xml"])

    def save_history(self):
        hist = self.request.request_config["sketch"]["history"]
        if not hist["schedule_reuse"] or self.incumbent is None:
            return
        from pathlib import Path
        from vericcl_b200.solver.history import save_schedule
        index = Path(hist["schedule_index"])
        if not index.is_absolute():
            index = self.ctx.project_root / "examples" / self.ctx.case / index
        save_schedule(index, self.incumbent.request, self.topology, self.incumbent.xml, self.incumbent.t_pred_us)

    def initial_candidates(self):
        t0 = time.monotonic()
        self.history_candidates()
        with self.budgets.acquire("initial") as lease:
            if self.request.hyperparameters.slice_size_bytes is not None:
                choices = [None]
            else:
                try:
                    choices = initial_parameter_domain(self.request)[:4]
                except InputValidationError as error:
                    from vericcl_b200.program.recommendations import describe, recommend_for_domain
                    recs = recommend_for_domain(self.request)
                    if not recs:
                        raise
                    raise InputValidationError("%s; recommended: %s" % (error, describe(recs))) from error
            methods = [self.request.selected_synthesis_method]
            if not self.request.request_config["atom"]["manual"]["enabled"]:
                methods.append("constructive_trees" if methods[0] == "hierarchy" else "hierarchy")
            # cheapest lower bound first; a choice whose bound already reaches the best candidate is skipped
            bounded = []
            for choice in choices:
                req = self.request if choice is None else self.request.with_slice(choice.slice_size_bytes)
                bounded.append((float(dependency_lower_bound(req, self.topology, self.model)), choice, req))
            bounded.sort(key=lambda item: item[0])
            for bound, choice, req in bounded:
                channels = 1 if choice is None else choice.channels
                best = min((b.t_pred_us for b in self.candidates if b.t_pred_us is not None), default=None)
                if best is not None and bound >= best:
                    self.ctx.emit("choice_pruned", slice_size_bytes=req.hyperparameters.slice_size_bytes,
                                  lower_bound_us=bound, best_t_pred_us=best)
                    continue
                jobs = []
                for method in methods:
                    if method == "hierarchy" and not req.request_config["atom"]["manual"]["enabled"]:
                        # the two best hierarchy plans by coarse score, then the direct plan
                        from vericcl_b200.planner.hierarchy import enumerate_hierarchy_plans
                        jobs.extend((method, plan) for plan in enumerate_hierarchy_plans(req, self.topology, 2))
                    else:
                        jobs.append((method, None))
                for method, plan in jobs:
                    lease.check()
                    try:
                        bundle = synthesize(replace(req, selected_synthesis_method=method), self.model,
                                            channels=channels, plan=plan)
                    except (SemanticError, SolverError) as error:
                        self.ctx.emit("candidate_failed", method=method, error=str(error))
                        if isinstance(error, ScratchBudgetError):
                            self.failure_recommendations.append(
                                {"kind": "increase_scratch_budget", "priority": 1,
                                 "parameters": {"scratch_bytes_per_rank": error.needed_bytes},
                                 "reason_codes": ["scratch"], "requires_resolve": False})
                        continue
                    self.store(bundle, "initial")
                # candidates built from the AllGather schedule of the same slices: reversed (a ReduceScatter),
                # or reversed and then run forward (an AllReduce)
                dual = {"reduce_scatter": ("allgather_dual", synthesize_reduce_scatter_dual),
                        "allreduce": ("reduce_scatter_allgather", synthesize_allreduce_rs_ag)}.get(
                            req.collective.kind.value)
                if dual is not None and req.hyperparameters.slice_count % req.rank_count == 0:
                    lease.check()
                    try:
                        bundle = dual[1](req, self.model, channels=channels)
                    except (SemanticError, SolverError, InputValidationError) as error:
                        self.ctx.emit("candidate_failed", method=dual[0], error=str(error))
                    else:
                        self.store(bundle, "initial")
        self.stage_times["initial_s"] = time.monotonic() - t0
        self.checkpoint("initial_done")

    def reevaluate(self, bundle):
        """The same schedule predicted under the current model version."""
        if bundle.prediction.model_version == self.model.version:
            return bundle
        from vericcl_b200.program.native import build_executable
        executable = build_executable(bundle.program, bundle.storage, bundle.request, self.topology,
                                      model_context(bundle.request))
        new = replace(bundle, executable=executable, prediction=predict(executable, self.model, exact=True))
        new.checks = dict(bundle.checks)
        new.checks["prediction"] = {"status": "valid" if new.prediction.t_pred_us is not None else "invalid",
                                    "detail": {"t_pred_us": new.prediction.t_pred_us}}
        if hasattr(bundle, "candidate_id"):
            new.candidate_id = bundle.candidate_id
        return new

    def baseline(self):
        ready = [self.reevaluate(b) for b in self.candidates]
        ready = [b for b in ready if b.can_execute]
        if not ready:
            return None
        ready.sort(key=lambda b: b.t_pred_us)
        self.adopt(ready[0], reason="baseline")
        return ready[0]

    def adopt(self, bundle, reason: str):
        self.incumbent = bundle
        if not hasattr(bundle, "candidate_id"):
            self.store(bundle, "adopted")
        d = self.ctx.process / "best"
        atomic_write_json(d / "accepted.json", {"id": bundle.candidate_id, "t_pred_us": bundle.t_pred_us,
                                                "reason": reason, "model_version": self.model.version})
        self.ctx.emit("candidate_adopted", id=bundle.candidate_id, t_pred_us=bundle.t_pred_us, reason=reason)

    def _calibration_identity(self):
        """Cache key of a calibration: the GPUs (UUIDs), driver, datatype, reduction and rank count."""
        from vericcl_b200.execution.transport import machine_inventory
        from vericcl_b200.online.campaign import calibration_identity
        inv = machine_inventory()
        return calibration_identity(self.request, [g["uuid"] for g in inv["gpus"]], inv.get("driver") or "")

    def reuse_calibration(self) -> bool:
        """Adopt a cached calibrated model of the same machine and workload when one is fresh enough."""
        from vericcl_b200.online.campaign import lookup_calibration
        hist = self.request.request_config["sketch"]["history"]
        if not hist.get("calibration_reuse"):
            return False
        cached = lookup_calibration(hist["calibration_index"], self._calibration_identity(),
                                    hist["calibration_max_age_s"])
        if cached is None or dict(cached.context) != dict(self.model.context):
            return False
        self.model = cached
        self.ctx.emit("calibration_reused", version=cached.version)
        if self.incumbent is not None:
            self.incumbent = self.reevaluate(self.incumbent)
        return True

    def calibration(self):
        from vericcl_b200.online.campaign import run_calibration, save_calibration
        if self.reuse_calibration():
            return True
        if self.probe_executor is None:
            self.ctx.emit("calibration_skipped", reason="no probe executor (GPU runtime) available")
            return False
        t0 = time.monotonic()
        try:
            with self.budgets.acquire("online") as lease:
                model, diff, report = run_calibration(self.request, self.topology, self.model, self.probe_executor,
                                                      lease=lease, record_dir=self.ctx.process / "models")
        except BudgetExhausted as error:
            self.ctx.emit("calibration_stopped", reason=str(error))
            return False
        self.stage_times["calibration_s"] = time.monotonic() - t0
        atomic_write_json(self.ctx.process / "reports" / "calibration.json", report)
        if model.version == self.model.version:
            return False
        self.model = model
        self.ctx.emit("model_published", version=model.version, components=len(diff))
        hist = self.request.request_config["sketch"]["history"]
        if hist.get("calibration_reuse"):
            save_calibration(hist["calibration_index"], self._calibration_identity(), model)
        if self.incumbent is not None:
            self.incumbent = self.reevaluate(self.incumbent)
        return True

    def tuning(self):
        from vericcl_b200.tuning.resynthesis import branches, resynthesize_branch
        from vericcl_b200.tuning.strategies import solve_repair
        from vericcl_b200.verification.bottlenecks import analyze
        from vericcl_b200.verification.global_bound import certify_global_cut, check_global_cut
        rounds = self.request.request_config["sketch"]["budgets"].get("max_tuning_rounds") or 0
        batch = self.request.request_config["sketch"]["repair"]["analysis_batch_size"]
        for index in range(rounds):
            if self.incumbent is None:
                return "no incumbent"
            self.budgets.new_round()
            record = {"round": index, "start_t_pred_us": self.incumbent.t_pred_us}
            bound = certify_global_cut(self.incumbent.request, self.topology, self.model)
            if bound is not None:
                record["cut_lower_bound_us"] = bound.lower_bound_us
                if check_global_cut(bound, self.incumbent.t_pred_us):
                    self.proof = {"kind": "directed_cut", "lower_bound_us": bound.lower_bound_us,
                                  "subset": list(bound.subset), "exact": list(bound.exact)}
                    record["result"] = "certified optimal"
                    self.rounds.append(record)
                    return "no-improvement proof"
            try:
                trace = None
                if self.trace_provider is not None:
                    try:
                        trace = self.trace_provider(self.incumbent)
                    except Exception as error:   # a failed capture leaves the round to the model alone
                        self.ctx.emit("trace_failed", round=index, reason=str(error))
                    if trace is not None:
                        record["trace_span_us"] = trace.get("global_span_us")
                with self.budgets.acquire("repair") as lease:
                    analysis = analyze(self.incumbent, self.model, batch_size=batch, trace=trace)
                    record["causes"] = [c.kind for c in analysis.causes][:20]
                    record["strategies"] = [s.as_json() for s in analysis.strategies]
                    lower = Lowerer(self.incumbent.request, self.topology, self.model)
                    outcome = solve_repair(self.incumbent, analysis.strategies, lower=lower, lease=lease,
                                           batch_size=self.request.request_config["sketch"]["repair"][
                                               "candidate_batch_size"])
                    candidates = [outcome.best] if outcome.improved else []
                    for branch in branches(self.incumbent.request, self.incumbent):
                        lease.check()
                        alt = resynthesize_branch(self.incumbent.request, branch, self.model, lease=lease)
                        if alt is not None:
                            self.store(alt, "resynth")
                            candidates.append(alt)
            except BudgetExhausted:
                record["result"] = "repair budget exhausted"
                self.rounds.append(record)
                return "repair budget exhausted"
            # a candidate the paired measurement already turned down is not measured again
            fresh = [c for c in candidates if accept_candidate(self.incumbent, c)
                     and self._xml_digest(c) not in self.measured_rejects]
            if len(fresh) < len([c for c in candidates if accept_candidate(self.incumbent, c)]):
                record["skipped_rejected"] = True
            best = min(fresh, key=lambda c: c.t_pred_us, default=None)
            if best is not None and self.measure is not None:
                verdict = self.measure(self.incumbent, best)
                record["measured"] = verdict.__dict__ if hasattr(verdict, "__dict__") else verdict
                if not getattr(verdict, "accepted", False):
                    self.measured_rejects.add(self._xml_digest(best))
                    best = None
            if best is None:
                record["result"] = "no improvement"
                record["scope_proof"] = self.scope_proof(index, analysis.strategies)
                self.rounds.append(record)
                self.checkpoint("round_%d" % index)
                continue
            self.adopt(best, reason="round %d" % index)
            record["result"] = "improved"
            record["t_pred_us"] = best.t_pred_us
            self.rounds.append(record)
            self.checkpoint("round_%d" % index)
        return "round limit"

    def scope_proof(self, index: int, strategies) -> dict:
        """Certify (and independently check) that no variant of this round's strategies beats the incumbent."""
        from vericcl_b200.verification.proof_check import certify_scope, check_no_improvement
        if not strategies or self.incumbent.network is None or self.incumbent.prediction is None:
            return {"status": "not_applicable"}
        lower = Lowerer(self.incumbent.request, self.topology, self.model)
        try:
            cert = certify_scope(self.incumbent, strategies, self.model, lower=lower)
            checked = check_no_improvement(cert, self.incumbent, strategies, self.model, lower=lower)
        except SemanticError as error:
            return {"status": "not_certified", "reason": str(error)}
        path = atomic_write_json(self.ctx.process / "proofs" / ("round_%d.json" % index), cert)
        self.ctx.emit("scope_proof", round=index, status=checked.status, form="bound" if cert["bound"] else "leaves")
        return {"status": checked.status, "form": "bound" if cert["bound"] else "leaves",
                "checked_leaves": checked.checked_leaves, "certificate": str(path.relative_to(self.ctx.directory))}

    @staticmethod
    def _xml_digest(bundle) -> str:
        import hashlib
        return hashlib.sha256(bundle.xml.encode()).hexdigest()

    def run(self) -> RunResult:
        t0 = time.monotonic()
        self.ctx.emit("workflow_started", purpose=self.purpose, tune=self.tune)
        stop = "finished"
        try:
            if self.purpose == "calibrate":
                changed = self.calibration()
                stop = "calibrated" if changed else "calibration produced no qualified component"
            else:
                if self.purpose == "verify":
                    from vericcl_b200.program.sidecar import bundle_from_sidecar
                    bundle = bundle_from_sidecar(self.request, self.topology, self.verify_inputs["xml"],
                                                 self.verify_inputs["sidecar"], self.model)
                    self.store(bundle, "verify")
                elif self.restored:
                    self.restore_candidates()
                else:
                    self.initial_candidates()
                self.baseline()
                cal = self.request.request_config["sketch"]["calibration"]["enabled"]
                if cal:
                    self.calibration()
                self.checkpoint("baseline")
                if self.purpose == "solve" or self.tune:
                    stop = self.tuning()
                else:
                    stop = "verified"
        except BudgetExhausted as error:
            stop = "budget: %s" % error
        self.stage_times["total_s"] = time.monotonic() - t0
        self.save_history()
        best = None
        if self.incumbent is not None:
            best = {"id": self.incumbent.candidate_id, "t_pred_us": self.incumbent.t_pred_us,
                    "model_version": self.model.version, "origin": self.incumbent.origin,
                    "checks": self.incumbent.checks,
                    "slice_size_bytes": self.incumbent.request.hyperparameters.slice_size_bytes}
        status = "ok" if (best is not None or self.purpose == "calibrate") else "no_candidate"
        result = RunResult(status, stop, best, self.rounds, self.proof, self.stage_times,
                           recommendations=self.recommendations())
        publish_results(self.ctx, xml=self.incumbent.xml if self.incumbent else None,
                        sidecar=to_sidecar(self.incumbent) if self.incumbent else None,
                        model=self.model.as_json(), result=result.as_json(), best=best)
        self.ctx.update_run_json(best=best, effective_request=dict(self.request.request_config),
                                 value_sources=dict(self.request.value_sources),
                                 size_accounting=dict(self.request.size_accounting), timing=self.stage_times)
        self.checkpoint("finished")
        finalize_run(self.ctx, result.as_json())
        return result

    def recommendations(self) -> list:
        """Input changes for candidates that failed their launch or storage check (none when one runs)."""
        if self.incumbent is not None and self.incumbent.can_execute:
            return []
        from vericcl_b200.program.recommendations import merge, recommend_for_program
        groups = [recommend_for_program(b.program, b.request, b.checks or {}) for b in self.candidates
                  if not b.can_execute and b.program is not None]
        return merge(groups + [self.failure_recommendations])

    def restore_candidates(self):
        from vericcl_b200.program.sidecar import bundle_from_sidecar
        from vericcl_b200.utils.jsonio import strict_load
        ids = [c for c in self.restored["state"].get("candidates", []) if c]
        for cid in ids:
            d = self.ctx.process / "candidates" / cid
            try:
                bundle = bundle_from_sidecar(self.request, self.topology, (d / "schedule.xml").read_text(),
                                             strict_load(d / "schedule.json"), self.model)
            except (OSError, SemanticError):
                continue
            bundle.candidate_id = cid
            self.candidates.append(bundle)
        if not self.candidates:
            self.initial_candidates()
