"""Structure and partition branches: full resynthesis inside the repair lease.

``structure`` switches the synthesis method (hierarchy ↔ constructive_trees,
or the direct plan) or, within the hierarchy method, the grouping: another
partition, or gateways instead of per-slice rails (or back) for the
inter-group stage; ``partition`` changes the slice size (doubling or halving
N within the legal parameter domain).  All rerun the whole initial pipeline
and are compared with the incumbent under the same model (reference:
vericcl/tuning/resynthesis.py:14-88).
"""
from __future__ import annotations

from dataclasses import dataclass, replace

from vericcl_b200.errors import BudgetExhausted, SemanticError, SolverError


@dataclass(frozen=True)
class ResynthesisRequest:
    kind: str              # structure | partition
    method: str | None = None
    slice_size_bytes: int | None = None
    plan_reason: str | None = None     # a specific hierarchy plan (its grouping and rail mode)


def branches(request, incumbent):
    out = []
    current = request.selected_synthesis_method
    for method in ("hierarchy", "constructive_trees"):
        if method != current:
            out.append(ResynthesisRequest("structure", method=method))
    if current == "hierarchy" and not request.request_config["atom"]["manual"]["enabled"]:
        from vericcl_b200.planner.group_search import CandidateStream
        from vericcl_b200.topology import load_topology
        used = getattr(getattr(incumbent, "plan", None), "reason", None)
        for plan in list(CandidateStream(request, load_topology(request)))[:4]:
            if plan.reason != used:
                out.append(ResynthesisRequest("structure", method="hierarchy", plan_reason=plan.reason))
    m = request.hyperparameters.total_size_bytes
    s = request.hyperparameters.slice_size_bytes
    for factor in (2, 0.5):
        new = int(s * factor)
        if new >= request.element_bytes and m % new == 0 and new % request.element_bytes == 0 and new != s:
            out.append(ResynthesisRequest("partition", slice_size_bytes=new))
    return out


def resynthesize_branch(request, branch: ResynthesisRequest, model, *, lease=None, channels: int = 1):
    from vericcl_b200.synthesis import synthesize
    if lease is not None:
        lease.check()
    req = request
    plan = None
    if branch.kind == "structure":
        req = replace(request, selected_synthesis_method=branch.method)
        if branch.plan_reason is not None:
            from vericcl_b200.planner.group_search import CandidateStream
            from vericcl_b200.topology import load_topology
            plan = next((p for p in CandidateStream(req, load_topology(req)) if p.reason == branch.plan_reason), None)
            if plan is None:
                return None
    elif branch.kind == "partition":
        req = request.with_slice(branch.slice_size_bytes)
    try:
        return synthesize(req, model, channels=channels, plan=plan)
    except (SemanticError, SolverError, BudgetExhausted):
        return None
