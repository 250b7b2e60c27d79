"""Structure and partition branches: full resynthesis inside the repair lease.

``structure`` switches the synthesis method (hierarchy ↔ constructive_trees,
or the direct plan); ``partition`` changes the slice size (doubling or
halving N within the legal parameter domain).  Both rerun the whole initial
pipeline and are compared with the incumbent under the same model
(reference: vericcl/tuning/resynthesis.py:14-88).
"""
from __future__ import annotations

from dataclasses import dataclass, replace

from vericcl_b200.errors import BudgetExhausted, SemanticError, SolverError


@dataclass(frozen=True)
class ResynthesisRequest:
    kind: str              # structure | partition
    method: str | None = None
    slice_size_bytes: int | None = None


def branches(request, incumbent):
    out = []
    current = request.selected_synthesis_method
    for method in ("hierarchy", "constructive_trees"):
        if method != current:
            out.append(ResynthesisRequest("structure", method=method))
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
    if branch.kind == "structure":
        req = replace(request, selected_synthesis_method=branch.method)
    elif branch.kind == "partition":
        req = request.with_slice(branch.slice_size_bytes)
    try:
        return synthesize(req, model, channels=channels)
    except (SemanticError, SolverError, BudgetExhausted):
        return None
