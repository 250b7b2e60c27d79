"""The ``hierarchy`` method's plan choice: group stages around an inter-group stage.

For AllReduce over groups G_1..G_k: (0) reduce each slice inside every group
into the group's inter-group member, (1) reduce across groups into the owner
group's member, (2) broadcast across groups, (3) broadcast inside every group.
AllGather uses the last two stages per source slice.  Which partitions,
members (rails or gateways) and in which order they are tried is decided by
:mod:`vericcl_b200.planner.group_search` (reference:
vericcl/planner/group_search.py:547 ``plan_hierarchy``).  With a single
group the direct plan is returned.
"""
from __future__ import annotations

from vericcl_b200.planner.direct import build_direct_plan
from vericcl_b200.planner.group_search import CandidateStream, partition_candidates  # noqa: F401


def plan_hierarchy(request, topology):
    """The hierarchy plan with the best coarse score whose stages all have route trees, else the direct plan."""
    from vericcl_b200.errors import SemanticError
    from vericcl_b200.solver.demands import build_demands
    for plan in CandidateStream(request, topology):
        try:
            build_demands(plan, topology)
        except SemanticError:
            continue
        return plan
    return build_direct_plan(request, topology, reason="single_group")


def enumerate_hierarchy_plans(request, topology, limit: int | None = None):
    """Hierarchy candidates in coarse-score order (lazy, at most ``limit``), followed by the direct plan."""
    for count, plan in enumerate(CandidateStream(request, topology)):
        if limit is not None and count >= limit:
            break
        yield plan
    yield build_direct_plan(request, topology, reason="direct_fallback")
