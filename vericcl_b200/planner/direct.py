"""Direct (flat) plans: one stage pair over the whole rank set.

* AllReduce: for every logical slice a ReduceScatter-style reduction into its
  owner followed by a Broadcast from the owner (reference:
  vericcl/planner/direct.py:280-371).  Owners are assigned in contiguous
  blocks when N is divisible by P, otherwise round-robin.
* AllGather: every original slice is broadcast from its source rank.
* Broadcast / Reduce / ReduceScatter / AllToAll / Scatter / Gather: one node
  per logical slice with the matching local collective.
"""
from __future__ import annotations

from vericcl_b200.errors import InputValidationError
from vericcl_b200.planner.model import PlanDAG, PlanEdge, PlanNode, PlanningMode, StageInterface
from vericcl_b200.semantics.collective import CollectiveKind, OutputSlot, required_outputs


def slice_owner(index: int, slice_count: int, rank_count: int):
    """(owner rank, offset) of a reduced slice for AllReduce/ReduceScatter."""
    if slice_count % rank_count:
        return index % rank_count, index // rank_count
    q = slice_count // rank_count
    return index // q, index % q


def _reduce_input(p, n, index):
    return StageInterface({OutputSlot(r, index): frozenset({r * n + index}) for r in range(p)})


def build_direct_plan(request, topology=None, *, reason: str = "direct_request") -> PlanDAG:
    spec = request.collective
    p = request.rank_count
    n = request.hyperparameters.slice_count
    if n is None:
        raise InputValidationError("a direct plan needs a resolved slice size")
    group = tuple(range(p))
    nodes, edges = [], []
    kind = spec.kind
    if kind is CollectiveKind.ALL_REDUCE:
        gathers = []
        for index in range(n):
            owner, _ = slice_owner(index, n, p)
            full = frozenset(r * n + index for r in range(p))
            inter = StageInterface({OutputSlot(owner, index): full})
            rs, ag = "allreduce-rs-a%08d" % index, "allreduce-ag-a%08d" % index
            nodes.append(PlanNode(rs, 0, CollectiveKind.REDUCE, group, owner, _reduce_input(p, n, index), inter))
            gathers.append(PlanNode(ag, 1, CollectiveKind.BROADCAST, group, owner, inter,
                                    StageInterface({OutputSlot(r, index): full for r in range(p)})))
            edges.append(PlanEdge(rs, ag))
        nodes.extend(gathers)
    elif kind is CollectiveKind.ALL_GATHER:
        for src in range(p):
            for index in range(n):
                sid = src * n + index
                nodes.append(PlanNode("allgather-bc-s%08d" % sid, 0, CollectiveKind.BROADCAST, group, src,
                                      StageInterface({OutputSlot(src, index): frozenset({sid})}),
                                      StageInterface({OutputSlot(r, sid): frozenset({sid}) for r in range(p)})))
    elif kind is CollectiveKind.BROADCAST:
        for index in range(n):
            sid = spec.root * n + index
            nodes.append(PlanNode("broadcast-a%08d" % index, 0, CollectiveKind.BROADCAST, group, spec.root,
                                  StageInterface({OutputSlot(spec.root, index): frozenset({sid})}),
                                  StageInterface({OutputSlot(r, index): frozenset({sid}) for r in range(p)})))
    elif kind in (CollectiveKind.REDUCE, CollectiveKind.REDUCE_SCATTER):
        outputs = required_outputs(spec, p, n)
        for slot, contributors in sorted(outputs.items()):
            index = min(contributors) % n
            nodes.append(PlanNode("%s-a%08d" % (kind.value, index), 0, CollectiveKind.REDUCE, group, slot.rank,
                                  _reduce_input(p, n, index), StageInterface({slot: contributors})))
    elif kind in (CollectiveKind.ALL_TO_ALL, CollectiveKind.SCATTER, CollectiveKind.GATHER):
        outputs = required_outputs(spec, p, n)
        for slot, contributors in sorted(outputs.items()):
            sid = min(contributors)
            src = sid // n
            nodes.append(PlanNode("%s-s%08d" % (kind.value, sid), 0, CollectiveKind.BROADCAST, (src, slot.rank),
                                  src, StageInterface({OutputSlot(src, sid % n): contributors}),
                                  StageInterface({slot: contributors})))
    else:  # pragma: no cover
        raise InputValidationError("unsupported collective " + kind.value)
    return PlanDAG(spec, p, n, tuple(nodes), tuple(edges), PlanningMode.DIRECT, reason)
