"""Logical stage plans: DAGs of local collectives on rank groups.

A :class:`PlanNode` is one local collective (reduce, broadcast, gather, …) on
a communication group with explicit input and output *state interfaces*:
``{(rank, logical offset): contributor set}``.  Edges carry the interface
between a producer and a consumer node.  The solver turns each node into
transfers; the composer times them (reference: vericcl/planner/model.py:68-194).
"""
from __future__ import annotations

from dataclasses import dataclass, field
from enum import Enum
from types import MappingProxyType
from typing import Mapping, Tuple

from vericcl_b200.errors import SemanticError
from vericcl_b200.semantics.collective import CollectiveKind, CollectiveSpec, OutputSlot


class PlanningMode(str, Enum):
    DIRECT = "direct"
    HIERARCHY = "hierarchy"
    MANUAL = "manual"
    TREES = "constructive_trees"


@dataclass(frozen=True)
class StageInterface:
    values: Mapping[OutputSlot, frozenset]

    def __post_init__(self):
        object.__setattr__(self, "values", MappingProxyType(dict(self.values)))

    def ranks(self):
        return sorted({slot.rank for slot in self.values})


@dataclass(frozen=True)
class PlanNode:
    node_id: str
    stage_id: int
    kind: CollectiveKind
    group: Tuple[int, ...]
    root: int | None
    logical_input: StageInterface
    logical_output: StageInterface
    relay_ranks: Tuple[int, ...] = ()
    forbidden_edges: frozenset = frozenset()   # {(slice_id, src, dst)}

    @property
    def reducing(self) -> bool:
        return self.kind in (CollectiveKind.REDUCE, CollectiveKind.REDUCE_SCATTER, CollectiveKind.ALL_REDUCE)


@dataclass(frozen=True)
class PlanEdge:
    producer_id: str
    consumer_id: str


@dataclass(frozen=True)
class PlanDAG:
    collective: CollectiveSpec
    rank_count: int
    slice_count: int
    nodes: Tuple[PlanNode, ...]
    edges: Tuple[PlanEdge, ...]
    mode: PlanningMode
    reason: str = ""
    metadata: Mapping[str, object] = field(default_factory=dict)

    def __post_init__(self):
        ids = [n.node_id for n in self.nodes]
        if len(set(ids)) != len(ids):
            raise SemanticError("duplicate plan node id")
        known = set(ids)
        for edge in self.edges:
            if edge.producer_id not in known or edge.consumer_id not in known:
                raise SemanticError("plan edge names an unknown node")

    def predecessors(self, node_id: str):
        return sorted(e.producer_id for e in self.edges if e.consumer_id == node_id)

    def node(self, node_id: str) -> PlanNode:
        for n in self.nodes:
            if n.node_id == node_id:
                return n
        raise SemanticError("unknown plan node " + node_id)

    def stage_count(self) -> int:
        return max((n.stage_id for n in self.nodes), default=-1) + 1
