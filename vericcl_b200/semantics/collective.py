"""Collective kinds and their required outputs.

An *original slice* is identified by ``slice_id = src_rank * N + index`` where
N is the number of slices per rank (reference: vericcl/semantics/slice.py:9).
``required_outputs`` maps every output slot ``(rank, offset)`` to the exact
set of original slices that must be combined there (reference:
vericcl/semantics/collective.py:95-172).  AllGather output slot offsets are
the global slice id; ReduceScatter/Scatter/AllToAll need N divisible by P.
"""
from __future__ import annotations

from dataclasses import dataclass
from enum import Enum
from types import MappingProxyType
from typing import FrozenSet, Mapping, Optional

from vericcl_b200.errors import SemanticError


class CollectiveKind(str, Enum):
    BROADCAST = "broadcast"
    REDUCE = "reduce"
    SCATTER = "scatter"
    GATHER = "gather"
    ALL_GATHER = "allgather"
    ALL_REDUCE = "allreduce"
    ALL_TO_ALL = "alltoall"
    REDUCE_SCATTER = "reduce_scatter"


ROOTED = frozenset({CollectiveKind.BROADCAST, CollectiveKind.REDUCE, CollectiveKind.SCATTER,
                    CollectiveKind.GATHER})
REDUCING = frozenset({CollectiveKind.REDUCE, CollectiveKind.ALL_REDUCE, CollectiveKind.REDUCE_SCATTER})
PARTITIONED = frozenset({CollectiveKind.SCATTER, CollectiveKind.ALL_TO_ALL, CollectiveKind.REDUCE_SCATTER})


@dataclass(frozen=True)
class CollectiveSpec:
    kind: CollectiveKind
    datatype: str = "float32"
    reduction_op: Optional[str] = None
    root: Optional[int] = None
    inplace: bool = False
    scale: Optional[float] = None

    @property
    def reducing(self) -> bool:
        return self.kind in REDUCING


@dataclass(frozen=True, order=True)
class OutputSlot:
    rank: int
    offset: int


def source_rank(slice_id: int, slice_count: int) -> int:
    return slice_id // slice_count


def validate_problem(spec: CollectiveSpec, rank_count: int, slice_count: int) -> None:
    if not isinstance(spec, CollectiveSpec):
        raise SemanticError("spec must be a CollectiveSpec")
    for name, value in (("rank_count", rank_count), ("slice_count", slice_count)):
        if isinstance(value, bool) or not isinstance(value, int) or value < 1:
            raise SemanticError(name + " must be a positive integer")
    if spec.kind in ROOTED:
        if isinstance(spec.root, bool) or not isinstance(spec.root, int) or not 0 <= spec.root < rank_count:
            raise SemanticError("%s requires a root inside the rank range" % spec.kind.value)
    elif spec.root is not None:
        raise SemanticError("%s must not define a root" % spec.kind.value)
    if spec.kind in PARTITIONED and slice_count % rank_count:
        raise SemanticError("slice count must be divisible by the rank count for " + spec.kind.value)


def _reduced(index: int, rank_count: int, slice_count: int) -> FrozenSet[int]:
    return frozenset(rank * slice_count + index for rank in range(rank_count))


def required_outputs(spec: CollectiveSpec, rank_count: int, slice_count: int) -> Mapping[OutputSlot, FrozenSet[int]]:
    """Return ``{OutputSlot: contributor set}`` for the collective."""
    validate_problem(spec, rank_count, slice_count)
    n, p = slice_count, rank_count
    out = {}
    kind = spec.kind
    if kind is CollectiveKind.BROADCAST:
        for rank in range(p):
            for index in range(n):
                out[OutputSlot(rank, index)] = frozenset({spec.root * n + index})
    elif kind is CollectiveKind.REDUCE:
        for index in range(n):
            out[OutputSlot(spec.root, index)] = _reduced(index, p, n)
    elif kind is CollectiveKind.SCATTER:
        q = n // p
        for index in range(n):
            out[OutputSlot(index // q, index % q)] = frozenset({spec.root * n + index})
    elif kind is CollectiveKind.GATHER:
        for src in range(p):
            for index in range(n):
                out[OutputSlot(spec.root, src * n + index)] = frozenset({src * n + index})
    elif kind is CollectiveKind.ALL_GATHER:
        for rank in range(p):
            for sid in range(p * n):
                out[OutputSlot(rank, sid)] = frozenset({sid})
    elif kind is CollectiveKind.ALL_REDUCE:
        for rank in range(p):
            for index in range(n):
                out[OutputSlot(rank, index)] = _reduced(index, p, n)
    elif kind is CollectiveKind.ALL_TO_ALL:
        q = n // p
        for src in range(p):
            for index in range(n):
                dst = index // q
                out[OutputSlot(dst, src * q + index % q)] = frozenset({src * n + index})
    elif kind is CollectiveKind.REDUCE_SCATTER:
        q = n // p
        for index in range(n):
            out[OutputSlot(index // q, index % q)] = _reduced(index, p, n)
    else:  # pragma: no cover - enum is closed
        raise SemanticError("unsupported collective")
    return MappingProxyType(out)


def input_ranks(spec: CollectiveSpec, rank_count: int):
    """Ranks that hold original input slices."""
    if spec.kind in (CollectiveKind.BROADCAST, CollectiveKind.SCATTER):
        return (spec.root,)
    return tuple(range(rank_count))


def output_slot_count(spec: CollectiveSpec, rank_count: int, slice_count: int, rank: int) -> int:
    slots = [slot.offset for slot in required_outputs(spec, rank_count, slice_count) if slot.rank == rank]
    return max(slots) + 1 if slots else 0


def runtime_chunks(spec: CollectiveSpec, rank_count: int, slice_count: int) -> int:
    """MSCCL ``nchunksperloop``: chunks of the runtime buffer per loop.

    AllGather/Gather runtime buffers are P×M, the others M (reference:
    vericcl/xml/v5_program.py:91, runtime/execution/schedule_store.cc:37).
    """
    if spec.kind in (CollectiveKind.ALL_GATHER, CollectiveKind.GATHER):
        return slice_count * rank_count
    return slice_count
