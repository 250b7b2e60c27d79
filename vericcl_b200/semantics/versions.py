"""Version replay: the "semantic" admission check on an executable program.

A program is a list of per-rank instructions that read and write
``(rank, buffer, offset)`` slots.  ``replay`` executes the instructions in a
dependency-respecting order over symbolic values (contributor sets), checks
that every reduction combines disjoint contributor sets at the same logical
index, and finally that every required output slot holds exactly the required
contributor set (reference: vericcl/semantics/version_schedule.py:138-174 and
vericcl/xml/v5_lower.py:228-243).
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Mapping

from vericcl_b200.semantics.collective import CollectiveKind, CollectiveSpec, input_ranks, required_outputs


@dataclass(frozen=True)
class SymbolicValue:
    contributors: frozenset
    scaled: bool = False


def initial_state(spec: CollectiveSpec, rank_count: int, slice_count: int) -> dict:
    """Symbolic contents of the input buffers before execution."""
    state = {}
    for rank in input_ranks(spec, rank_count):
        for index in range(slice_count):
            value = SymbolicValue(frozenset({rank * slice_count + index}))
            state[(rank, "i", index)] = value
            for alias in input_aliases(spec, rank_count, slice_count, rank, index):
                state[alias] = value
    return state


def input_aliases(spec, rank_count, slice_count, rank, index):
    """Other buffer coordinates that name the same memory as input slot ``index`` (in-place layouts)."""
    if not spec.inplace:
        return ()
    if spec.kind is CollectiveKind.ALL_GATHER:
        return ((rank, "o", rank * slice_count + index),)
    if spec.kind is CollectiveKind.REDUCE_SCATTER:
        q = slice_count // rank_count
        if rank * q <= index < (rank + 1) * q:
            return ((rank, "o", index - rank * q),)
        return ()
    return ((rank, "o", index),)


def canonical(spec, rank_count, slice_count, rank, buffer, offset):
    """Map an in-place alias to one canonical coordinate."""
    if not spec.inplace or buffer == "s":
        return (rank, buffer, offset)
    if spec.kind is CollectiveKind.ALL_GATHER:
        return (rank, "o", rank * slice_count + offset) if buffer == "i" else (rank, "o", offset)
    if spec.kind is CollectiveKind.REDUCE_SCATTER:
        q = slice_count // rank_count
        return (rank, "i", offset + rank * q) if buffer == "o" else (rank, "i", offset)
    return (rank, "o", offset)


def check_outputs(spec: CollectiveSpec, rank_count: int, slice_count: int, state: Mapping) -> list:
    """Return a list of human-readable mismatches (empty when valid)."""
    problems = []
    for slot, expected in sorted(required_outputs(spec, rank_count, slice_count).items()):
        key = canonical(spec, rank_count, slice_count, slot.rank, "o", slot.offset)
        value = state.get(key)
        if value is None:
            problems.append("output %d:%d is never written" % (slot.rank, slot.offset))
        elif value.contributors != expected:
            problems.append("output %d:%d holds %s, expected %s" % (slot.rank, slot.offset,
                                                                    sorted(value.contributors), sorted(expected)))
    return problems
