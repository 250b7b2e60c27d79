"""Collective semantics (reference layer L1)."""
from .collective import (CollectiveKind, CollectiveSpec, OutputSlot, required_outputs, runtime_chunks,
                         validate_problem, input_ranks, source_rank)

__all__ = ["CollectiveKind", "CollectiveSpec", "OutputSlot", "required_outputs", "runtime_chunks",
           "validate_problem", "input_ranks", "source_rank"]
