"""Resolved request records produced by :func:`vericcl_b200.input.loader.load_request`.

Field names follow the reference's ``ResolvedInput`` (vericcl/input/models.py:72-87)
so that downstream stages read the same facts.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Mapping, Optional, Tuple

from vericcl_b200.semantics.collective import CollectiveSpec


@dataclass(frozen=True)
class Hyperparameters:
    total_size_bytes: int
    slice_size_bytes: Optional[int]
    reference_slice_size_bytes: Optional[int] = None

    @property
    def slice_count(self) -> Optional[int]:
        return None if self.slice_size_bytes is None else self.total_size_bytes // self.slice_size_bytes

    def with_slice(self, slice_size_bytes: int) -> "Hyperparameters":
        return Hyperparameters(self.total_size_bytes, slice_size_bytes, self.reference_slice_size_bytes)


@dataclass(frozen=True)
class SolverConfig:
    backend: str = "highs"
    per_model_timeout_s: float = 60.0
    cpu_budget: int = 1
    max_threads_per_model: int = 12
    max_parallel_models: int = 1
    max_channels: int = 7
    solver_seed: int = 0
    mip_gap: float = 0.0
    require_proven_optimal: bool = False


@dataclass(frozen=True)
class ForbiddenTransfer:
    slice_id: int
    src_rank: int
    dst_rank: int
    stage_id: int


@dataclass(frozen=True)
class AtomConstraints:
    stage_num: Optional[int]
    forbidden_transfers: Tuple[ForbiddenTransfer, ...] = ()


@dataclass(frozen=True)
class ResolvedInput:
    collective: CollectiveSpec
    hyperparameters: Hyperparameters
    solver: SolverConfig
    atom_constraints: AtomConstraints
    rank_count: int
    selected_synthesis_method: str
    input_sha256: str
    request_config: Mapping[str, object] = field(default_factory=dict)
    value_sources: Mapping[str, object] = field(default_factory=dict)
    size_accounting: Mapping[str, object] = field(default_factory=dict)
    purpose: str = "solve"

    @property
    def element_bytes(self) -> int:
        from vericcl_b200.input.schema import DATATYPE_BYTES
        return DATATYPE_BYTES[self.collective.datatype]

    def with_slice(self, slice_size_bytes: int) -> "ResolvedInput":
        """Return a copy bound to another slice size (parameter-domain search)."""
        from dataclasses import replace
        hyper = self.hyperparameters.with_slice(slice_size_bytes)
        accounting = dict(self.size_accounting)
        accounting["slice_size_bytes"] = slice_size_bytes
        accounting["slices_per_rank"] = hyper.slice_count
        return replace(self, hyperparameters=hyper, size_accounting=accounting)
