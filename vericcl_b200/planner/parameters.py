"""Parameter domain: legal (slice size S, channel count C) choices.

For every channel count 1..max_channels the domain bounds N = M/S from both
sides: N must be a whole number of slices of whole elements, divisible by P
for partitioned collectives, and small enough that the program fits the
runtime limits (steps per TB, TBs per rank, dependency ids, buffer offsets)
and the scratch budget.  The reference additionally bounds S by the MSCCL
Simple-protocol FIFO slot (NCCL_BUFFSIZE); this runtime pulls directly from
peer buffers, so the bound it keeps is the interpreter's: every chunk must be
a whole number of 16-byte vectors.  Candidates are ordered largest legal N
(smallest S) first, like the reference (vericcl/planner/parameters.py:60-219).
"""
from __future__ import annotations

from dataclasses import dataclass

from vericcl_b200.errors import InputValidationError
from vericcl_b200.semantics.collective import PARTITIONED, CollectiveKind


@dataclass(frozen=True, order=True)
class ParameterChoice:
    slice_count: int
    channels: int
    slice_size_bytes: int


def _divisors(m: int):
    small, large = [], []
    i = 1
    while i * i <= m:
        if m % i == 0:
            small.append(i)
            if i * i != m:
                large.append(m // i)
        i += 1
    return small + large[::-1]


def initial_parameter_domain(request, *, max_candidates: int = 16, max_channels: int | None = None,
                             scratch_bytes: int | None = None, free_slice: bool = False):
    """Legal choices; the keywords relax the request's channel limit, scratch budget or fixed slice."""
    spec = request.collective
    p = request.rank_count
    m = request.hyperparameters.total_size_bytes
    elem = request.element_bytes
    limits = request.request_config["runtime"]["limits"]
    scratch = request.request_config["runtime"]["scratch_bytes_per_rank"] if scratch_bytes is None else scratch_bytes
    max_channels = request.solver.max_channels if max_channels is None else max_channels
    fixed = None if free_slice else request.hyperparameters.slice_size_bytes
    out = []
    for n in sorted(_divisors(m // elem), reverse=True):
        s = m // n
        if fixed is not None and s != fixed:
            continue
        if s % elem:
            continue
        if spec.kind in PARTITIONED and n % p:
            continue
        runtime_chunks = n * p if spec.kind is CollectiveKind.ALL_GATHER else n
        if (m * (p if spec.kind is CollectiveKind.ALL_GATHER else 1)) % runtime_chunks:
            continue
        if (s // elem) % max(1, 16 // elem) and fixed is None:
            continue
        # per-TB step bound: a TB per (peer, channel) carries about N*P/C steps for AllGather, N/C otherwise
        for c in range(1, max_channels + 1):
            per_tb = (n * p if spec.kind is CollectiveKind.ALL_GATHER else 2 * n) / c
            if per_tb > limits["steps_per_tb"]:
                continue
            if runtime_chunks - 1 > limits["buffer_offset"]:
                continue
            if 2 * (p - 1) * c > limits["tbs_per_rank"]:
                continue
            if spec.reducing and s > scratch and p > 2:
                continue
            out.append(ParameterChoice(n, c, s))
        if len(out) >= max_candidates:
            break
    if not out:
        raise InputValidationError("no legal (slice size, channel) choice fits the runtime limits")
    return out


def resolve_parameters(request, choice: ParameterChoice):
    """Request bound to one parameter choice (slice size and channel limit)."""
    return request.with_slice(choice.slice_size_bytes)


def bind_artifact_partition(request, slice_size_bytes: int):
    """Bind the slice partition recorded in a schedule's sidecar (verify path)."""
    m = request.hyperparameters.total_size_bytes
    if slice_size_bytes <= 0 or m % slice_size_bytes or slice_size_bytes % request.element_bytes:
        raise InputValidationError("sidecar slice size does not partition the request")
    return request.with_slice(slice_size_bytes)
