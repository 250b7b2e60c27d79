"""Physical work records replayed by the event simulator.

A :class:`WorkOperation` is one native transfer or local operation with its
cost component, payload, dependencies, shared resources and flow identity
(reference: vericcl/performance/events.py:11-80).
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Mapping

from vericcl_b200.errors import SemanticError
from vericcl_b200.performance.model import finite

COMM_KINDS = frozenset({"send", "rrc", "mc_reduce", "mc_store"})
KINDS = COMM_KINDS | {"copy", "reduce", "nop"}


@dataclass(frozen=True)
class WorkOperation:
    operation_id: str
    kind: str
    cost_key: str | None
    payload_bytes: int
    dependencies: tuple = ()
    resources: tuple = ()
    flow_id: str | None = None
    not_before_us: float = 0.0
    source_override: str | None = None

    def __post_init__(self):
        if not isinstance(self.operation_id, str) or not self.operation_id:
            raise SemanticError("work operation needs an identity")
        if self.kind not in KINDS:
            raise SemanticError("unknown physical work kind " + repr(self.kind))
        if self.source_override not in (None, "estimated"):
            raise SemanticError("operation source may only downgrade to estimated")
        if isinstance(self.payload_bytes, bool) or not isinstance(self.payload_bytes, int) or self.payload_bytes < 0:
            raise SemanticError("payload must be a nonnegative integer")
        if self.kind == "nop":
            if self.payload_bytes or self.cost_key is not None:
                raise SemanticError("NOP carries no data or cost")
        elif not self.payload_bytes or not self.cost_key:
            raise SemanticError("data operation needs payload and a cost component")
        if self.kind in COMM_KINDS and not self.flow_id:
            raise SemanticError("communication needs a flow identity")
        if self.kind in ("copy", "reduce", "nop") and self.resources:
            raise SemanticError("local operations use no communication resources")
        for name in ("dependencies", "resources"):
            values = tuple(getattr(self, name))
            if len(set(values)) != len(values) or not all(isinstance(v, str) and v for v in values):
                raise SemanticError("invalid operation " + name)
            object.__setattr__(self, name, values)
        object.__setattr__(self, "not_before_us", finite(self.not_before_us, "release time"))


@dataclass(frozen=True)
class Executable:
    operations: tuple
    output_operations: tuple | None = None
    context: Mapping[str, object] = field(default_factory=dict)

    def __post_init__(self):
        ops = tuple(self.operations)
        ids = {op.operation_id for op in ops}
        if len(ids) != len(ops):
            raise SemanticError("duplicate physical operation")
        for op in ops:
            if set(op.dependencies) - ids:
                raise SemanticError("unknown dependency of " + op.operation_id)
        outputs = tuple(ids) if self.output_operations is None else tuple(self.output_operations)
        if set(outputs) - ids:
            raise SemanticError("unknown output operation")
        object.__setattr__(self, "operations", ops)
        object.__setattr__(self, "output_operations", tuple(sorted(outputs)))
