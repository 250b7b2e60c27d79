"""The physical work graph a cost model prices.

Lowering turns a schedule into :class:`WorkOperation` records: one per
transfer, per receive-reduce, per local copy or reduce, per NVLS operation and
per dependency-only step.  Each names the cost component that prices it, its
payload, the operations it waits for, the shared resources its bytes cross and,
for transfers, a flow identity that measured sharing modes refer to.  An
:class:`Executable` is the whole graph plus the operations whose completion
makes the collective's outputs ready.  (Reference counterpart of the record
set: vericcl/performance/events.py:11-80.)
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Mapping

from vericcl_b200.errors import SemanticError
from vericcl_b200.performance.model import real

# per kind: (moves bytes over the network, carries data, may name shared resources)
_KIND_RULES = {
    "send": (True, True, True),
    "rrc": (True, True, True),
    "mc_reduce": (True, True, True),
    "mc_store": (True, True, True),
    "copy": (False, True, False),
    "reduce": (False, True, False),
    "nop": (False, False, False),
}
COMM_KINDS = frozenset(k for k, rule in _KIND_RULES.items() if rule[0])
KINDS = frozenset(_KIND_RULES)


def _names(values, what: str, owner: str) -> tuple:
    out = tuple(values)
    bad = [v for v in out if not (isinstance(v, str) and v)]
    if bad:
        raise SemanticError("%s of %s must be non-empty strings: %r" % (what, owner, bad))
    if len(set(out)) < len(out):
        raise SemanticError("%s of %s repeat an entry" % (what, owner))
    return out


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
    source_override: str | None = None   # "estimated": price it but do not count it as measured

    def __post_init__(self):
        me = self.operation_id if isinstance(self.operation_id, str) else repr(self.operation_id)
        if not me:
            raise SemanticError("a work operation needs a non-empty id")
        rule = _KIND_RULES.get(self.kind)
        if rule is None:
            raise SemanticError("%s: kind %r is none of %s" % (me, self.kind, sorted(KINDS)))
        network, data, shares = rule
        size = self.payload_bytes
        if isinstance(size, bool) or not isinstance(size, int) or size < 0:
            raise SemanticError("%s: payload %r is not a byte count" % (me, size))
        if data != (size > 0) or data != bool(self.cost_key):
            raise SemanticError("%s: a %s %s" % (me, self.kind, "needs a payload and a cost component" if data
                                                 else "has neither payload nor cost component"))
        if network and not self.flow_id:
            raise SemanticError("%s: network work needs a flow id" % me)
        deps = _names(self.dependencies, "dependencies", me)
        res = _names(self.resources, "resources", me)
        if res and not shares:
            raise SemanticError("%s: %s work does not cross shared resources" % (me, self.kind))
        if self.source_override is not None and self.source_override != "estimated":
            raise SemanticError("%s: source_override can only be 'estimated'" % me)
        object.__setattr__(self, "dependencies", deps)
        object.__setattr__(self, "resources", res)
        object.__setattr__(self, "not_before_us", real(self.not_before_us, me + " not_before_us"))


@dataclass(frozen=True)
class Executable:
    operations: tuple
    output_operations: tuple | None = None
    context: Mapping[str, object] = field(default_factory=dict)

    def __post_init__(self):
        ops = tuple(self.operations)
        index = {}
        for op in ops:
            if op.operation_id in index:
                raise SemanticError("operation %s appears twice" % op.operation_id)
            index[op.operation_id] = op
        for op in ops:
            dangling = [d for d in op.dependencies if d not in index]
            if dangling:
                raise SemanticError("%s waits for unknown operations %s" % (op.operation_id, dangling))
        outs = tuple(index) if self.output_operations is None else tuple(self.output_operations)
        stray = [o for o in outs if o not in index]
        if stray:
            raise SemanticError("output operations %s are not in the graph" % stray)
        object.__setattr__(self, "operations", ops)
        object.__setattr__(self, "output_operations", tuple(sorted(set(outs))))

    def by_id(self) -> dict:
        return {op.operation_id: op for op in self.operations}
