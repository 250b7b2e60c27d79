"""The physical work graph a cost model prices.

Lowering turns a schedule into :class:`WorkOperation` records: one per
transfer, per receive-reduce, per local copy or reduce, per NVLS operation and
per dependency-only step.  A data-moving operation carries one
:class:`Movement` (the cost component that prices it and its bytes); every
operation names the operations it starts after and, for transfers, the shared
resources its bytes cross and a flow identity that measured sharing modes
refer to.  An
:class:`Executable` is the whole graph plus the operations whose completion
makes the collective's outputs ready.  (Reference counterpart of the record
set: vericcl/performance/events.py:11-80.)
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Mapping

from vericcl_b200.errors import SemanticError
from vericcl_b200.performance.model import real

# per kind: (moves bytes over the network, moves data at all, may name shared resources)
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
class Movement:
    """The data one operation moves: the cost component that prices it and its size in bytes.

    An operation either moves data (it has one) or only orders other work (it
    has none), so a payload without a price, or a price without a payload,
    cannot be written down.
    """
    component: str
    nbytes: int

    def __post_init__(self):
        if not (isinstance(self.component, str) and self.component):
            raise SemanticError("a movement needs the cost component that prices it")
        n = self.nbytes
        if isinstance(n, bool) or not isinstance(n, int) or n <= 0:
            raise SemanticError("a movement of %r bytes moves nothing" % (n,))


@dataclass(frozen=True)
class WorkOperation:
    """One node of the work graph.

    ``movement`` is None for a dependency-only step; ``after`` lists the
    operations that must complete first; ``crosses`` the shared resources its
    bytes cross (network kinds only); ``flow_id`` the flow that measured
    sharing modes name (required for network kinds); ``release_us`` the
    earliest start; ``estimated`` marks work whose price stands in for an
    unmeasured cost (priced, but never counted as measured).
    """
    operation_id: str
    kind: str
    movement: Movement | None = None
    after: tuple = ()
    crosses: tuple = ()
    flow_id: str | None = None
    release_us: float = 0.0
    estimated: bool = False

    def __post_init__(self):
        me = self.operation_id if isinstance(self.operation_id, str) else repr(self.operation_id)
        if not me:
            raise SemanticError("a work operation needs a non-empty id")
        rule = _KIND_RULES.get(self.kind)
        if rule is None:
            raise SemanticError("%s: kind %r is none of %s" % (me, self.kind, sorted(KINDS)))
        network, data, shares = rule
        if data != (self.movement is not None):
            raise SemanticError("%s: a %s %s" % (me, self.kind, "moves data and needs a movement" if data
                                                 else "only orders work and takes no movement"))
        if network and not self.flow_id:
            raise SemanticError("%s: network work needs a flow id" % me)
        after = _names(self.after, "predecessors", me)
        crosses = _names(self.crosses, "shared resources", me)
        if crosses and not shares:
            raise SemanticError("%s: %s work does not cross shared resources" % (me, self.kind))
        if not isinstance(self.estimated, bool):
            raise SemanticError("%s: estimated is a flag" % me)
        object.__setattr__(self, "after", after)
        object.__setattr__(self, "crosses", crosses)
        object.__setattr__(self, "release_us", real(self.release_us, me + " release_us"))

    @property
    def component(self) -> str | None:
        return None if self.movement is None else self.movement.component

    @property
    def nbytes(self) -> int:
        return 0 if self.movement is None else self.movement.nbytes


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
            dangling = [d for d in op.after if d not in index]
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
