"""Local repair: turn strategies into candidate variants and keep strict improvements.

A strategy names a family and the operations it may change (its repair
domain); every other decision of the incumbent — data assignment, paths,
channels and relative order — stays fixed, and timing is re-derived by
lowering and the exact predictor.  Families:

* ``path``     — reroute a broadcast transfer a→b through the least-loaded relay c;
* ``allocation`` / ``channel`` — move the transfer to another channel (another TB);
* ``order``    — advance the transfer's priority inside its TBs;
* ``joint``    — channel and path together;
* ``internal_root`` — reshape the reduction chain into a binomial tree;
* ``structure`` / ``partition`` — handled by resynthesis (:mod:`resynthesis`).

``solve_repair`` lowers and checks every variant, evaluates exact T_pred under
the incumbent's model, then solves a small selection MILP over the improving
variants (pairwise-compatible ones may be combined: the "event columns"
model, :mod:`event_columns`) and accepts only a combination whose exact T_pred
is strictly better (reference: vericcl/tuning/strategies.py:23-431).
"""
from __future__ import annotations

from dataclasses import dataclass, replace

from vericcl_b200.composer.compose import NetworkCandidate, NetworkOperation, list_schedule
from vericcl_b200.errors import BudgetExhausted, SemanticError
from vericcl_b200.topology.model import LinkKey


@dataclass(frozen=True)
class RepairDomain:
    operations: frozenset
    family: str

    def outside_invariant(self, before: NetworkCandidate, after: NetworkCandidate) -> bool:
        """Operations outside the domain keep endpoints, channel and contributors."""
        old = {op.operation_id: op for op in before.operations}
        new = {op.operation_id: op for op in after.operations}
        for key, op in old.items():
            if key in self.operations:
                continue
            other = new.get(key)
            if other is None or (other.src_rank, other.dst_rank, other.channel, other.contributors) != \
                    (op.src_rank, op.dst_rank, op.channel, op.contributors):
                return False
        return True


def _replace_ops(candidate, ops, topology, origin):
    timed = list_schedule(ops, topology, candidate.slice_size_bytes)
    # keep the incumbent's priorities for unchanged operations so their relative order stays fixed
    prior = {op.operation_id: op.priority_time for op in candidate.operations}
    fixed = [replace(op, priority_time=prior.get(op.operation_id, op.priority_time)) for op in timed]
    return NetworkCandidate(candidate.rank_count, candidate.slice_count, candidate.slice_size_bytes, tuple(fixed),
                            origin, candidate.channels)


def variant_channel(candidate, topology, op_id, channel):
    ops = [replace(op, channel=channel) if op.operation_id == op_id else op for op in candidate.operations]
    return _replace_ops(candidate, ops, topology, "repair:channel")


def variant_order(candidate, topology, op_id, advance=1.0):
    ops = []
    for op in candidate.operations:
        if op.operation_id == op_id:
            op = replace(op, priority_time=max(0.0, op.priority_time - advance))
        ops.append(op)
    return NetworkCandidate(candidate.rank_count, candidate.slice_count, candidate.slice_size_bytes, tuple(ops),
                            "repair:order", candidate.channels)


def variant_path(candidate, topology, op_id, avoid=(), via=None):
    """Reroute a send a→b through relay c (a→c then c→b): ``via`` when given, else the least-loaded relay."""
    by_id = {op.operation_id: op for op in candidate.operations}
    op = by_id[op_id]
    if op.kind != "send":
        raise SemanticError("only broadcast transfers can be rerouted through a relay")
    load = {}
    for other in candidate.operations:
        load[other.src_rank] = load.get(other.src_rank, 0) + 1
        load[other.dst_rank] = load.get(other.dst_rank, 0) + 1
    relays = [c for c in range(candidate.rank_count) if c not in (op.src_rank, op.dst_rank)
              and topology.has_link(op.src_rank, c) and topology.has_link(c, op.dst_rank)]
    if via is not None:
        relays = [c for c in relays if c == via]
    if not relays:
        raise SemanticError("no relay available for " + op_id)
    c = min(relays, key=lambda r: (load.get(r, 0), r))
    first = replace(op, operation_id=op_id + "@via%d" % c, dst_rank=c)
    second = replace(op, operation_id=op_id, src_rank=c, dependencies=frozenset({first.operation_id}))
    ops = []
    for other in candidate.operations:
        if other.operation_id == op_id:
            ops.extend([first, second])
        else:
            ops.append(other)
    return _replace_ops(candidate, ops, topology, "repair:path")


def variant_reshape(candidate, topology, op_id):
    """Turn the chain of reductions into the root of ``op_id`` into a binomial tree."""
    by_id = {op.operation_id: op for op in candidate.operations}
    target = by_id[op_id]
    chain = [op for op in candidate.operations if op.kind == "rrc" and op.dst_rank == target.dst_rank
             and op.index == target.index and op.target_contributors <= target.target_contributors | frozenset()]
    chain = [op for op in chain if len(op.contributors) == 1]
    if len(chain) < 3:
        raise SemanticError("reduction chain too short to reshape")
    root = target.dst_rank
    members = sorted(op.src_rank for op in chain)
    contrib = {op.src_rank: op.contributors for op in chain}
    base = set(target.target_contributors)
    for op in chain:
        base -= op.contributors
    order = [root] + members
    new_ops, holder = [], {r: (None, frozenset(contrib.get(r, frozenset()))) for r in order}
    holder[root] = (None, frozenset(base))
    step = 1
    n = len(order)
    names = 0
    while step < n:
        for i in range(0, n, 2 * step):
            j = i + step
            if j >= n:
                continue
            a, b = order[j], order[i]
            dep_a, val_a = holder[a]
            dep_b, val_b = holder[b]
            names += 1
            oid = "%s#tree%d" % (op_id, names)
            deps = frozenset(d for d in (dep_a, dep_b) if d)
            chan = min(target.channel, topology.link(LinkKey(a, b)).max_channels - 1) if topology.has_link(a, b) else 0
            if not topology.has_link(a, b):
                raise SemanticError("binomial edge %d->%d has no link" % (a, b))
            new_ops.append(NetworkOperation(oid, "rrc", a, b, chan, target.stage_id, val_a, val_a | val_b, deps, 0.0,
                                            target.index))
            holder[b] = (oid, val_a | val_b)
        step *= 2
    final = holder[root][0]
    removed = {op.operation_id for op in chain}
    last = max(chain, key=lambda op: op.priority_time).operation_id
    ops = []
    for op in candidate.operations:
        if op.operation_id in removed:
            continue
        deps = frozenset((final if d in removed else d) for d in op.dependencies)
        ops.append(replace(op, dependencies=deps))
    ops.extend(new_ops)
    # the final tree edge replaces the chain's last reduction for everyone downstream
    ops = [replace(op, dependencies=frozenset((final if d == last else d) for d in op.dependencies)) for op in ops]
    return _replace_ops(candidate, ops, topology, "repair:internal_root")


def implementations(strategy, candidate, topology, *, max_channels: int = 16):
    """Candidate variants for one strategy (empty when it does not apply)."""
    params = dict(strategy.parameters)
    out = []
    for op_id in strategy.operations:
        try:
            if strategy.family in ("allocation", "channel"):
                out.append(variant_channel(candidate, topology, op_id, params.get("channel", 0) % max_channels))
            elif strategy.family == "order":
                out.append(variant_order(candidate, topology, op_id, float(params.get("advance", 1))))
            elif strategy.family == "path":
                out.append(variant_path(candidate, topology, op_id, params.get("avoid", ()), params.get("via")))
            elif strategy.family == "joint":
                v = variant_channel(candidate, topology, op_id, params.get("channel", 0) % max_channels)
                out.append(variant_path(v, topology, op_id, params.get("avoid", ())))
            elif strategy.family == "internal_root":
                out.append(variant_reshape(candidate, topology, op_id))
        except (SemanticError, KeyError):
            continue
    return out


@dataclass
class RepairOutcome:
    improved: bool
    best: object
    evaluated: int
    improving: list
    reason: str = ""


def solve_repair(incumbent, strategies, *, lower, lease=None, max_channels: int = 16, batch_size: int | None = None):
    """Evaluate strategy variants; return the best strictly-improving bundle (if any).

    The ``batch_size`` best improving variants (by exact T_pred) enter the
    event-column combination model together (all of them when None).
    """
    from vericcl_b200.tuning.event_columns import solve_event_columns
    network = incumbent.network
    if network is None:
        return RepairOutcome(False, incumbent, 0, [], "incumbent has no network form to repair")
    topology = lower.topology
    improving = []
    evaluated = 0
    for strategy in strategies:
        if lease is not None:
            try:
                lease.check()
            except BudgetExhausted:
                break
        domain = RepairDomain(frozenset(strategy.operations), strategy.family)
        for variant in implementations(strategy, network, topology, max_channels=max_channels):
            if not domain.outside_invariant(network, variant) and strategy.family not in ("path", "joint",
                                                                                        "internal_root"):
                continue
            try:
                bundle = lower(variant)
            except SemanticError:
                continue
            evaluated += 1
            if bundle.can_execute and bundle.t_pred_us is not None and bundle.t_pred_us < incumbent.t_pred_us - 1e-9:
                improving.append((strategy, variant, bundle))
    if not improving:
        return RepairOutcome(False, incumbent, evaluated, [], "no strictly better variant")
    improving.sort(key=lambda item: item[2].t_pred_us)
    best = improving[0][2]
    combined = solve_event_columns(incumbent, improving[:batch_size] if batch_size else improving, lower=lower)
    if combined is not None and combined.t_pred_us < best.t_pred_us - 1e-9:
        best = combined
    return RepairOutcome(True, best, evaluated, [(s.strategy_id, b.t_pred_us) for s, _, b in improving])
