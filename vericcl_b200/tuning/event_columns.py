"""Joint selection of compatible repair variants ("event columns").

Every improving variant is a column with its measured exact gain (incumbent
T_pred minus the variant's).  A MILP chooses a set of pairwise-compatible
columns (disjoint repair domains) maximising the summed gain; the chosen
changes are merged into one network candidate, which is lowered, checked and
predicted exactly.  Gains do not simply add up — merged changes share ports
and thread blocks — so the MILP's choice is only a starting point: a greedy
pass then adds compatible columns one at a time, best single gain first, and
keeps an addition only when the exact replay of the merged schedule (the
event simulator: operations start as soon as their dependencies finish, at
the rates of the sharing mode that is active) improves.  The best merged
candidate is accepted only when it beats every single variant (reference:
vericcl/tuning/event_columns.py:24-111, where the columns carry exact
active-mode rates inside a SCIP disjunction model).
"""
from __future__ import annotations


from vericcl_b200.composer.compose import NetworkCandidate
from vericcl_b200.errors import SemanticError
from vericcl_b200.solver.milp import Model


def _changes(base, variant):
    old = {op.operation_id: op for op in base.operations}
    return {op.operation_id: op for op in variant.operations if old.get(op.operation_id) != op}, \
        set(old) - {op.operation_id for op in variant.operations}


def _merge(base, variants):
    merged = {op.operation_id: op for op in base.operations}
    for variant in variants:
        changed, removed = _changes(base, variant)
        for key in removed:
            merged.pop(key, None)
        merged.update(changed)
    return NetworkCandidate(base.rank_count, base.slice_count, base.slice_size_bytes, tuple(merged.values()),
                            "repair:joint", base.channels)


def _lowered(lower, candidate):
    try:
        bundle = lower(candidate)
    except SemanticError:
        return None
    return bundle if bundle.can_execute and bundle.t_pred_us is not None else None


def greedy_exact(incumbent, improving, *, lower, limit: int = 8):
    """Add compatible columns best-first while the exact T_pred of the merged schedule keeps dropping."""
    base = incumbent.network
    order = sorted(range(len(improving)), key=lambda i: improving[i][2].t_pred_us)
    touched = []
    for _, variant, _ in improving:
        changed, removed = _changes(base, variant)
        touched.append(set(changed) | removed)
    chosen, best = [order[0]], improving[order[0]][2]
    used = set(touched[order[0]])
    for i in order[1:limit]:
        if touched[i] & used:
            continue
        trial = _lowered(lower, _merge(base, [improving[j][1] for j in chosen + [i]]))
        if trial is not None and trial.t_pred_us < best.t_pred_us:
            chosen.append(i)
            used |= touched[i]
            best = trial
    return best if len(chosen) > 1 else None


def solve_event_columns(incumbent, improving, *, lower):
    if len(improving) < 2:
        return None
    greedy = greedy_exact(incumbent, improving, lower=lower)
    milp = _solve_selection(incumbent, improving, lower=lower)
    found = [b for b in (greedy, milp) if b is not None]
    return min(found, key=lambda b: b.t_pred_us) if found else None


def _solve_selection(incumbent, improving, *, lower):
    base = incumbent.network
    model = Model("event-columns")
    x = []
    touched = []
    for index, (strategy, variant, bundle) in enumerate(improving):
        var = model.binary("x%d" % index)
        x.append(var)
        changed, removed = _changes(base, variant)
        touched.append(set(changed) | removed)
    for i in range(len(improving)):
        for j in range(i + 1, len(improving)):
            if touched[i] & touched[j]:
                model.add_le([(1, x[i]), (1, x[j])], 1, name="compat%d_%d" % (i, j))
    gains = [incumbent.t_pred_us - b.t_pred_us for _, _, b in improving]
    model.minimize([(-g, v) for g, v in zip(gains, x)])
    sol = model.solve(time_limit=10.0)
    if not sol.usable:
        return None
    chosen = [i for i, v in enumerate(x) if sol.values[v.name] > 0.5]
    if len(chosen) < 2:
        return None
    merged = {op.operation_id: op for op in base.operations}
    for i in chosen:
        changed, removed = _changes(base, improving[i][1])
        for key in removed:
            merged.pop(key, None)
        merged.update(changed)
    candidate = NetworkCandidate(base.rank_count, base.slice_count, base.slice_size_bytes,
                                 tuple(merged.values()), "repair:joint", base.channels)
    try:
        bundle = lower(candidate)
    except SemanticError:
        return None
    return bundle if bundle.can_execute else None
