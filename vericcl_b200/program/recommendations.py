"""Input changes that would make a rejected schedule or an empty domain runnable.

When a lowered program fails its launch or storage check (or no slice /
channel choice fits the runtime limits at all), the run reports what to
change, cheapest first:

* ``renumber_threadblocks`` — dependency ids exceed the limit although the
  number of distinct dependency targets fits it (no re-solve);
* ``increase_scratch_budget`` / ``increase_device_memory_budget`` — the
  bytes a rank needs (runtime documents only, no re-solve);
* ``increase_channels`` — the channel count that brings steps per TB and
  TBs per channel direction under their limits (re-solve);
* ``increase_slice_size`` — the next legal larger slice, which means fewer
  slices and so fewer steps and buffer offsets (re-solve);
* ``use_slice_size`` — for an empty parameter domain, the legal slice that
  the domain would pick without the fixed one (re-solve).

Each is ``{"kind", "priority", "parameters", "reason_codes",
"requires_resolve"}`` (reference: vericcl/xml/recommendations.py:23-198,
which derives the first, fourth and fifth kinds from its MSCCL limits).
"""
from __future__ import annotations

import math

from vericcl_b200.errors import InputValidationError
from vericcl_b200.semantics.collective import PARTITIONED

MAX_CHANNELS = 16


def _rec(kind, priority, parameters, reasons, requires_resolve):
    return {"kind": kind, "priority": priority, "parameters": dict(parameters),
            "reason_codes": sorted(set(reasons)), "requires_resolve": requires_resolve}


def _legal_slice(request, s: int) -> bool:
    m, elem, p = request.hyperparameters.total_size_bytes, request.element_bytes, request.rank_count
    if s <= 0 or m % s or s % elem:
        return False
    n = m // s
    return not (request.collective.kind in PARTITIONED and n % p)


def _legal_slices(request) -> list:
    """Every slice size that partitions the request, ascending."""
    from vericcl_b200.planner.parameters import _divisors
    m = request.hyperparameters.total_size_bytes
    return [s for s in _divisors(m) if _legal_slice(request, s)]


def larger_slice(request) -> int:
    """The smallest legal slice size above the current one (0: none)."""
    s = request.hyperparameters.slice_size_bytes or 0
    return next((x for x in _legal_slices(request) if x > s), 0)


def recommend_for_program(program, request, checks: dict) -> list:
    """Recommendations for a lowered program whose launch or storage check failed."""
    failing = {k for k, v in checks.items() if v.get("status") == "invalid"}
    if not failing & {"launch", "storage"}:
        return []
    runtime = request.request_config["runtime"]
    limits = runtime["limits"]
    size = request.hyperparameters.slice_size_bytes
    recs, codes = [], set()
    deps = {st.dependency_tb for b in program.blocks for st in b.steps if st.dependency_tb >= 0}
    max_steps = max((len(b.steps) for b in program.blocks), default=0)
    directions, per_rank = {}, {}
    for b in program.blocks:
        per_rank[b.rank] = per_rank.get(b.rank, 0) + 1
        for d, peer in (("send", b.send_peer), ("recv", b.recv_peer)):
            if peer >= 0:
                directions[(b.rank, b.channel, d)] = directions.get((b.rank, b.channel, d), 0) + 1
    if deps and max(deps) > limits["dependency_id"]:
        codes.add("dependency_id")
        if len(deps) <= limits["dependency_id"] + 1:
            recs.append(_rec("renumber_threadblocks", 0, {"dependent_tb_count": len(deps)}, ("dependency_id",),
                             False))
    if "storage" in failing:
        need = max((c * size for c in program.scratch_slots.values()), default=0)
        if need > runtime["scratch_bytes_per_rank"]:
            recs.append(_rec("increase_scratch_budget", 1, {"scratch_bytes_per_rank": need}, ("scratch",), False))
        budget = runtime.get("device_memory_budget_bytes") or 0
        total = max(((program.input_slots.get(r, 0) + program.output_slots.get(r, 0)
                      + program.scratch_slots.get(r, 0)) * size for r in range(program.rank_count)), default=0)
        if budget > 0 and total > budget:
            recs.append(_rec("increase_device_memory_budget", 1, {"device_memory_budget_bytes": total},
                             ("device_memory",), False))
    channels = max(1, program.channels)
    required = channels
    if max_steps > limits["steps_per_tb"]:
        codes.add("steps_per_tb")
        required = max(required, math.ceil(channels * max_steps / limits["steps_per_tb"]))
    for (_, _, d), count in directions.items():
        if count > limits[d + "_tbs_per_channel"]:
            codes.add(d + "_tbs_per_channel")
            required = max(required, math.ceil(channels * count / limits[d + "_tbs_per_channel"]))
    # more channels multiply the TBs of a rank; they must still fit the per-rank limit
    tbs_after = max(per_rank.values(), default=0) * required / channels
    if channels < required <= MAX_CHANNELS and tbs_after <= limits["tbs_per_rank"]:
        recs.append(_rec("increase_channels", 2, {"max_channels": required}, codes, True))
    if any(("offset" in str(checks.get(k, {}).get("detail", ""))) for k in ("launch", "storage")):
        codes.add("buffer_offset")
    if codes & {"steps_per_tb", "buffer_offset", "send_tbs_per_channel", "recv_tbs_per_channel"}:
        bigger = larger_slice(request)
        if bigger:
            recs.append(_rec("increase_slice_size", 3, {"slice_size_bytes": bigger}, codes, True))
    return sorted(recs, key=lambda r: r["priority"])


def recommend_for_domain(request) -> list:
    """Recommendations when no (slice size, channel) choice fits the runtime limits.

    Each single relaxation is tried first (channel limit up to 16, scratch
    budget unbounded, fixed slice released); when none alone helps, all three
    together, reporting every parameter the first legal choice needs.
    """
    from vericcl_b200.planner.parameters import initial_parameter_domain
    fixed = request.hyperparameters.slice_size_bytes
    scratch = request.request_config["runtime"]["scratch_bytes_per_rank"]

    def domain(**relax):
        try:
            return initial_parameter_domain(request, **relax)
        except InputValidationError:
            return []

    def needs(choice, reason):
        out = []
        if choice.channels > request.solver.max_channels:
            out.append(_rec("increase_channels", 2, {"max_channels": choice.channels}, (reason,), True))
        if request.collective.reducing and request.rank_count > 2 and choice.slice_size_bytes > scratch:
            out.append(_rec("increase_scratch_budget", 1, {"scratch_bytes_per_rank": choice.slice_size_bytes},
                            (reason,), False))
        if fixed is not None and choice.slice_size_bytes != fixed:
            out.append(_rec("use_slice_size", 3, {"slice_size_bytes": choice.slice_size_bytes}, (reason,), True))
        return out

    recs = []
    relaxations = [{"max_channels": MAX_CHANNELS}, {"scratch_bytes": 1 << 62}]
    if fixed is not None:
        relaxations.append({"free_slice": True})
    for relax in relaxations:
        found = domain(**relax)
        if found:
            # the choice needing the fewest channels, then the largest slice count
            best = min(found, key=lambda c: (c.channels, -c.slice_count))
            recs += needs(best, "parameter_domain")
    if not recs:
        found = domain(max_channels=MAX_CHANNELS, scratch_bytes=1 << 62, free_slice=True)
        if found:
            recs = needs(min(found, key=lambda c: (c.channels, -c.slice_count)), "parameter_domain_combined")
    return sorted(recs, key=lambda r: r["priority"])


def merge(groups) -> list:
    """One recommendation per kind over several candidates: the most demanding parameters."""
    out = {}
    for recs in groups:
        for r in recs:
            have = out.get(r["kind"])
            if have is None:
                out[r["kind"]] = dict(r, parameters=dict(r["parameters"]), reason_codes=list(r["reason_codes"]))
                continue
            for key, value in r["parameters"].items():
                have["parameters"][key] = max(have["parameters"].get(key, 0), value)
            have["reason_codes"] = sorted(set(have["reason_codes"]) | set(r["reason_codes"]))
    return sorted(out.values(), key=lambda r: (r["priority"], r["kind"]))


def describe(recs: list) -> str:
    return "; ".join("%s %s" % (r["kind"], ", ".join("%s=%s" % kv for kv in sorted(r["parameters"].items())))
                     for r in recs)
