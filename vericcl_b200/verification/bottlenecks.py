"""Bottleneck analysis of an exact prediction and lazy repair-strategy streams.

The exact prediction gives every operation's start/end and the rate segments
it ran at.  ``analyze`` walks the critical chain that ends at T_pred, then the
other operations with zero slack (``slack_index``: chains that end at T_pred
too), and classifies each operation:

* ``resource_overlap`` — the operation ran below its own link rate because a
  shared resource (NVLink port, NIC) was split with concurrent flows;
* ``tb_wait`` — the operation started later than its data was ready because
  its thread block was still busy with earlier work (TB order);
* ``critical_service`` — the operation's own α + β·S dominates; for a send
  whose link is slower than both hops of some relay a→c→b, the cause names
  that relay and a ``path`` strategy moves the send onto it;
* ``storage_wait`` — the chain passes a dependency that no data flow needs:
  the storage plan added it because the operation reuses a scratch slot
  whose previous value still had this reader (a read-completion edge).  Every
  other dependency on the chain is mandatory (it carries data, or orders
  operations of one thread block).  Such a cause comes with the scratch
  budget that would let the storage plan keep both values.

Strategies are then generated lazily, round-robin over the eight families
(path, allocation, order, channel, joint, internal_root, structure,
partition) from the causes, and a compatible batch (no two strategies touch
the same operation) is chosen with the BDD selector (reference:
vericcl/verification/bottlenecks.py:164-453, search_coverage.py:9).
"""
from __future__ import annotations

from collections import defaultdict
from dataclasses import dataclass, field

from vericcl_b200.verification.bdd import select_compatible

FAMILIES = ("path", "allocation", "order", "channel", "joint", "internal_root", "structure", "partition")


@dataclass(frozen=True)
class Cause:
    kind: str
    operation_id: str
    detail: dict = field(default_factory=dict, hash=False, compare=False)


@dataclass(frozen=True)
class StrategyRecord:
    strategy_id: str
    family: str
    operations: tuple
    parameters: tuple = ()

    def as_json(self):
        return {"id": self.strategy_id, "family": self.family, "operations": list(self.operations),
                "parameters": dict(self.parameters)}


@dataclass
class Analysis:
    t_pred_us: float
    critical_path: list
    causes: list
    utilisation: dict
    strategies: list


def _utilisation(executable, prediction):
    busy = defaultdict(float)
    ops = {op.operation_id: op for op in executable.operations}
    for key, t0, t1, rate, _src in prediction.segments:
        for res in ops[key].crosses:
            busy[res] += t1 - t0
    span = max(prediction.t_pred_us or 0.0, 1e-12)
    return {res: round(t / span, 6) for res, t in sorted(busy.items())}


def causes_on_path(executable, prediction, model, path):
    ops = {op.operation_id: op for op in executable.operations}
    seg_by_op = defaultdict(list)
    for key, t0, t1, rate, src in prediction.segments:
        seg_by_op[key].append((t0, t1, rate, src))
    out = []
    for key in path:
        op = ops[key]
        if op.kind == "nop":
            continue
        ready = max((prediction.end_times.get(d, 0.0) for d in op.after), default=0.0)
        start = prediction.start_times.get(key, 0.0)
        cost = model.service_for(op.component, op.nbytes)
        own_rate = 1.0 / cost.beta_us_per_byte if cost else None
        slowed = [s for s in seg_by_op[key] if own_rate and s[2] < own_rate * (1 - 1e-9)]
        if slowed:
            out.append(Cause("resource_overlap", key, {"min_rate": min(s[2] for s in slowed), "own_rate": own_rate,
                                                        "resources": list(op.crosses)}))
        elif start > ready + 1e-9:
            out.append(Cause("tb_wait", key, {"waited_us": start - ready}))
        else:
            detail = {"alpha_us": cost.alpha_us if cost else None}
            relay = _faster_relay(model, op)
            if relay is not None:
                detail["relay"] = relay
            out.append(Cause("critical_service", key, detail))
    return out


def _faster_relay(model, op):
    """A rank c whose two hops a→c→b each move this payload faster than the direct link a→b, or None."""
    if not (op.component or "").startswith("link:"):
        return None
    _, a, b = op.component.split(":")
    direct = model.service_for(op.component, op.nbytes)
    if direct is None:
        return None
    limit = direct.time_us(op.nbytes)
    best = None
    for key in model.services:
        parts = key.split(":")
        if parts[0] != "link" or parts[1] != a or parts[2] == b:
            continue
        c = parts[2]
        first = model.service_for(key, op.nbytes)
        second = model.service_for("link:%s:%s" % (c, b), op.nbytes)
        if first is None or second is None:
            continue
        slower = max(first.time_us(op.nbytes), second.time_us(op.nbytes))
        if slower < limit and (best is None or slower < best[0]):
            best = (slower, int(c))
    return None if best is None else best[1]


def strategy_stream(causes, network, *, max_channels: int = 16):
    """Yield strategies round-robin over families, derived from the causes."""
    per_family = {f: [] for f in FAMILIES}
    by_id = {op.operation_id: op for op in (network.operations if network is not None else ())}
    for index, cause in enumerate(causes):
        op = by_id.get(cause.operation_id)
        if op is None:
            continue
        if cause.kind == "resource_overlap":
            per_family["path"].append(StrategyRecord("path-%d" % index, "path", (op.operation_id,),
                                                     (("avoid", tuple(cause.detail.get("resources", ()))),)))
            per_family["allocation"].append(StrategyRecord("alloc-%d" % index, "allocation", (op.operation_id,),
                                                           (("channel", (op.channel + 1) % max_channels),)))
            per_family["joint"].append(StrategyRecord("joint-%d" % index, "joint", (op.operation_id,),
                                                      (("channel", (op.channel + 1) % max_channels),
                                                       ("avoid", tuple(cause.detail.get("resources", ()))))))
        elif cause.kind == "tb_wait":
            per_family["order"].append(StrategyRecord("order-%d" % index, "order", (op.operation_id,),
                                                      (("advance", 1),)))
            per_family["channel"].append(StrategyRecord("chan-%d" % index, "channel", (op.operation_id,),
                                                        (("channel", (op.channel + 1) % max_channels),)))
        else:
            if op.kind == "send" and cause.detail.get("relay") is not None:
                per_family["path"].append(StrategyRecord("relay-%d" % index, "path", (op.operation_id,),
                                                         (("via", cause.detail["relay"]),)))
            if op.kind == "rrc":
                per_family["internal_root"].append(StrategyRecord("root-%d" % index, "internal_root",
                                                                  (op.operation_id,), (("reshape", "binomial"),)))
            per_family["order"].append(StrategyRecord("prio-%d" % index, "order", (op.operation_id,),
                                                      (("advance", 1),)))
    per_family["structure"].append(StrategyRecord("structure-0", "structure", (), (("method", "alternate"),)))
    per_family["partition"].append(StrategyRecord("partition-0", "partition", (), (("slices", "double"),)))
    cursors = {f: 0 for f in FAMILIES}
    while any(cursors[f] < len(per_family[f]) for f in FAMILIES):
        for f in FAMILIES:
            if cursors[f] < len(per_family[f]):
                yield per_family[f][cursors[f]]
                cursors[f] += 1


def choose_batch(strategies, batch_size: int):
    """Pick up to ``batch_size`` pairwise-compatible strategies (BDD selection)."""
    strategies = list(strategies)[: max(batch_size * 4, batch_size)]
    names = [s.strategy_id for s in strategies]
    conflicts = []
    for i, a in enumerate(strategies):
        for b in strategies[i + 1:]:
            if set(a.operations) & set(b.operations) or (not a.operations and not b.operations):
                conflicts.append((a.strategy_id, b.strategy_id))
    weights = {s.strategy_id: 1.0 / (1 + i) + 1.0 for i, s in enumerate(strategies)}
    chosen = set(select_compatible(names, conflicts, weights))
    return [s for s in strategies if s.strategy_id in chosen][:batch_size]


def trace_causes(report, bundle, *, tails: int = 5):
    """``trace_tail`` causes: the slowest measured device steps, mapped back to their operations.

    ``report`` is a trace report whose timeline rows carry the XML origin
    (``xml_tb``, ``xml_step``) of each device step; the schedule's blocks map
    an XML (rank, thread block, step) to its operation.
    """
    if not report or bundle.program is None:
        return []
    ops_of = {(b.rank, b.tb_id): [x.operation_id for x in b.steps] for b in bundle.program.blocks}
    # only network transfers can be repaired; local copies of the lowering are skipped
    network = {op.operation_id for op in bundle.network.operations} if bundle.network is not None else None
    rows = sorted((r for r in report.get("timeline", ()) if r.get("xml_tb", -1) is not None
                   and r.get("xml_tb", -1) >= 0), key=lambda r: (-r["duration_us"], r["rank"], r["step"]))
    out, seen = [], set()
    for row in rows:
        ops = ops_of.get((row["rank"], row["xml_tb"]))
        if not ops or not 0 <= row["xml_step"] < len(ops):
            continue
        op = ops[row["xml_step"]]
        if op in seen or (network is not None and op not in network):
            continue
        seen.add(op)
        out.append(Cause("trace_tail", op, {"duration_us": row["duration_us"], "wait_us": row.get("wait_us"),
                                            "rank": row["rank"]}))
        if len(out) >= tails:
            break
    return out


def dependency_kinds(storage) -> dict:
    """``{(reader, writer): kind}`` for every dependency the storage plan created.

    ``data`` — the later operation consumes the earlier one's output;
    ``storage`` — the writer overwrites a scratch
    slot whose previous value the earlier operation still reads, and nothing
    else links them (a read-completion edge that more scratch would remove).
    """
    if storage is None:
        return {}
    producer = {sid: v.producer for sid, v in storage.values.items()}
    kinds = {}
    for ins in storage.instructions:
        for sid in ins.inputs:
            if producer.get(sid) is not None:
                kinds[(producer[sid], ins.operation_id)] = "data"
    for record in getattr(storage, "reuse", ()) or ():
        writer = record["writer"]
        for reader in record["previous_readers"]:
            kinds.setdefault((reader, writer), "storage")
    return kinds


def storage_causes(bundle, path) -> list:
    """``storage_wait`` causes for consecutive critical-path operations linked only by slot reuse."""
    kinds = dependency_kinds(getattr(bundle, "storage", None))
    out = []
    for a, b in zip(path, path[1:]):
        if kinds.get((a, b)) == "storage":
            slot = next((r for r in bundle.storage.reuse if r["writer"] == b and a in r["previous_readers"]), {})
            size = bundle.request.hyperparameters.slice_size_bytes if bundle.request is not None else None
            budget = bundle.request.request_config["runtime"]["scratch_bytes_per_rank"] \
                if bundle.request is not None else None
            out.append(Cause("storage_wait", b, {"after": a, "rank": slot.get("rank"), "offset": slot.get("offset"),
                                                 "scratch_bytes_per_rank_to_remove": None if budget is None
                                                 or size is None else budget + size}))
    return out


def slack_index(executable, prediction) -> dict:
    """Per operation, how much later (µs) it could end without moving T_pred, the predicted durations fixed.

    An operation nothing waits for may end as late as T_pred; any other as late as the earliest latest start
    of the operations that wait for it (latest end minus predicted duration), computed over the dependency
    graph in reverse topological order.  Zero slack marks every operation on some critical chain, not only the
    one chain :meth:`Prediction.critical_path` follows.  Shared-resource effects are taken as predicted.
    """
    if prediction.t_pred_us is None or not prediction.end_times:
        return {}
    ops = executable.by_id()
    succ = defaultdict(list)
    for op in executable.operations:
        for d in op.after:
            succ[d].append(op.operation_id)
    pending = {k: len(succ[k]) for k in ops}
    todo = [k for k, n in pending.items() if n == 0]
    latest_end = {}
    end, start, horizon = prediction.end_times, prediction.start_times, prediction.t_pred_us
    while todo:
        key = todo.pop()
        after = succ[key]
        latest_end[key] = horizon if not after else min(
            latest_end[s] - (end.get(s, 0.0) - start.get(s, end.get(s, 0.0))) for s in after)
        for d in ops[key].after:
            pending[d] -= 1
            if pending[d] == 0:
                todo.append(d)
    return {k: max(0.0, latest_end[k] - end.get(k, 0.0)) for k in latest_end}


def near_critical(executable, prediction, *, tolerance: float = 1e-3) -> list:
    """Operations whose slack is within ``tolerance`` × T_pred, latest-ending first."""
    slack = slack_index(executable, prediction)
    limit = tolerance * (prediction.t_pred_us or 0.0)
    ops = executable.by_id()
    keys = [k for k, v in slack.items() if v <= limit and ops[k].kind != "nop"]
    return sorted(keys, key=lambda k: (-prediction.end_times.get(k, 0.0), k))


def analyze(bundle, model, *, batch_size: int = 16, trace=None) -> Analysis:
    """Causes on the predicted critical path, then on the other near-critical operations (zero slack: other
    chains that end at T_pred), and, with a measured ``trace`` report, its slowest steps."""
    pred = bundle.prediction
    path = pred.critical_path(bundle.executable)
    on_path = set(path)
    others = [k for k in near_critical(bundle.executable, pred) if k not in on_path][:max(len(path), 1)]
    causes = trace_causes(trace, bundle) + storage_causes(bundle, path) + \
        causes_on_path(bundle.executable, pred, model, path) + \
        causes_on_path(bundle.executable, pred, model, others)
    stream = list(strategy_stream(causes, bundle.network))
    return Analysis(pred.t_pred_us, path, causes, _utilisation(bundle.executable, pred),
                    choose_batch(stream, batch_size))
