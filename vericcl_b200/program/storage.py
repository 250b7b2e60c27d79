"""Storage plan: logical values → i/o/s slots with read-completion reuse.

Walks the network operations in dependency order (ties by priority time),
creates one :class:`Value` per delivered state, writes final values straight
into their output slot when possible, and places intermediates in scratch
slots that are reused once all readers of the previous occupant completed
(the reuse adds those readers as dependencies of the writer).  Required
outputs that no transfer delivers get a local copy.  In-place layouts alias
input and output slots; a write into an aliased slot waits for every reader
of the original value (reference: vericcl/xml/v5_buffers.py:117-288).
"""
from __future__ import annotations

import heapq
from collections import defaultdict
from types import MappingProxyType

from vericcl_b200.errors import ScratchBudgetError, SemanticError
from vericcl_b200.program.model import Address, Instruction, StoragePlan, Value
from vericcl_b200.semantics.collective import CollectiveKind, input_ranks, required_outputs
from vericcl_b200.semantics.versions import canonical


def _ordered(operations):
    by_id = {op.operation_id: op for op in operations}
    indeg = {k: 0 for k in by_id}
    succ = defaultdict(list)
    for op in operations:
        for dep in op.dependencies:
            if dep not in by_id:
                raise SemanticError("unknown network dependency " + dep)
            indeg[op.operation_id] += 1
            succ[dep].append(op.operation_id)
    heap = [(by_id[k].priority_time, by_id[k].stage_id, k) for k, d in indeg.items() if d == 0]
    heapq.heapify(heap)
    out = []
    while heap:
        _, _, key = heapq.heappop(heap)
        out.append(by_id[key])
        for nxt in succ[key]:
            indeg[nxt] -= 1
            if indeg[nxt] == 0:
                op = by_id[nxt]
                heapq.heappush(heap, (op.priority_time, op.stage_id, nxt))
    if len(out) != len(by_id):
        raise SemanticError("network dependencies contain a cycle")
    return out


def build_storage_plan(candidate, request, scratch_budget_bytes: int | None = None, *,
                       _probe: bool = False) -> StoragePlan:
    spec = request.collective
    p, n = candidate.rank_count, candidate.slice_count
    size = candidate.slice_size_bytes
    if scratch_budget_bytes is None:
        scratch_budget_bytes = request.request_config["runtime"]["scratch_bytes_per_rank"]
    scratch_capacity = scratch_budget_bytes // size if size else 0
    expected = required_outputs(spec, p, n)
    required_at = defaultdict(list)      # (rank, contributors) -> output slots
    for slot, contributors in expected.items():
        required_at[(slot.rank, contributors)].append(slot)
    states, by_pos, addresses, initial = {}, defaultdict(list), {}, []
    for rank in input_ranks(spec, p):
        for index in range(n):
            sid = "input-r%d-s%d" % (rank, index)
            value = Value(sid, rank, index, frozenset({rank * n + index}), None)
            states[sid] = value
            by_pos[rank, index].append(value)
            addresses[sid] = Address(rank, "i", index)
            initial.append(sid)
    instructions = []
    for op in _ordered(candidate.operations):
        index = op.index if op.index >= 0 else min(op.contributors) % n
        matches = [v for v in by_pos[op.src_rank, index] if v.contributors == op.contributors]
        if not matches:
            raise SemanticError("source state of %s is unavailable" % op.operation_id)
        source = matches[-1]
        reads = [source.state_id]
        combined = op.contributors
        if op.kind == "rrc":
            options = [v for v in by_pos[op.dst_rank, index]
                       if not v.contributors & op.contributors and v.contributors <= op.target_contributors]
            if not options:
                raise SemanticError("reduction %s has no disjoint accumulator" % op.operation_id)
            acc = max(options, key=lambda v: (len(v.contributors), v.state_id))
            reads.append(acc.state_id)
            combined = combined | acc.contributors
        elif op.kind != "send":
            raise SemanticError("network operation must be send or rrc")
        deps = set(op.dependencies)
        deps.update(states[k].producer for k in reads if states[k].producer is not None)
        sid = "state-" + op.operation_id
        value = Value(sid, op.dst_rank, index, combined, op.operation_id)
        states[sid] = value
        by_pos[op.dst_rank, index].append(value)
        instructions.append(Instruction(op.operation_id, op.kind, tuple(reads), sid, op.dst_rank, op.src_rank,
                                        op.channel, op.stage_id, frozenset(deps), op.priority_time))
    # final outputs: direct placement or a local copy
    outputs, direct = {}, {}
    last_priority = max((i.priority_time for i in instructions), default=0.0) + 1.0
    last_stage = max((i.stage_id for i in instructions), default=0)
    for slot, contributors in sorted(expected.items()):
        index = min(contributors) % n
        matches = [v for v in by_pos[slot.rank, index] if v.contributors == contributors]
        if not matches:
            raise SemanticError("output %d:%d is never produced" % (slot.rank, slot.offset))
        value = matches[-1]
        target = Address(slot.rank, "o", slot.offset)
        origin = addresses.get(value.state_id)
        if origin is not None and canonical(spec, p, n, *_a(origin)) == canonical(spec, p, n, *_a(target)):
            outputs[slot] = value.state_id
            continue
        if value.producer is not None and value.state_id not in direct and not spec.inplace:
            direct[value.state_id] = target
            outputs[slot] = value.state_id
            continue
        if value.producer is not None and value.state_id not in direct and spec.inplace:
            # an in-place final write must not clobber a still-needed input alias; it is
            # placed directly and ordered after the readers below
            direct[value.state_id] = target
            outputs[slot] = value.state_id
            continue
        op_id = "output-copy-r%d-o%d" % (slot.rank, slot.offset)
        sid = "state-" + op_id
        states[sid] = Value(sid, slot.rank, index, contributors, op_id)
        addresses[sid] = target
        deps = frozenset({value.producer}) if value.producer else frozenset()
        instructions.append(Instruction(op_id, "copy", (value.state_id,), sid, slot.rank, -1, -1, last_stage,
                                        deps, last_priority))
        outputs[slot] = sid
    readers = defaultdict(set)
    for ins in instructions:
        for k in ins.inputs:
            readers[k].add(ins.operation_id)
    # writes into a physical slot that aliases an initial input wait for that input's readers
    initial_regions = defaultdict(list)
    for k in initial:
        initial_regions[canonical(spec, p, n, *_a(addresses[k]))].append(k)
    protected = []
    for ins in instructions:
        deps = set(ins.dependencies)
        target = direct.get(ins.output) or addresses.get(ins.output)
        if target is not None:
            for k in initial_regions.get(canonical(spec, p, n, *_a(target)), ()):
                deps.update(readers[k] - {ins.operation_id})
        protected.append(_replace(ins, dependencies=frozenset(deps)))
    instructions = _topo(protected)
    # scratch allocation with read-completion reuse
    position = {ins.operation_id: i for i, ins in enumerate(instructions)}
    ancestors, pools, reuse, final = {}, defaultdict(dict), [], []
    for ins in instructions:
        deps = set(ins.dependencies)
        up = set(deps)
        for d in deps:
            up |= ancestors[d]
        if ins.output in direct:
            addresses[ins.output] = direct[ins.output]
        elif ins.output not in addresses:
            pool = pools[ins.rank]
            choice = None
            for slot_index, prior in sorted(pool.items()):
                consumers = readers[prior] - ({ins.operation_id} if prior in ins.inputs else set())
                if all(position[r] < position[ins.operation_id] for r in consumers) and consumers <= up | {
                        ins.operation_id}:
                    choice = (slot_index, prior, consumers)
                    break
            if choice is None and len(pool) >= scratch_capacity:
                for slot_index, prior in sorted(pool.items()):
                    consumers = readers[prior] - ({ins.operation_id} if prior in ins.inputs else set())
                    if all(position[r] < position[ins.operation_id] for r in consumers):
                        choice = (slot_index, prior, consumers)
                        break
            if choice is not None:
                slot_index, prior, consumers = choice
                deps |= consumers
                reuse.append({"writer": ins.operation_id, "old_state": prior, "new_state": ins.output,
                              "previous_readers": sorted(consumers), "rank": ins.rank, "offset": slot_index})
            elif len(pool) < scratch_capacity:
                slot_index = len(pool)
            else:
                if _probe:
                    raise ScratchBudgetError("scratch budget too small", 0)
                needed = _needed_scratch(candidate, request, scratch_capacity, size)
                raise ScratchBudgetError("scratch budget (%d slots) cannot hold this execution order; %d bytes "
                                         "per rank would" % (scratch_capacity, needed), needed)
            addresses[ins.output] = Address(ins.rank, "s", slot_index)
            pool[slot_index] = ins.output
        all_up = set(deps)
        for d in deps:
            all_up |= ancestors[d]
        ancestors[ins.operation_id] = all_up
        final.append(_replace(ins, dependencies=frozenset(deps)))
    output_slots = {r: max((s.offset + 1 for s in expected if s.rank == r), default=0) for r in range(p)}
    input_slots = {r: (n if r in input_ranks(spec, p) else 0) for r in range(p)}
    if spec.kind is CollectiveKind.BROADCAST or spec.kind is CollectiveKind.SCATTER:
        input_slots = {r: n for r in range(p)}
    return StoragePlan(MappingProxyType(states), tuple(initial), tuple(final), MappingProxyType(addresses),
                       MappingProxyType(outputs), MappingProxyType(input_slots), MappingProxyType(output_slots),
                       MappingProxyType({r: len(pools[r]) for r in range(p)}), tuple(reuse))


def _needed_scratch(candidate, request, capacity: int, size: int) -> int:
    """The smallest scratch budget (bytes per rank) that holds this execution order."""
    unbounded = build_storage_plan(candidate, request, scratch_budget_bytes=1 << 62, _probe=True)
    most = max(unbounded.scratch_slots.values(), default=0)
    for slots in range(capacity + 1, most):
        try:
            build_storage_plan(candidate, request, scratch_budget_bytes=slots * size, _probe=True)
            return slots * size
        except ScratchBudgetError:
            continue
    return most * size


def _a(address: Address):
    return address.rank, address.buffer, address.offset


def _replace(ins: Instruction, **kw) -> Instruction:
    from dataclasses import replace
    return replace(ins, **kw)


def _topo(instructions):
    by_id = {i.operation_id: i for i in instructions}
    indeg = {k: 0 for k in by_id}
    succ = defaultdict(list)
    for ins in instructions:
        for d in ins.dependencies:
            indeg[ins.operation_id] += 1
            succ[d].append(ins.operation_id)
    heap = [(by_id[k].priority_time, k) for k, d in indeg.items() if d == 0]
    heapq.heapify(heap)
    out = []
    while heap:
        _, k = heapq.heappop(heap)
        out.append(by_id[k])
        for nxt in succ[k]:
            indeg[nxt] -= 1
            if indeg[nxt] == 0:
                heapq.heappush(heap, (by_id[nxt].priority_time, nxt))
    if len(out) != len(by_id):
        raise SemanticError("storage and reference orders contain a dependency cycle")
    return out
