"""Lower a storage plan to the MSCCL-style native program and its XML text.

Each instruction becomes endpoints: a ``send`` is an ``s`` step on the sender
and an ``r`` step on the receiver; an ``rrc`` is ``s`` + ``rrc``; a local
``copy`` is ``cpy``.  Endpoints go to thread blocks keyed by (rank,
direction, peer, channel) — or (rank, fused, peer, channel) with the fused
layout; a rank's copies share one TB, split round-robin over more when they
exceed the steps-per-TB limit.  A step carries at most one cross-TB dependency, so extra waits become
dependency-only ``nop`` steps; waits already implied by TB order or earlier
waits are dropped using per-endpoint ancestor bitsets (reference:
vericcl/xml/v5_program.py:15-94).  The XML uses the MSCCL attribute set
(``proto="Simple"``, ``cnt=1``) so it stays loadable by MSCCL-compatible
runtimes as well as by this package's interpreter.
"""
from __future__ import annotations

from collections import defaultdict
from dataclasses import replace

from vericcl_b200.errors import SemanticError
from vericcl_b200.program.model import NativeBlock, NativeProgram, NativeStep
from vericcl_b200.semantics.collective import CollectiveKind, runtime_chunks


def _endpoints(ins, storage, lane=0):
    src = storage.addresses[ins.inputs[0]]
    dst = storage.addresses[ins.output]
    if ins.kind == "copy":
        return ((ins.rank, "copy", -1, -1 - lane, "cpy", src, dst),)
    recv_src = storage.addresses[ins.inputs[1]] if ins.kind == "rrc" else dst
    return ((src.rank, "send", dst.rank, ins.channel, "s", src, dst),
            (dst.rank, "recv", src.rank, ins.channel, "rrc" if ins.kind == "rrc" else "r", recv_src, dst))


def lower_program(storage, request, *, tb_layout: str | None = None, name: str = "vericcl_b200") -> NativeProgram:
    layout = tb_layout or request.request_config["runtime"]["tb_layout"]
    p = request.rank_count
    n = request.hyperparameters.slice_count
    blocks = defaultdict(list)
    location, step_owner, dep_of = {}, {}, {}
    bits, ancestors, order = {}, {}, {}
    block_anc, seq = defaultdict(int), defaultdict(int)
    # a rank's local copies share one TB unless they exceed the steps-per-TB limit; then they are dealt
    # round-robin over as many copy TBs as the limit needs
    limit = request.request_config["runtime"]["limits"]["steps_per_tb"]
    copies = defaultdict(int)
    for ins in storage.instructions:
        if ins.kind == "copy":
            copies[ins.rank] += 1
    lanes = {r: -(-c // limit) for r, c in copies.items()}
    dealt = defaultdict(int)
    for ins in storage.instructions:
        lane = 0
        if ins.kind == "copy":
            lane = dealt[ins.rank] % lanes[ins.rank]
            dealt[ins.rank] += 1
        eps = _endpoints(ins, storage, lane)
        ranks = {e[0] for e in eps}
        assigned = defaultdict(list)
        for pred in sorted(ins.dependencies):
            cands = [r for r in ranks if (pred, r) in location]
            if not cands:
                raise SemanticError("dependency %s -> %s has no same-rank endpoint" % (pred, ins.operation_id))
            for r in cands:
                assigned[r].append(location[pred, r])
        for rank, direction, peer, channel, kind, src, dst in eps:
            key = (rank, "fused" if layout == "fused" and direction != "copy" else direction, peer, channel)
            covered = block_anc[key]
            waits = []
            for target in sorted(set(assigned[rank]), key=order.__getitem__, reverse=True):
                if not covered & bits[target]:
                    waits.append(target)
                    covered |= ancestors[target]
            for i, target in enumerate(waits[:-1]):
                sid = "nop:%s:%d:%d" % (ins.operation_id, rank, i)
                blocks[key].append((sid, NativeStep("nop", None, None, operation_id=ins.operation_id)))
                step_owner[sid] = key
                dep_of[sid] = target
            sid = "%s:%s:%d" % (ins.operation_id, direction, rank)
            blocks[key].append((sid, NativeStep(kind, src, dst, operation_id=ins.operation_id)))
            step_owner[sid] = key
            if waits:
                dep_of[sid] = waits[-1]
            location[ins.operation_id, rank] = sid
            order[sid] = seq[rank]
            bits[sid] = 1 << seq[rank]
            seq[rank] += 1
            ancestors[sid] = covered | bits[sid]
            block_anc[key] = ancestors[sid]
    targets = {step_owner[t] for t in dep_of.values()}
    block_ids = {}
    for rank in range(p):
        keys = sorted((k for k in blocks if k[0] == rank), key=lambda k: (k not in targets, str(k)))
        block_ids.update({k: i for i, k in enumerate(keys)})
    step_loc = {sid: (block_ids[k], i) for k, steps in blocks.items() for i, (sid, _) in enumerate(steps)}
    depended = set(dep_of.values())
    result = []
    for key in sorted(blocks, key=lambda k: (k[0], block_ids[k])):
        rank, direction, peer, channel = key
        steps = []
        for sid, step in blocks[key]:
            dep = step_loc[dep_of[sid]] if sid in dep_of else (-1, -1)
            steps.append(replace(step, dependency_tb=dep[0], dependency_step=dep[1], has_dependence=sid in depended))
        send_peer = peer if direction in ("send", "fused") and any(s.kind == "s" for s in steps) else -1
        recv_peer = peer if direction in ("recv", "fused") and any(s.kind in ("r", "rrc") for s in steps) else -1
        result.append(NativeBlock(rank, block_ids[key], max(channel, 0), send_peer, recv_peer, tuple(steps)))
    channels = max((b.channel for b in result), default=0) + 1
    spec = request.collective
    runtime_bytes = request.hyperparameters.total_size_bytes * (p if spec.kind is CollectiveKind.ALL_GATHER else 1)
    return NativeProgram(name, spec.kind.value, spec.inplace, p, channels, runtime_chunks(spec, p, n),
                         tuple(result), dict(storage.input_slots), dict(storage.output_slots),
                         dict(storage.scratch_slots), min_bytes=runtime_bytes, max_bytes=runtime_bytes + 1)


def build_executable(program: NativeProgram, storage, request, topology, model_context: dict):
    """Physical work graph for T_pred: instruction deps + TB order + NOP waits."""
    from vericcl_b200.performance.events import Executable, Movement, WorkOperation
    from vericcl_b200.topology.model import LinkKey
    deps, _ = execution_dependencies(program)
    instructions = {i.operation_id: i for i in storage.instructions}
    if set(deps) != set(instructions):
        raise SemanticError("native program and storage plan cover different operations")
    size = request.hyperparameters.slice_size_bytes
    ops = []
    for key, ins in instructions.items():
        src = storage.addresses[ins.inputs[0]]
        dst = storage.addresses[ins.output]
        if ins.kind in ("send", "rrc"):
            suffix = "%d:%d" % (src.rank, dst.rank)
            cost = ("rrc:" if ins.kind == "rrc" else "link:") + suffix
            edge_res = topology.link(LinkKey(src.rank, dst.rank)).resource_ids
            resources = tuple(sorted(set(("link:" + suffix,) + tuple(edge_res))))
            flow = "%s:%d:%d:c%d" % (ins.kind, src.rank, dst.rank, ins.channel)
        else:
            cost, resources, flow = "copy:%d" % ins.rank, (), None
        ops.append(WorkOperation(key, ins.kind, Movement(cost, size), after=tuple(sorted(deps[key])),
                                 crosses=resources, flow_id=flow))
    outputs = sorted({storage.values[s].producer for s in storage.outputs.values()
                      if storage.values[s].producer is not None})
    return Executable(tuple(ops), tuple(outputs), dict(model_context))


def execution_dependencies(program: NativeProgram):
    """Operation-level dependencies implied by the native program.

    Collapses NOP chains onto the following step, adds TB order, checks that
    every dependency target publishes completion, and that each transfer has
    exactly one send and one matching receive on the same channel
    (reference: vericcl/xml/v5_program.py:140-190).
    """
    steps = {(b.rank, b.tb_id, i): s for b in program.blocks for i, s in enumerate(b.steps)}
    deps, members = defaultdict(set), defaultdict(list)
    for block in program.blocks:
        previous, waiting = None, set()
        for i, step in enumerate(block.steps):
            if (step.dependency_tb == -1) != (step.dependency_step == -1):
                raise SemanticError("native dependency must name both TB and step")
            if step.dependency_tb >= 0:
                target = steps.get((block.rank, step.dependency_tb, step.dependency_step))
                if target is None or target.kind == "nop" or not target.has_dependence:
                    raise SemanticError("dependency target is absent or does not publish completion")
                if step.dependency_tb == block.tb_id and step.dependency_step >= i:
                    raise SemanticError("dependency points at the same or a later step")
                waiting.add(target.operation_id)
            if step.kind == "nop":
                if step.dependency_tb < 0:
                    raise SemanticError("dependency-only NOP must carry a dependency")
                continue
            if waiting and step.dependency_tb < 0:
                raise SemanticError("a NOP chain must end in a step that also carries a dependency")
            if previous is not None and previous != step.operation_id:
                deps[step.operation_id].add(previous)
            deps[step.operation_id].update(waiting)
            if step.operation_id in deps[step.operation_id]:
                raise SemanticError("operation depends on its own completion")
            waiting.clear()
            previous = step.operation_id
            members[step.operation_id].append((block, step))
        if waiting:
            raise SemanticError("a trailing NOP chain has no native operation")
    for key, eps in members.items():
        if len(eps) == 1 and eps[0][1].kind in ("cpy", "re"):
            continue
        sends = [(b, s) for b, s in eps if s.kind == "s"]
        recvs = [(b, s) for b, s in eps if s.kind in ("r", "rrc")]
        if len(eps) != 2 or len(sends) != 1 or len(recvs) != 1:
            raise SemanticError("transfer %s must have exactly one send and one receive" % key)
        (sb, _), (rb, _) = sends[0], recvs[0]
        if sb.send_peer != rb.rank or rb.recv_peer != sb.rank or sb.channel != rb.channel:
            raise SemanticError("transfer %s endpoints disagree on peers or channel" % key)
    _check_acyclic({k: deps[k] for k in members})
    return {k: frozenset(deps[k]) for k in members}, members


def _check_acyclic(graph):
    indeg = {k: 0 for k in graph}
    succ = defaultdict(list)
    for k, ds in graph.items():
        for d in ds:
            if d not in graph:
                raise SemanticError("native dependency names an unknown operation")
            indeg[k] += 1
            succ[d].append(k)
    stack = [k for k, d in indeg.items() if d == 0]
    seen = 0
    while stack:
        k = stack.pop()
        seen += 1
        for nxt in succ[k]:
            indeg[nxt] -= 1
            if indeg[nxt] == 0:
                stack.append(nxt)
    if seen != len(graph):
        raise SemanticError("native endpoint/TB dependency graph is deadlocked")
