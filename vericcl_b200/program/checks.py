"""The eight admission checks of a lowered candidate.

Dimensions (reference: vericcl/xml/v5_lower.py:27 and 246-335):
semantic, storage, endpoint, deadlock, xml, launch, compatibility,
prediction.  Each check returns ``{"status": valid|invalid|not_run,
"detail": ...}``; a candidate may execute only when the first seven required
ones are valid and compatibility is valid or not run.

* semantic — symbolic replay of the native program under MSCCL FIFO
  semantics; every required output slot must hold exactly its contributor
  set and every reduction must combine disjoint sets of one logical index.
* storage — every address inside its i/o/s slots; scratch within budget.
* endpoint / deadlock — send/receive pairing and acyclicity of the
  operation graph (TB order + explicit dependencies + NOP chains).
* xml — parse(emit(program)) re-emits the identical canonical XML.
* launch — runtime structural limits (steps per TB, TBs per rank, channels,
  dependency ids, buffer offsets) and the interpreter's device-block limit.
* compatibility — the native compiler accepts the program under pull
  semantics (no reliance on FIFO buffering) and its device blocks (after
  block merging) fit the 148 co-resident CTAs of a B200; not run when the
  native module cannot be built.
* prediction — exact T_pred exists with no missing cost component.
"""
from __future__ import annotations

from collections import defaultdict, deque

from vericcl_b200.errors import SemanticError
from vericcl_b200.program.native import execution_dependencies
from vericcl_b200.program.xmlio import canonical_xml, emit_xml, parse_xml
from vericcl_b200.semantics.collective import CollectiveKind, required_outputs
from vericcl_b200.semantics.versions import canonical

MAX_DEVICE_BLOCKS = 512
# The interpreter is a cooperative launch of 512-thread CTAs using up to 128 registers each, so one CTA is
# resident per SM: a rank's device blocks (each with at least one lane) must fit the 148 SMs of a B200.
B200_RESIDENT_CTAS = 148


def _ok(detail=None):
    return {"status": "valid", "detail": detail}


def _bad(detail):
    return {"status": "invalid", "detail": str(detail)}


def symbolic_replay(program, spec, slice_count):
    """Replay ``program`` on contributor sets; return the final state map."""
    p = program.rank_count
    n = slice_count
    state = {}
    for rank in range(p):
        if spec.kind in (CollectiveKind.BROADCAST, CollectiveKind.SCATTER) and rank != spec.root:
            continue
        for index in range(program.input_slots.get(rank, 0)):
            state[canonical(spec, p, n, rank, "i", index)] = frozenset({rank * n + index})
    blocks = {(b.rank, b.tb_id): b for b in program.blocks}
    pc = {k: 0 for k in blocks}
    done = defaultdict(set)
    fifos = defaultdict(deque)
    remaining = sum(len(b.steps) for b in blocks.values())

    def read(rank, addr, k=0):
        key = canonical(spec, p, n, rank, addr.buffer, addr.offset + k)
        if key not in state:
            raise SemanticError("rank %d reads %s[%d] before it holds a value" % (rank, addr.buffer, addr.offset + k))
        return state[key]

    def write(rank, addr, value, k=0):
        state[canonical(spec, p, n, rank, addr.buffer, addr.offset + k)] = value

    def reduce(a, b):
        if a & b:
            raise SemanticError("reduction combines overlapping contributors %s and %s" % (sorted(a), sorted(b)))
        if len({s % n for s in a | b}) != 1:
            raise SemanticError("reduction mixes logical slice positions")
        return a | b

    while remaining:
        progressed = False
        for key, block in blocks.items():
            while pc[key] < len(block.steps):
                st = block.steps[pc[key]]
                rank = block.rank
                if st.dependency_tb >= 0 and (st.dependency_tb, st.dependency_step) not in done[rank]:
                    break
                kind = st.kind
                cnt = st.count
                if kind in ("r", "rrc", "rcs", "rrs", "rrcs"):
                    fifo = fifos[(block.recv_peer, rank, block.channel)]
                    if not fifo:
                        break
                    values = fifo.popleft()
                    for k in range(cnt):
                        v = values[k]
                        if kind in ("rrc", "rrs", "rrcs"):
                            v = reduce(v, read(rank, st.src, k))
                        if kind in ("r", "rcs", "rrc", "rrcs"):
                            write(rank, st.dst, v, k)
                        values[k] = v
                    if kind in ("rcs", "rrs", "rrcs"):
                        fifos[(rank, block.send_peer, block.channel)].append(list(values))
                elif kind == "s":
                    fifos[(rank, block.send_peer, block.channel)].append([read(rank, st.src, k) for k in range(cnt)])
                elif kind == "cpy":
                    for k in range(cnt):
                        write(rank, st.dst, read(rank, st.src, k), k)
                elif kind == "re":
                    for k in range(cnt):
                        write(rank, st.dst, reduce(read(rank, st.src, k), read(rank, st.dst, k)), k)
                done[rank].add((block.tb_id, pc[key]))
                pc[key] += 1
                remaining -= 1
                progressed = True
        if not progressed:
            raise SemanticError("symbolic replay deadlocks")
    if any(fifos.values()):
        raise SemanticError("sends remain unconsumed")
    return state


def check_semantics(program, spec, slice_count):
    state = symbolic_replay(program, spec, slice_count)
    p = program.rank_count
    problems = []
    for slot, expected in sorted(required_outputs(spec, p, slice_count).items()):
        got = state.get(canonical(spec, p, slice_count, slot.rank, "o", slot.offset))
        if got != expected:
            problems.append("output %d:%d holds %s, expected %s" % (slot.rank, slot.offset,
                                                                    None if got is None else sorted(got),
                                                                    sorted(expected)))
    return problems


def check_storage(program, request):
    size = request.hyperparameters.slice_size_bytes
    budget = request.request_config["runtime"]["scratch_bytes_per_rank"]
    limits = request.request_config["runtime"]["limits"]
    issues = []
    for block in program.blocks:
        slots = {"i": program.input_slots.get(block.rank, 0), "o": program.output_slots.get(block.rank, 0),
                 "s": program.scratch_slots.get(block.rank, 0)}
        for st in block.steps:
            # a send's dst and a receive's src name the peer's buffer and are informational
            used = {"s": (st.src,), "r": (st.dst,), "rcs": (st.dst,), "nop": ()}.get(st.kind, (st.src, st.dst))
            for addr in used:
                if addr is None:
                    continue
                if addr.offset > limits["buffer_offset"]:
                    issues.append("offset %d exceeds the runtime buffer_offset limit" % addr.offset)
                if addr.offset + st.count > slots[addr.buffer] and not (program.inplace and addr.buffer == "i"):
                    issues.append("rank %d %s[%d] outside its %d slots" % (block.rank, addr.buffer, addr.offset,
                                                                          slots[addr.buffer]))
    for rank, count in program.scratch_slots.items():
        if count * size > budget:
            issues.append("rank %d needs %d scratch bytes, budget %d" % (rank, count * size, budget))
    device_budget = request.request_config["runtime"].get("device_memory_budget_bytes") or 0
    if device_budget > 0:
        # input, output and scratch buffers of the schedule, per rank (0 = no budget)
        for rank in range(program.rank_count):
            total = (program.input_slots.get(rank, 0) + program.output_slots.get(rank, 0)
                     + program.scratch_slots.get(rank, 0)) * size
            if total > device_budget:
                issues.append("rank %d needs %d device bytes, budget %d" % (rank, total, device_budget))
    return issues


def check_launch(program, request):
    limits = request.request_config["runtime"]["limits"]
    issues = []
    per_rank = defaultdict(int)
    directions = defaultdict(int)
    for block in program.blocks:
        per_rank[block.rank] += 1
        if len(block.steps) > limits["steps_per_tb"]:
            issues.append("rank %d tb %d has %d steps" % (block.rank, block.tb_id, len(block.steps)))
        for st in block.steps:
            if st.dependency_tb > limits["dependency_id"]:
                issues.append("dependency id %d exceeds the limit" % st.dependency_tb)
        if block.send_peer >= 0:
            directions[(block.rank, block.channel, "send")] += 1
        if block.recv_peer >= 0:
            directions[(block.rank, block.channel, "recv")] += 1
    for rank, count in per_rank.items():
        if count > limits["tbs_per_rank"]:
            issues.append("rank %d has %d TBs" % (rank, count))
        if count > MAX_DEVICE_BLOCKS:
            issues.append("rank %d has more TBs than the interpreter's flag table" % rank)
    for (rank, channel, d), count in directions.items():
        if count > limits[d + "_tbs_per_channel"]:
            issues.append("rank %d channel %d has %d %s TBs" % (rank, channel, count, d))
    if program.channels > 16:
        issues.append("%d channels exceed 16" % program.channels)
    return issues


def evaluate_program(bundle, topology) -> dict:
    request = bundle.request
    program = bundle.program
    n = request.hyperparameters.slice_count
    checks = {}
    try:
        problems = check_semantics(program, request.collective, n)
        checks["semantic"] = _ok() if not problems else _bad("; ".join(problems[:5]))
    except SemanticError as error:
        checks["semantic"] = _bad(error)
    issues = check_storage(program, request)
    checks["storage"] = (_ok({"scratch_slots": dict(program.scratch_slots)}) if not issues
                         else _bad("; ".join(issues[:5])))
    try:
        deps, members = execution_dependencies(program)
        checks["endpoint"] = _ok({"operations": len(members)})
        checks["deadlock"] = _ok()
    except SemanticError as error:
        text = str(error)
        checks["endpoint"] = _bad(text) if "send" in text or "endpoint" in text else _ok()
        checks["deadlock"] = _bad(text) if "deadlock" in text or "cycle" in text else checks.get("deadlock", _ok())
    try:
        again = emit_xml(parse_xml(bundle.xml))
        checks["xml"] = _ok() if canonical_xml(again) == canonical_xml(bundle.xml) else _bad("re-emission differs")
    except SemanticError as error:
        checks["xml"] = _bad(error)
    issues = check_launch(program, request)
    checks["launch"] = _ok() if not issues else _bad("; ".join(issues[:5]))
    if request.request_config["sketch"]["runtime_compatibility"]["enabled"]:
        try:
            from vericcl_b200.program.device import compile_xml
            compiled = compile_xml(bundle.xml, nlanes=1, niters=1)
            blocks = compiled.max_blocks
            if blocks > B200_RESIDENT_CTAS:
                checks["compatibility"] = _bad("%d device blocks on one rank exceed the %d CTAs that are co-resident "
                                               "on a B200 (one 512-thread interpreter CTA per SM)"
                                               % (blocks, B200_RESIDENT_CTAS))
            else:
                checks["compatibility"] = _ok(dict(compiled.stats, device_blocks=blocks))
        except SemanticError as error:
            checks["compatibility"] = _bad(error)
        except Exception as error:  # native module unavailable
            checks["compatibility"] = {"status": "not_run", "detail": str(error)}
    else:
        checks["compatibility"] = {"status": "not_run", "detail": "disabled by sketch.runtime_compatibility"}
    pred = bundle.prediction
    if pred is None or pred.t_pred_us is None:
        checks["prediction"] = _bad("missing components: %s" % (sorted(pred.missing_components) if pred else "all"))
    else:
        checks["prediction"] = _ok({"t_pred_us": pred.t_pred_us, "coverage": pred.model_coverage})
    return checks
