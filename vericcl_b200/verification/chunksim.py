"""Numeric chunk simulator of a native (XML) program with MSCCL semantics.

Every thread block executes its steps in order; a step first waits for its
explicit ``(depid, deps)`` dependency on the same rank.  Sends push one chunk
into the FIFO of their (sender, receiver, channel) connection and receives pop
from it in order, so a send never waits for its receiver.  The step kinds are
the MSCCL interpreter's: ``s r rrc rcs rrs rrcs cpy re nop``.  The simulator
runs on real NumPy buffers (float64 by default), so a schedule is checked on
numbers, not only on contributor sets: each output must equal the collective
of seeded inputs (the P=8 AllGather 1 MiB acceptance case uses uniform(-1, 1)).
It is also the CPU oracle for the GPU interpreter.
"""
from __future__ import annotations

from collections import defaultdict, deque

import numpy as np

from vericcl_b200.errors import SemanticError

OPS = {"sum": np.add, "prod": np.multiply, "max": np.maximum, "min": np.minimum, "avg": np.add}


def _views(program, rank, count, chunk, inputs, outputs, scratch):
    coll = program.collective
    n_in = program.input_slots.get(rank, 0)
    out = outputs[rank]
    if program.inplace:
        if coll == "allgather":
            inp = out[rank * n_in * chunk:(rank + 1) * n_in * chunk]
        elif coll == "reduce_scatter":
            inp = inputs[rank]
            out = inp[rank * program.output_slots[rank] * chunk:(rank + 1) * program.output_slots[rank] * chunk]
        else:
            inp = out
    else:
        inp = inputs[rank]
    return {"i": inp, "o": out, "s": scratch[rank]}


def run_program(program, inputs, outputs, *, op: str = "sum", chunk_elems: int, scratch=None, max_events=10_000_000,
                scale: float | None = None):
    """Execute ``program`` on per-rank arrays in place.  Returns per-rank outputs."""
    fn = OPS[op]
    p = program.rank_count
    if scratch is None:
        scratch = [np.zeros(max(1, program.scratch_slots.get(r, 0)) * chunk_elems, dtype=outputs[r].dtype)
                   for r in range(p)]
    views = [_views(program, r, None, chunk_elems, inputs, outputs, scratch) for r in range(p)]

    def region(rank, addr, cnt):
        buf = views[rank][addr.buffer]
        lo = addr.offset * chunk_elems
        hi = lo + cnt * chunk_elems
        if hi > buf.shape[0]:
            raise SemanticError("rank %d buffer %s offset %d exceeds its slots" % (rank, addr.buffer, addr.offset))
        return buf[lo:hi]

    blocks = {(b.rank, b.tb_id): b for b in program.blocks}
    pc = {key: 0 for key in blocks}
    done = defaultdict(set)            # rank -> {(tb, step)}
    fifos = defaultdict(deque)         # (src, dst, chan) -> chunks
    remaining = sum(len(b.steps) for b in blocks.values())
    events = 0
    while remaining:
        progressed = False
        for key, block in blocks.items():
            while pc[key] < len(block.steps):
                step = block.steps[pc[key]]
                rank = block.rank
                if step.dependency_tb >= 0 and (step.dependency_tb, step.dependency_step) not in done[rank]:
                    break
                kind = step.kind
                if kind in ("r", "rrc", "rcs", "rrs", "rrcs"):
                    fifo = fifos[(block.recv_peer, rank, block.channel)]
                    if not fifo:
                        break
                    value = fifo.popleft()
                    if kind == "r":
                        region(rank, step.dst, step.count)[:] = value
                    elif kind == "rcs":
                        region(rank, step.dst, step.count)[:] = value
                        fifos[(rank, block.send_peer, block.channel)].append(value.copy())
                    elif kind == "rrc":
                        region(rank, step.dst, step.count)[:] = fn(value, region(rank, step.src, step.count))
                    elif kind == "rrs":
                        fifos[(rank, block.send_peer, block.channel)].append(fn(value, region(rank, step.src,
                                                                                              step.count)))
                    else:
                        result = fn(value, region(rank, step.src, step.count))
                        region(rank, step.dst, step.count)[:] = result
                        fifos[(rank, block.send_peer, block.channel)].append(result.copy())
                elif kind == "s":
                    if block.send_peer < 0:
                        raise SemanticError("send step in a TB without a send peer")
                    fifos[(rank, block.send_peer, block.channel)].append(region(rank, step.src, step.count).copy())
                elif kind == "cpy":
                    region(rank, step.dst, step.count)[:] = region(rank, step.src, step.count)
                elif kind == "re":
                    dst = region(rank, step.dst, step.count)
                    dst[:] = fn(region(rank, step.src, step.count), dst)
                done[rank].add((block.tb_id, pc[key]))
                pc[key] += 1
                remaining -= 1
                progressed = True
                events += 1
                if events > max_events:
                    raise SemanticError("chunk simulation exceeded its event budget")
        if not progressed:
            stuck = [(k, blocks[k].steps[pc[k]].kind) for k in blocks if pc[k] < len(blocks[k].steps)]
            raise SemanticError("chunk simulation deadlocked at %s" % stuck[:8])
    leftovers = {k: len(v) for k, v in fifos.items() if v}
    if leftovers:
        raise SemanticError("unconsumed sends remain on connections %s" % sorted(leftovers))
    if scale is not None or op == "avg":
        factor = scale if scale is not None else 1.0 / p
        for r in range(p):
            outputs[r][:] = outputs[r] * factor if op != "avg" or scale is not None else outputs[r] / p
    return outputs


def reference_result(collective: str, inputs, *, op="sum", root=0, slice_count=1, rank_count=None):
    """fp64 NumPy reference of the collective on per-rank inputs."""
    p = len(inputs) if rank_count is None else rank_count
    x = [np.asarray(a, dtype=np.float64) for a in inputs]
    if collective == "allreduce":
        total = x[0].copy()
        for a in x[1:]:
            total = OPS[op](total, a)
        if op == "avg":
            total = total / p
        return [total.copy() for _ in range(p)]
    if collective == "allgather":
        full = np.concatenate(x)
        return [full.copy() for _ in range(p)]
    if collective == "reduce_scatter":
        total = x[0].copy()
        for a in x[1:]:
            total = OPS[op](total, a)
        part = total.shape[0] // p
        return [total[r * part:(r + 1) * part].copy() for r in range(p)]
    if collective == "broadcast":
        return [x[root].copy() for _ in range(p)]
    if collective == "reduce":
        total = x[0].copy()
        for a in x[1:]:
            total = OPS[op](total, a)
        return [total if r == root else None for r in range(p)]
    if collective == "alltoall":
        part = x[0].shape[0] // p
        return [np.concatenate([x[s][d * part:(d + 1) * part] for s in range(p)]) for d in range(p)]
    raise SemanticError("no reference for " + collective)


def check_program_numerics(program, *, count_per_rank: int, op: str = "sum", seed: int = 0, root: int = 0,
                           distribution: str = "uniform", atol=1e-9, rtol=1e-9):
    """Run ``program`` on seeded data; return (ok, max_abs_error)."""
    rng = np.random.default_rng(seed)
    p = program.rank_count
    coll = program.collective
    runtime = count_per_rank * (p if coll == "allgather" else 1)
    if runtime % program.chunks_per_loop:
        raise SemanticError("count is not divisible by nchunksperloop")
    chunk = runtime // program.chunks_per_loop
    if distribution == "uniform":
        inputs = [rng.uniform(-1, 1, count_per_rank) for _ in range(p)]
    else:
        inputs = [rng.standard_normal(count_per_rank) for _ in range(p)]
    out_len = {"allgather": count_per_rank * p, "reduce_scatter": count_per_rank // p}.get(coll, count_per_rank)
    outputs = [np.full(out_len, np.nan) for _ in range(p)]
    if program.inplace:
        if coll == "allgather":
            for r in range(p):
                outputs[r][r * count_per_rank:(r + 1) * count_per_rank] = inputs[r]
        elif coll != "reduce_scatter":
            outputs = [a.copy() for a in inputs]
    expected = reference_result(coll, [a.copy() for a in inputs], op=op, root=root, rank_count=p)
    run_program(program, inputs, outputs, op=op, chunk_elems=chunk)
    if coll == "reduce_scatter" and program.inplace:
        outputs = [inputs[r][r * out_len:(r + 1) * out_len] for r in range(p)]
    worst = 0.0
    for r in range(p):
        if expected[r] is None:
            continue
        err = np.abs(outputs[r] - expected[r])
        if not np.all(np.isfinite(outputs[r])):
            return False, float("inf")
        worst = max(worst, float(err.max(initial=0.0)))
        if not np.allclose(outputs[r], expected[r], atol=atol, rtol=rtol):
            return False, worst
    return True, worst
