"""Step traces of the interpreter: binary format, parsing and causality.

With tracing enabled the interpreter's CTAs record, for every (iteration,
step), the %globaltimer value when the step's waits were satisfied and when
its data work finished.  A rank's trace file is a 40-byte header (magic,
version, rank, CTA count, steps per CTA, record count) followed by 64-byte
records (CTA, block, lane, iteration, step, op, start, end, wait, reserved),
mirroring the reference's fixed-size layout (vericcl/verification/online/
trace_format.py:18-19 and runtime/msccl-trace/include/vericcl_trace_format.h).
``analyze_trace_causality`` maps every record to host time with the clock
maps, then reports per-rank spans, the slowest steps ("tails"), waits that
dominate, and the cross-GPU orderings that are uncertain.
"""
from __future__ import annotations

import struct
from dataclasses import dataclass

from vericcl_b200.online.clock_sync import ordered

MAGIC = 0x56425452      # "VBTR"
HEADER = struct.Struct("<IIiiiiqq")            # magic, version, rank, ctas, steps, pad, records, reserved
RECORD = struct.Struct("<iiiiiiqqq" + "16x")   # cta, block, lane, iter, step, op, start, end, wait
assert HEADER.size == 40 and RECORD.size == 64


@dataclass(frozen=True)
class TraceRecord:
    rank: int
    cta: int
    block: int
    lane: int
    iteration: int
    step: int
    op: int
    start_ns: int
    end_ns: int
    wait_ns: int


def write_trace(path, rank: int, ctas: int, steps: int, records) -> None:
    with open(path, "wb") as handle:
        handle.write(HEADER.pack(MAGIC, 1, rank, ctas, steps, 0, len(records), 0))
        for r in records:
            handle.write(RECORD.pack(r.cta, r.block, r.lane, r.iteration, r.step, r.op, r.start_ns, r.end_ns,
                                     r.wait_ns))


def parse_trace(data: bytes, *, partial_ok: bool = True):
    if len(data) < HEADER.size:
        raise ValueError("trace shorter than its header")
    magic, version, rank, ctas, steps, _pad, count, _res = HEADER.unpack_from(data, 0)
    if magic != MAGIC or version != 1:
        raise ValueError("not a vericcl_b200 trace")
    available = (len(data) - HEADER.size) // RECORD.size
    if available < count and not partial_ok:
        raise ValueError("trace truncated: %d of %d records" % (available, count))
    out = []
    for i in range(min(count, available)):
        f = RECORD.unpack_from(data, HEADER.size + i * RECORD.size)
        out.append(TraceRecord(rank, *f))
    return {"rank": rank, "ctas": ctas, "steps": steps, "declared": count, "records": out,
            "complete": available >= count}


def records_from_buffer(rank, buffer, *, nblocks, nlanes, steps_per_iter, niters, ops=None, block_ops=None):
    """Decode the kernel's raw (start, end, wait) triples into records.

    CTA ``c`` (block ``c // nlanes``) owns ``steps_per_iter * niters`` slots
    from ``c * steps_per_iter * niters``; its record for (iteration ``i``,
    step ``s``) sits at slot ``i * nsteps(block) + s``.  ``block_ops`` gives
    every block's step opcodes (and so its step count); ``ops`` is the
    single-layout form where every block has ``steps_per_iter`` steps.
    """
    out = []
    per_cta = steps_per_iter * niters
    for cta in range(nblocks * nlanes):
        block, lane = cta // nlanes, cta % nlanes
        bops = block_ops[block] if block_ops is not None else (ops or [])
        nsteps = len(bops) if block_ops is not None else steps_per_iter
        for it in range(niters):
            for s in range(nsteps):
                base = (cta * per_cta + it * nsteps + s) * 3
                start, end, wait = buffer[base], buffer[base + 1], buffer[base + 2]
                if start == 0 and end == 0:
                    continue
                out.append(TraceRecord(rank, cta, block, lane, it, s, bops[s] if s < len(bops) else -1, int(start),
                                       int(end), int(wait)))
    return out


def step_counters(records) -> dict:
    """Per-step counters over every captured launch, iteration and lane.

    ``{(rank, block, step): {"samples", "service_ns", "dependency_wait_ns",
    "mean_service_ns", "mean_wait_ns", "max_service_ns", "first_ns",
    "last_ns"}}`` where service is end − start (data work after the waits)
    and the wait is the time the step spent on its dependencies — the same
    quantities as the reference's light probe counters
    (runtime/msccl-trace/patches/0003 lines 62-78), accumulated on the host
    from trace records instead of in a device table, so the interpreter's
    hot loop carries no extra atomics.
    """
    out = {}
    for r in records:
        key = (r.rank, r.block, r.step)
        c = out.get(key)
        service = max(0, r.end_ns - r.start_ns)
        if c is None:
            c = out[key] = {"samples": 0, "service_ns": 0, "dependency_wait_ns": 0, "max_service_ns": 0,
                            "first_ns": r.start_ns, "last_ns": r.end_ns}
        c["samples"] += 1
        c["service_ns"] += service
        c["dependency_wait_ns"] += max(0, r.wait_ns)
        c["max_service_ns"] = max(c["max_service_ns"], service)
        c["first_ns"] = min(c["first_ns"], r.start_ns)
        c["last_ns"] = max(c["last_ns"], r.end_ns)
    for c in out.values():
        c["mean_service_ns"] = c["service_ns"] / c["samples"]
        c["mean_wait_ns"] = c["dependency_wait_ns"] / c["samples"]
    return out


def analyze_trace_causality(traces, clock_maps, *, tails: int = 5):
    """Span per rank, slowest steps, dominant waits and uncertain cross-rank orders."""
    spans, steps, waits = {}, [], []
    for rank, recs in traces.items():
        cmap = clock_maps[rank]
        if not recs:
            continue
        t0 = min(cmap.to_host(r.start_ns) for r in recs)
        t1 = max(cmap.to_host(r.end_ns) for r in recs)
        spans[rank] = (t0, t1)
        for r in recs:
            steps.append((cmap.to_host(r.end_ns) - cmap.to_host(r.start_ns), rank, r.step, r.iteration, r.lane))
            waits.append((r.wait_ns, rank, r.step, r.iteration, r.lane))
    steps.sort(reverse=True)
    waits.sort(reverse=True)
    uncertain = []
    ranks = sorted(spans)
    for i, a in enumerate(ranks):
        for b in ranks[i + 1:]:
            if ordered(spans[a], spans[b]) == "uncertain":
                uncertain.append((a, b))
    first = min((s[0] for s in spans.values()), default=0.0)
    last = max((s[1] for s in spans.values()), default=0.0)
    return {"global_span_us": (last - first) / 1e3,
            "rank_spans_us": {r: ((s[1] - s[0]) / 1e3) for r, s in spans.items()},
            "tails": [{"duration_us": d / 1e3, "rank": r, "step": s, "iteration": it, "lane": l}
                      for d, r, s, it, l in steps[:tails]],
            "dominant_waits": [{"wait_us": w / 1e3, "rank": r, "step": s, "iteration": it, "lane": l}
                               for w, r, s, it, l in waits[:tails]],
            "overlapping_ranks": uncertain}


def capture_once(comm, plan, inp, out, *, warmup: int = 3, op: str = "sum", scale=None, count_per_rank=None,
                 steady: bool = False):
    """Warm up, bracket one traced invocation with clock samples, return this rank's records + clock map.

    Every rank calls this collectively.  The returned dict holds the rank's
    decoded records and its fitted :class:`ClockMap`; gather them (for example
    with ``comm.all_gather_object``) and pass them to
    :func:`analyze_trace_causality`.  By default the traced launch follows a
    barrier (ranks start it at their own host pace); with ``steady`` it is
    enqueued right behind the warm-up launches, so the ranks enter it the way
    they enter back-to-back launches.
    """
    import torch
    from vericcl_b200.online.clock_sync import fit_transform
    buf = comm.trace_buffer(plan)
    if steady:
        torch.cuda.synchronize()
        before = comm.clock_samples()
        comm.barrier()
        for _ in range(max(1, warmup)):
            comm.run(plan, inp, out, op=op, scale=scale, count_per_rank=count_per_rank)
        comm.run(plan, inp, out, op=op, scale=scale, count_per_rank=count_per_rank, trace=buf)
    else:
        for _ in range(warmup):
            comm.run(plan, inp, out, op=op, scale=scale, count_per_rank=count_per_rank)
        torch.cuda.synchronize()
        before = comm.clock_samples()
        comm.barrier()
        comm.run(plan, inp, out, op=op, scale=scale, count_per_rank=count_per_rank, trace=buf)
    torch.cuda.synchronize()
    comm.check_status()
    after = comm.clock_samples()
    raw = buf.cpu().tolist()
    records = records_from_buffer(comm.rank, raw, nblocks=plan.device_plan.nblocks, nlanes=plan.nlanes,
                                  steps_per_iter=plan.device_plan.max_steps(), niters=plan.niters,
                                  block_ops=plan.device_plan.block_ops())
    return {"rank": comm.rank, "records": records, "clock": fit_transform(before + after)}
