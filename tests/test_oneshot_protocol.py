"""Model check of the one-shot flag-in-data protocol (csrc/cuda/oneshot.cu) under adversarial interleavings.

Every rank runs launches 0..K-1 in stream order.  A launch pushes each of
its lines, as two independently delivered 8-byte halves {data, tag}, into
its slot of every peer's region half ``seq & 1``, then waits for every
peer's lines of this launch (both tags equal ``tag(seq)``) and checks the
data.  Stores become visible in any order and at any later time (only each
8-byte half is atomic).  The checker explores random schedules: with the
two-half region every read sees the right launch's data and every run
finishes; with a single region (no parity), some schedule deadlocks or
reads the wrong launch, which is why the kernel alternates halves.
"""
import random

import pytest


def tag(seq):
    return seq % 0xFFFFFFFE + 1


def simulate(p, launches, units, seed, halves=2, max_events=200000):
    rng = random.Random(seed)
    # region[dst][half][src][unit] = [(tag, data) low, (tag, data) high]
    region = [[[[[(0, None), (0, None)] for _ in range(units)] for _ in range(p)] for _ in range(halves)]
              for _ in range(p)]
    in_flight = []                        # (dst, half, src, unit, which, tag, data)
    state = [{"seq": 0, "phase": "push", "next": 0} for _ in range(p)]
    events = 0
    while any(s["seq"] < launches for s in state):
        events += 1
        if events > max_events:
            return "deadlock"
        choices = [("deliver", i) for i in range(len(in_flight))]
        for r in range(p):
            if state[r]["seq"] < launches:
                choices.append(("rank", r))
        kind, idx = rng.choice(choices)
        if kind == "deliver":
            dst, half, src, unit, which, t, data = in_flight.pop(idx)
            region[dst][half][src][unit][which] = (t, data)
            continue
        r = idx
        s = state[r]
        seq = s["seq"]
        h = seq % halves
        if s["phase"] == "push":
            u = s["next"]
            for q in range(p):
                if q == r:
                    continue
                for which in (0, 1):
                    in_flight.append((q, h, r, u, which, tag(seq), (r, seq, u, which)))
            s["next"] += 1
            if s["next"] == units:
                s["phase"], s["next"] = "read", 0
            continue
        # read phase: one (source, unit) slot per step, in order; spin (no progress) until both tags match
        pending = [(src, u) for src in range(p) if src != r for u in range(units)]
        if s["next"] < len(pending):
            src, u = pending[s["next"]]
            lo, hi = region[r][h][src][u]
            if lo[0] == tag(seq) and hi[0] == tag(seq):
                if lo[1] != (src, seq, u, 0) or hi[1] != (src, seq, u, 1):
                    return "wrong data"
                s["next"] += 1
            continue
        s["seq"], s["phase"], s["next"] = seq + 1, "push", 0
    return "ok"


@pytest.mark.parametrize("seed", range(40))
def test_two_halves_always_deliver_the_right_launch(seed):
    assert simulate(3, 5, 2, seed) == "ok"


def test_single_region_is_unsafe():
    outcomes = {simulate(3, 5, 2, seed, halves=1, max_events=20000) for seed in range(60)}
    assert outcomes - {"ok"}, "expected some schedule to deadlock or read another launch's data"


def simulate_mixed(p, kinds, units, seed, max_events=400000):
    """One-shot and two-shot AllReduce launches sharing the same two region halves (flat addresses)."""
    rng = random.Random(seed)
    halves = 2
    mem = [[{} for _ in range(halves)] for _ in range(p)]          # mem[dst][half][address] = (tag, data)
    in_flight = []
    line = 2                                                         # two 8-byte halves per line

    def addr_one(src, u, which):                                     # one-shot: [src][units lines]
        return (src * units + u) * line + which

    def addr_rs(src, u, which):                                      # two-shot: reduce-scatter area first
        return (src * units + u) * line + which

    def addr_ag(owner, u, which):                                    # then the all-gather area
        return ((p + owner) * units + u) * line + which

    def push(dst, h, addr, t, data):
        in_flight.append((dst, h, addr, t, data))

    def ready(r, h, addr, t):
        got = mem[r][h].get(addr)
        return got is not None and got[0] == t, (got[1] if got else None)

    state = [{"i": 0, "step": 0, "pc": 0} for _ in range(p)]
    events = 0
    while any(s["i"] < len(kinds) for s in state):
        events += 1
        if events > max_events:
            return "deadlock"
        choices = [("deliver", i) for i in range(len(in_flight))] + \
                  [("rank", r) for r in range(p) if state[r]["i"] < len(kinds)]
        kind, idx = rng.choice(choices)
        if kind == "deliver":
            dst, h, addr, t, data = in_flight.pop(idx)
            mem[dst][h][addr] = (t, data)
            continue
        r, s = idx, state[idx]
        seq = s["i"]
        t, h = tag(seq), seq % halves
        if kinds[seq] == "one":
            program = [("push", None)] + [("read", (src, u)) for src in range(p) if src != r for u in range(units)]
        else:
            program = [("rs_push", None)] + [("rs_read", (src, u)) for src in range(p) if src != r
                                               for u in range(units)] + [("ag_push", None)] + \
                      [("ag_read", (j, u)) for j in range(p) if j != r for u in range(units)]
        if s["pc"] == len(program):
            s["i"], s["pc"] = seq + 1, 0
            continue
        op, arg = program[s["pc"]]
        if op == "push":
            for q in range(p):
                if q != r:
                    for u in range(units):
                        for w in (0, 1):
                            push(q, h, addr_one(r, u, w), t, ("one", r, seq, u, w))
        elif op == "rs_push":
            for j in range(p):
                if j != r:
                    for u in range(units):
                        for w in (0, 1):
                            push(j, h, addr_rs(r, u, w), t, ("rs", r, j, seq, u, w))
        elif op == "ag_push":
            for q in range(p):
                if q != r:
                    for u in range(units):
                        for w in (0, 1):
                            push(q, h, addr_ag(r, u, w), t, ("ag", r, seq, u, w))
        else:
            src, u = arg
            if op == "read":
                addr, want = addr_one, lambda w: ("one", src, seq, u, w)
            elif op == "rs_read":
                addr, want = addr_rs, lambda w: ("rs", src, r, seq, u, w)
            else:
                addr, want = addr_ag, lambda w: ("ag", src, seq, u, w)
            ok0, d0 = ready(r, h, addr(src, u, 0), t)
            ok1, d1 = ready(r, h, addr(src, u, 1), t)
            if not (ok0 and ok1):
                continue                                             # spin
            if d0 != want(0) or d1 != want(1):
                return "wrong data"
        s["pc"] += 1
    return "ok"


@pytest.mark.parametrize("seed", range(30))
def test_mixed_one_and_two_shot_launches_share_the_halves_safely(seed):
    rng = random.Random(1000 + seed)
    kinds = [rng.choice(["one", "two"]) for _ in range(6)]
    assert simulate_mixed(3, kinds, 2, seed) == "ok"
