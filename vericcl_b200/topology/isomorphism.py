"""Exact isomorphism signature of a topology's rank domain.

Used by the history index to reuse schedules across rank relabellings
(reference: vericcl/topology/isomorphism.py:293).  The signature is a
canonical form computed by trying every relabelling that is consistent with
iteratively refined vertex colours (Weisfeiler-Lehman); for the symmetric
NVSwitch domains used here that collapses to one candidate quickly.
"""
from __future__ import annotations

import itertools

from vericcl_b200.topology.model import Topology
from vericcl_b200.utils.hashing import digest


def _costs(topology: Topology):
    return {(k.src, k.dst): (round(l.alpha_us, 9), round(l.beta_us_per_byte, 15), l.max_channels)
            for k, l in topology.links.items()}


def refine_colors(topology: Topology, rounds: int = 4):
    costs = _costs(topology)
    colors = {r: 0 for r in range(topology.rank_count)}
    for _ in range(rounds):
        sig = {}
        for r in range(topology.rank_count):
            out = sorted((colors[d], costs[(r, d)]) for (s, d) in costs if s == r)
            inn = sorted((colors[s], costs[(s, r)]) for (s, d) in costs if d == r)
            sig[r] = (colors[r], tuple(out), tuple(inn))
        order = {value: i for i, value in enumerate(sorted(set(sig.values()), key=repr))}
        new = {r: order[sig[r]] for r in sig}
        if new == colors:
            break
        colors = new
    return colors


def canonical_labelling(topology: Topology, max_candidates: int = 5040):
    """Return (signature digest, mapping old->canonical rank)."""
    costs = _costs(topology)
    colors = refine_colors(topology)
    classes = {}
    for r, c in colors.items():
        classes.setdefault(c, []).append(r)
    ordered = [sorted(classes[c]) for c in sorted(classes)]
    best = None
    count = 0
    for perms in itertools.product(*[itertools.permutations(group) for group in ordered]):
        count += 1
        if count > max_candidates:
            break
        order = [r for group in perms for r in group]
        mapping = {old: new for new, old in enumerate(order)}
        form = tuple(sorted((mapping[s], mapping[d], v) for (s, d), v in costs.items()))
        if best is None or form < best[0]:
            best = (form, mapping)
    return digest([list(map(list, best[0])), topology.rank_count]), best[1]


def exact_domain_signature(topology: Topology) -> str:
    return canonical_labelling(topology)[0]
