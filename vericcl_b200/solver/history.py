"""Cross-run schedule history: find, adapt and save accepted schedules.

Entries are keyed by the topology's exact isomorphism signature, the
collective (kind, datatype, reduction, in-place) and the slice partition.
A lookup relabels a stored schedule's ranks onto the current topology's
canonical labelling and accepts it when the relative bandwidth scale between
the stored and the current links stays within the tolerance; the adapted
XML is then revalidated by the normal checks (reference:
vericcl/solver/history_index.py:62-146).
"""
from __future__ import annotations

import json
import time
from pathlib import Path

from vericcl_b200.topology.isomorphism import canonical_labelling


def _key(request, signature):
    c = request.collective
    return "|".join([signature, c.kind.value, c.datatype, str(c.reduction_op), str(c.inplace),
                     str(request.hyperparameters.total_size_bytes), str(request.hyperparameters.slice_size_bytes)])


def save_schedule(index_path, request, topology, xml: str, t_pred_us: float) -> None:
    sig, mapping = canonical_labelling(topology)
    path = Path(index_path)
    data = json.loads(path.read_text()) if path.exists() else {}
    inverse = {new: old for old, new in mapping.items()}
    data.setdefault(_key(request, sig), []).append({
        "xml_canonical": relabel_xml(xml, mapping), "t_pred_us": t_pred_us, "saved": time.time(),
        "bandwidth": sorted(1.0 / l.beta_us_per_byte for l in topology.links.values())})
    path.parent.mkdir(parents=True, exist_ok=True)
    path.write_text(json.dumps(data, indent=1))


def find_schedules(index_path, request, topology, *, tolerance: float, limit: int):
    path = Path(index_path)
    if not path.exists():
        return []
    sig, mapping = canonical_labelling(topology)
    inverse = {new: old for old, new in mapping.items()}
    current = sorted(1.0 / l.beta_us_per_byte for l in topology.links.values())
    out = []
    data = json.loads(path.read_text())
    if request.hyperparameters.slice_size_bytes is None:
        # no fixed slice size: schedules saved for any slice size of this problem qualify
        prefix = _key(request, sig).rsplit("|", 1)[0] + "|"
        entries = [e for k in sorted(data) if k.startswith(prefix) for e in data[k]]
    else:
        entries = data.get(_key(request, sig), [])
    for entry in entries:
        scales = [a / b for a, b in zip(current, entry["bandwidth"]) if b]
        if scales and max(scales) / min(scales) - 1.0 > tolerance:
            continue
        out.append({"xml": relabel_xml(entry["xml_canonical"], inverse), "t_pred_us": entry["t_pred_us"]})
        if len(out) >= limit:
            break
    return out


def relabel_xml(xml: str, mapping: dict) -> str:
    """Rename ranks of an XML schedule (gpu ids and TB peers) with ``mapping``."""
    from vericcl_b200.program.model import NativeBlock
    from vericcl_b200.program.xmlio import emit_xml, parse_xml
    from dataclasses import replace
    prog = parse_xml(xml)
    m = lambda r: mapping.get(r, r) if r >= 0 else r
    blocks = []
    for b in prog.blocks:
        steps = tuple(replace(s, src=None if s.src is None else replace(s.src, rank=m(b.rank)),
                              dst=None if s.dst is None else replace(s.dst, rank=m(b.rank))) for s in b.steps)
        blocks.append(NativeBlock(m(b.rank), b.tb_id, b.channel, m(b.send_peer), m(b.recv_peer), steps))
    relabel = lambda d: {m(k): v for k, v in d.items()}
    prog = replace(prog, blocks=tuple(sorted(blocks, key=lambda x: (x.rank, x.tb_id))),
                   input_slots=relabel(prog.input_slots), output_slots=relabel(prog.output_slots),
                   scratch_slots=relabel(prog.scratch_slots))
    return emit_xml(prog)
