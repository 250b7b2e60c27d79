"""MSCCL-style XML emission and parsing.

Emission writes the attribute set used by MSCCL 0.1 algorithm files:
``<algo name nchannels nchunksperloop proto coll inplace redop ngpus minBytes
maxBytes>`` / ``<gpu id i_chunks o_chunks s_chunks>`` / ``<tb id send recv
chan>`` / ``<step s type srcbuf srcoff dstbuf dstoff cnt depid deps hasdep>``
(format: third_party/msccl/src/graph/topo.cc:771-970 in the reference tree).
Parsing accepts any such file, including hand-written MSCCL algorithms, and
returns a :class:`NativeProgram`.
"""
from __future__ import annotations

import xml.etree.ElementTree as ET

from vericcl_b200.errors import SemanticError
from vericcl_b200.program.model import Address, NativeBlock, NativeProgram, NativeStep

STEP_TYPES = frozenset({"s", "r", "rrc", "rcs", "rrs", "rrcs", "cpy", "re", "nop"})


def emit_xml(program: NativeProgram) -> str:
    lines = ['<algo name="%s" nchannels="%d" nchunksperloop="%d" proto="%s" coll="%s" inplace="%d" redop="%s" '
             'ngpus="%d" minBytes="%d" maxBytes="%d">' % (
                 program.name, program.channels, program.chunks_per_loop, program.proto, program.collective,
                 int(program.inplace), program.redop, program.rank_count, program.min_bytes, program.max_bytes)]
    for rank in range(program.rank_count):
        lines.append('  <gpu id="%d" i_chunks="%d" o_chunks="%d" s_chunks="%d">' % (
            rank, program.input_slots.get(rank, 0), program.output_slots.get(rank, 0),
            program.scratch_slots.get(rank, 0)))
        for block in program.rank_blocks(rank):
            lines.append('    <tb id="%d" send="%d" recv="%d" chan="%d">' % (block.tb_id, block.send_peer,
                                                                           block.recv_peer, block.channel))
            for i, step in enumerate(block.steps):
                src = step.src
                dst = step.dst
                lines.append('      <step s="%d" type="%s" srcbuf="%s" srcoff="%d" dstbuf="%s" dstoff="%d" cnt="%d" '
                             'depid="%d" deps="%d" hasdep="%d"/>' % (
                                 i, step.kind, src.buffer if src else "i", src.offset if src else -1,
                                 dst.buffer if dst else "o", dst.offset if dst else -1, step.count,
                                 step.dependency_tb, step.dependency_step, int(step.has_dependence)))
            lines.append("    </tb>")
        lines.append("  </gpu>")
    lines.append("</algo>")
    return "\n".join(lines) + "\n"


def _int(el, key, default=None):
    value = el.get(key)
    if value is None:
        if default is None:
            raise SemanticError("XML element <%s> lacks attribute %s" % (el.tag, key))
        return default
    try:
        return int(value)
    except ValueError:
        raise SemanticError("XML attribute %s=%r is not an integer" % (key, value)) from None


def parse_xml(text: str) -> NativeProgram:
    try:
        root = ET.fromstring(text)
    except ET.ParseError as error:
        raise SemanticError("invalid XML: %s" % error) from error
    if root.tag != "algo":
        raise SemanticError("root element must be <algo>")
    ngpus = _int(root, "ngpus")
    blocks, ins, outs, scr = [], {}, {}, {}
    for gpu in root.findall("gpu"):
        rank = _int(gpu, "id")
        ins[rank] = _int(gpu, "i_chunks", 0)
        outs[rank] = _int(gpu, "o_chunks", 0)
        scr[rank] = _int(gpu, "s_chunks", 0)
        for tb in gpu.findall("tb"):
            steps = []
            for i, st in enumerate(tb.findall("step")):
                kind = st.get("type")
                if kind not in STEP_TYPES:
                    raise SemanticError("unknown step type %r" % kind)
                if _int(st, "s") != i:
                    raise SemanticError("step indices must be dense and ordered")
                srcoff, dstoff = _int(st, "srcoff", -1), _int(st, "dstoff", -1)
                src = Address(rank, st.get("srcbuf", "i"), srcoff) if srcoff >= 0 else None
                dst = Address(rank, st.get("dstbuf", "o"), dstoff) if dstoff >= 0 else None
                if kind == "nop":
                    src = dst = None
                steps.append(NativeStep(kind, src, dst, _int(st, "depid", -1), _int(st, "deps", -1),
                                        bool(_int(st, "hasdep", 0)), _int(st, "cnt", 1)))
            blocks.append(NativeBlock(rank, _int(tb, "id"), _int(tb, "chan", 0), _int(tb, "send", -1),
                                      _int(tb, "recv", -1), tuple(steps)))
    return NativeProgram(root.get("name", "algo"), root.get("coll", "allreduce"), bool(_int(root, "inplace", 0)),
                         ngpus, _int(root, "nchannels", 1), _int(root, "nchunksperloop"), tuple(blocks), ins, outs,
                         scr, root.get("proto", "Simple"), root.get("redop", "nop"), _int(root, "minBytes", 0),
                         _int(root, "maxBytes", 0))


def canonical_xml(text: str) -> str:
    """Attribute-order- and whitespace-independent canonical form (C14N)."""
    root = ET.fromstring(text)
    for el in root.iter():
        el.text = None
        el.tail = None
    return ET.canonicalize(ET.tostring(root, encoding="unicode"), strip_text=True)
