"""Device-program compilation front end and geometry.

``compile_xml`` runs the native schedule compiler on XML text.  The runtime
buffer of a collective is divided into ``nchunksperloop`` chunks of
``chunk_elems`` elements; every chunk is cut into ``nlanes × niters`` pieces of
``piece_elems`` elements (a multiple of one 16-byte vector), so each CTA moves
whole vectors.  ``run_cpu`` executes a compiled program with the CPU
interpreter (the oracle of the GPU kernel).
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from vericcl_b200.errors import SemanticError
from vericcl_b200.ops import native

DTYPES = {"float32": (0, 4), "bfloat16": (1, 2), "float16": (2, 2)}
REDOPS = {"sum": 0, "avg": 0, "prod": 1, "min": 2, "max": 3}
REDUCING = ("allreduce", "reduce", "reduce_scatter")


@dataclass(frozen=True)
class Geometry:
    count_per_rank: int     # input elements per rank
    runtime_elems: int      # elements of the collective's runtime buffer
    chunk_elems: int
    piece_elems: int
    nlanes: int
    niters: int
    elem_bytes: int


def geometry(collective: str, ranks: int, nchunks: int, count_per_rank: int, elem_bytes: int, nlanes: int,
             niters: int) -> Geometry:
    runtime = count_per_rank * (ranks if collective in ("allgather", "gather") else 1)
    if runtime % nchunks:
        raise SemanticError("%d elements do not split into %d chunks" % (runtime, nchunks))
    chunk = runtime // nchunks
    vec = 16 // elem_bytes
    if chunk % vec:
        raise SemanticError("chunk of %d elements is not a whole number of 16-byte vectors" % chunk)
    pieces = nlanes * niters
    piece = -(-chunk // pieces)
    piece = -(-piece // vec) * vec
    return Geometry(count_per_rank, runtime, chunk, piece, nlanes, niters, elem_bytes)


def compile_xml(xml: str, *, nlanes: int = 1, niters: int = 1, elide: bool = True, fuse: bool = True,
                multicast: bool = False, collective: str | None = None, merge: bool = True, push: bool = False):
    mod = native.plan()
    if collective is None:
        import re
        found = re.search(r'coll="([a-z_]+)"', xml)
        collective = found.group(1) if found else "allreduce"
    try:
        return mod.parse_and_compile(xml, nlanes, niters, elide, fuse, multicast, collective in REDUCING, merge,
                                     push)
    except mod.CompileError as error:
        raise SemanticError(str(error)) from error


def _to_storage(array: np.ndarray, dtype: str) -> np.ndarray:
    if dtype == "float32":
        return np.ascontiguousarray(array, dtype=np.float32)
    if dtype == "float16":
        return np.ascontiguousarray(array, dtype=np.float16)
    import torch
    return torch.from_numpy(np.ascontiguousarray(array, dtype=np.float32)).to(torch.bfloat16).view(
        torch.int16).numpy().copy()


def _from_storage(array: np.ndarray, dtype: str) -> np.ndarray:
    if dtype == "bfloat16":
        import torch
        return torch.from_numpy(array.copy()).view(torch.bfloat16).to(torch.float32).numpy()
    return array.astype(np.float64 if dtype == "float64" else np.float32)


def run_cpu(compiled, inputs, *, dtype: str = "float32", op: str = "sum", scale: float = 1.0, seed: int = 0,
            launches: int = 1, outputs=None):
    """Run ``compiled`` on per-rank input arrays; return per-rank output arrays (fp32)."""
    code, esize = DTYPES[dtype]
    p = compiled.ranks
    count = len(inputs[0])
    geo = geometry(compiled.collective, p, compiled.nchunks, count, esize, compiled.nlanes, compiled.niters)
    ins, outs, scrs = [], [], []
    for r in range(p):
        i_chunks, o_chunks, s_chunks = compiled.slots(r)
        data = _to_storage(np.asarray(inputs[r]), dtype)
        buf = np.zeros(max(i_chunks * geo.chunk_elems, 1), dtype=data.dtype)
        buf[:len(data)] = data[:len(buf)]
        ins.append(buf)
        out = np.zeros(max(o_chunks * geo.chunk_elems, 1), dtype=data.dtype)
        if outputs is not None:
            init = _to_storage(np.asarray(outputs[r]), dtype)
            out[:len(init)] = init
        outs.append(out)
        scrs.append(np.zeros(max(s_chunks * geo.chunk_elems, 1), dtype=data.dtype))
    if compiled.inplace:
        # in-place programs address the output buffer; seed it with the input where it aliases
        for r in range(p):
            if compiled.collective == "allgather":
                outs[r][r * count:(r + 1) * count] = ins[r][:count]
            elif compiled.collective == "reduce_scatter":
                pass
            else:
                outs[r][:count] = ins[r][:count]
    ok, error, _ = native.plan().cpu_interpret(compiled, ins, outs, scrs, code, REDOPS[op], float(scale),
                                               geo.chunk_elems, geo.piece_elems, seed, launches)
    if not ok:
        raise SemanticError("CPU interpreter: " + error)
    if compiled.inplace and compiled.collective == "reduce_scatter":
        part = len(ins[0]) // p
        return [_from_storage(ins[r][r * part:(r + 1) * part], dtype) for r in range(p)]
    return [_from_storage(o, dtype) for o in outs]
