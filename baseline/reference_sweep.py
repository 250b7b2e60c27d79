"""Size sweep of the reference's own MSCCL/NCCL 2.12.12 build (the baseline of ``sweep.py``).

    torchrun --nproc-per-node N --master-addr 127.0.0.1 baseline/reference_sweep.py \
             [--colls allreduce,allgather] [--dtype bfloat16] [--min-bytes 1024] [--max-bytes 1073741824]
             [--iters 20] [--warmup 5]

The same points and timing protocol as ``sweep.py``: per size, warm-up calls,
then ``--iters`` calls between two CUDA events on one stream, the mean per
call, the max over ranks.  AllReduce (SUM) runs in place on M bytes per rank;
AllGather out of place, M bytes in and P·M out.  busbw follows nccl-tests
(AllReduce algbw·2(P−1)/P, AllGather algbw·(P−1)/P with size P·M), the
convention of the reference's own baseline protocol (README.md:456-503).
The library is loaded by ``baseline/reference_arm.py`` (no PyTorch, no
vericcl_b200); rank 0 prints one JSON line per point.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import sys

import numpy as np

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
import reference_arm as ra  # noqa: E402

DTYPES = {"bfloat16": (9, 2), "float32": (7, 4), "float16": (6, 2)}


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--colls", default="allreduce,allgather")
    ap.add_argument("--dtype", default="bfloat16", choices=sorted(DTYPES))
    ap.add_argument("--min-bytes", type=int, default=1024)
    ap.add_argument("--max-bytes", type=int, default=1 << 30)
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    args = ap.parse_args()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    reason = ra.unavailable_reason(world)
    if reason is not None:
        if rank == 0:
            print(json.dumps({"impl": "reference", "unavailable": reason}), flush=True)
        return 0
    os.environ.setdefault("NCCL_SOCKET_IFNAME", "lo")
    rt = ra.CudaRT()
    rt.call("cudaSetDevice", local)
    nccl = ra.RefNccl()
    nccl.lib.ncclAllGather.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int,
                                       ctypes.c_void_p, ctypes.c_void_p]
    uid = ra.exchange_unique_id(nccl, rank, world) if world > 1 else nccl.unique_id()
    comm = nccl.init_rank(world, uid, rank)
    stream = rt.stream()
    code, esize = DTYPES[args.dtype]
    send = rt.malloc(args.max_bytes)
    recv = rt.malloc(args.max_bytes * world)
    rt.call("cudaMemsetAsync", ctypes.c_void_p(send), 0, args.max_bytes, ctypes.c_void_p(stream))
    small = rt.malloc(64)

    def all_max(x: float) -> float:
        v = np.array([x], dtype=np.float64)
        rt.call("cudaMemcpy", ctypes.c_void_p(small), v.ctypes.data_as(ctypes.c_void_p), 8, ra.H2D)
        nccl.all_reduce(small, small, 1, ra.NCCL_F64, ra.NCCL_MAX, comm, stream)
        rt.call("cudaStreamSynchronize", ctypes.c_void_p(stream))
        rt.call("cudaMemcpy", v.ctypes.data_as(ctypes.c_void_p), ctypes.c_void_p(small), 8, ra.D2H)
        return float(v[0])

    t0, t1 = rt.event(), rt.event()
    sizes = []
    b = args.min_bytes
    while b <= args.max_bytes:
        sizes.append(b)
        b *= 4
    points = []
    for coll in args.colls.split(","):
        for nbytes in sizes:
            count = nbytes // esize
            if coll == "allreduce":
                call = lambda: nccl.all_reduce(send, send, count, code, ra.NCCL_SUM, comm, stream)
            else:
                call = lambda: nccl.check(nccl.lib.ncclAllGather(send, recv, count, code, comm, stream),
                                          "ncclAllGather")
            for _ in range(args.warmup):
                call()
            all_max(0.0)
            rt.call("cudaEventRecord", ctypes.c_void_p(t0), ctypes.c_void_p(stream))
            for _ in range(args.iters):
                call()
            rt.call("cudaEventRecord", ctypes.c_void_p(t1), ctypes.c_void_p(stream))
            rt.call("cudaEventSynchronize", ctypes.c_void_p(t1))
            us = all_max(rt.elapsed_ms(t0, t1) / args.iters * 1000.0)
            factor = 2.0 * (world - 1) / world if coll == "allreduce" else (world - 1) / world
            size = nbytes if coll == "allreduce" else nbytes * world
            busbw = size / (us * 1e-6) / 1e9 * factor if world > 1 else 0.0
            point = {"impl": "reference", "coll": coll, "bytes_per_rank": nbytes, "dtype": args.dtype,
                     "ranks": world, "us": round(us, 3), "busbw_gbs": round(busbw, 2),
                     "library": "MSCCL/NCCL 2.12.12 (reference build, sm_100)"}
            points.append(point)
            if rank == 0:
                print(json.dumps(point), flush=True)
    if rank == 0:
        print(json.dumps({"impl": "reference", "summary": True, "points": len(points)}), flush=True)
    nccl.lib.ncclCommDestroy(ctypes.c_void_p(comm))
    return 0


if __name__ == "__main__":
    sys.exit(main())
