"""Single-GPU timing of the native kernels against the HBM roofline.

    python -m vericcl_b200.ops.kernel_bench --kernel local_reduce --k 4 --elems 67108864 --dtype bfloat16
    python -m vericcl_b200.ops.kernel_bench --kernel fp8_allgather --elems 268435456 --dtype bfloat16
    python -m vericcl_b200.ops.kernel_bench --kernel push_allgather --elems 268435456 --dtype bfloat16

Options: ``--k`` sources of the local reduce, ``--no-scale`` (K = 1 is then a plain
copy), ``--lean`` (the register-lean instance), ``--bulk 1|3`` (TMA-staged loads,
and TMA stores for plain copies), ``--fanout`` (push AllGather fan-out order).

Each run: ``--warmup`` untimed launches, then ``--iters`` launches between two
CUDA events on the current stream; the inputs are larger than the 126 MB L2
at the default sizes, so no flush is needed.  Bytes are the algorithmic HBM
bytes of one launch (every source read once, every destination written
once); the fraction is against the measured copy bandwidth in
MEASURED_PEAKS.json when present (``hbm_gbs``), else 6.65 TB/s.  One JSON
line per run.  This is also the small case for ncu captures of one kernel.
"""
from __future__ import annotations

import argparse
import json
from pathlib import Path

import torch

DTYPES = {"float32": torch.float32, "bfloat16": torch.bfloat16, "float16": torch.float16}


def hbm_peak_gbs() -> tuple:
    path = Path(__file__).resolve().parents[2] / "MEASURED_PEAKS.json"
    try:
        return float(json.loads(path.read_text())["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback"


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="vericcl_b200.ops.kernel_bench")
    ap.add_argument("--kernel", required=True, choices=("local_reduce", "fp8_allgather", "push_allgather"))
    ap.add_argument("--elems", type=int, default=64 << 20)
    ap.add_argument("--k", type=int, default=4, help="sources of the local reduce")
    ap.add_argument("--dtype", default="bfloat16", choices=sorted(DTYPES))
    ap.add_argument("--lanes", type=int, default=0, help="CTAs of the local reduce (0: every SM)")
    ap.add_argument("--bulk", type=int, default=0, choices=(0, 1, 3),
                    help="local reduce: 1 the TMA-staged kernel instance, 3 also TMA stores for plain copies")
    ap.add_argument("--no-scale", action="store_true", help="local reduce: no scale (K=1 is then a plain copy)")
    ap.add_argument("--lean", action="store_true", help="local reduce: the register-lean instance (one-rank default)")
    ap.add_argument("--fanout", action="store_true", help="push AllGather: the fan-out mode")
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--iters", type=int, default=10)
    args = ap.parse_args(argv)
    from vericcl_b200.models import CollectiveEngine
    from vericcl_b200.parallel import Communicator
    dtype = DTYPES[args.dtype]
    esize = torch.tensor([], dtype=dtype).element_size()
    n = args.elems
    heap = 3 * n * esize + (256 << 20)
    comm = Communicator(heap_bytes=heap)
    mod = comm._mod
    stream = torch.cuda.current_stream()
    if args.kernel == "local_reduce":
        srcs = torch.randn(args.k, n, device="cuda").to(dtype)
        dst = torch.empty(n, device="cuda", dtype=dtype)
        lanes = args.lanes or min(148, mod.max_ctas(512))
        keep = []
        scaled = not args.no_scale
        fn = lambda: keep.append(mod.local_reduce(dst, srcs, 0, 0.5 if scaled else 1.0, scaled, lanes, 1,  # noqa: E731
                                                  args.lean, args.bulk))
        nbytes = (args.k + 1) * n * esize
        label = "interp_kernel local reduce K=%d%s%s%s" % (args.k, "" if scaled else " no scale", " lean" if args.lean else "",
                                                         {0: "", 1: " (TMA-staged)", 3: " (TMA loads + stores)"}[args.bulk])
    elif args.kernel == "fp8_allgather":
        eng = CollectiveEngine(comm)
        x = torch.randn(n, device="cuda").to(dtype)
        out = torch.empty(n, device="cuda", dtype=dtype)
        fn = lambda: eng.all_gather_fp8(x, out, fused=True)                                     # noqa: E731
        # one rank: read the input, write e4m3 bytes + scales, write the dequantized output
        nbytes = n * esize + n + 4 * (n // 128) + n * esize
        label = "fp8_allgather_kernel (one rank: quantize, stage, dequantize own part)"
    else:
        ctas = max(1, min(mod.push_allgather_max_ctas(), 148))
        flags = comm.empty(4 * (ctas + 1), torch.float16)
        flags.zero_()
        x = torch.randn(n, device="cuda").to(dtype)
        out = comm.empty(n, dtype)
        fn = lambda: mod.push_allgather(comm.heap, x.data_ptr(), comm.offset_of(out), n * esize,   # noqa: E731
                                        comm.offset_of(flags), ctas, 10.0, args.fanout)
        nbytes = 2 * n * esize
        label = "push_allgather_kernel (one rank: own part copy%s)" % (", fan-out" if args.fanout else "")
    for _ in range(args.warmup):
        fn()
    torch.cuda.synchronize()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for _ in range(args.iters):
        fn()
    t1.record(stream)
    torch.cuda.synchronize()
    comm.check_status()
    us = t0.elapsed_time(t1) / args.iters * 1e3
    peak, source = hbm_peak_gbs()
    gbs = nbytes / (us * 1e-6) / 1e9
    print(json.dumps({"kernel": label, "elems": n, "dtype": args.dtype, "us": round(us, 2), "bytes": nbytes,
                      "gbs": round(gbs, 1), "frac_of_hbm": round(gbs / peak, 3), "hbm_peak": source,
                      "device": torch.cuda.get_device_name()}), flush=True)
    comm.close()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
