"""Single-process NVLink probe: pull / push / local copy bandwidth between two GPUs.

Runs the calibration copy kernel (``csrc/cuda/probes.cu``) on GPU 0 reading
from GPU 1 (pull), writing to GPU 1 (push), and copying locally, with peer
access enabled, and reports device-timed bandwidths.  It launches no
cross-GPU waits, so it can also be profiled with Nsight Compute.

    python -m vericcl_b200.online.nvlink_probe --bytes 268435456 --ctas 148 --reps 3
"""
from __future__ import annotations

import argparse
import json


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--bytes", type=int, default=1 << 28)
    ap.add_argument("--ctas", type=int, default=148)
    ap.add_argument("--threads", type=int, default=512)
    ap.add_argument("--unroll", type=int, default=4)
    ap.add_argument("--reps", type=int, default=5)
    ap.add_argument("--modes", default="pull,push,local")
    args = ap.parse_args(argv)
    import torch
    from vericcl_b200.ops import native
    m = native.cuda()
    if torch.cuda.device_count() < 2:
        raise SystemExit("needs two GPUs")
    m.enable_peer_access(0, 1)
    m.enable_peer_access(1, 0)
    n = args.bytes
    a0 = torch.empty(n, dtype=torch.uint8, device="cuda:0")
    b0 = torch.empty(n, dtype=torch.uint8, device="cuda:0")
    a1 = torch.empty(n, dtype=torch.uint8, device="cuda:1")
    plans = {"pull": (b0, a1, 1), "push": (a1, b0, 1), "local": (b0, a0, 2)}
    out = {}
    torch.cuda.set_device(0)
    for mode in args.modes.split(","):
        dst, src, factor = plans[mode]
        m.copy_probe(dst.data_ptr(), src.data_ptr(), n, args.ctas, args.threads, args.unroll)
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(args.reps):
            m.copy_probe(dst.data_ptr(), src.data_ptr(), n, args.ctas, args.threads, args.unroll)
        e.record()
        torch.cuda.synchronize()
        ms = s.elapsed_time(e) / args.reps
        out[mode + "_gbs"] = round(factor * n / (ms * 1e-3) / 1e9, 2)
    out.update({"bytes": n, "ctas": args.ctas, "threads": args.threads, "unroll": args.unroll})
    print(json.dumps(out))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
