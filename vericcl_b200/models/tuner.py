"""Measured engine thresholds for this machine and rank count.

    torchrun --nproc-per-node P --master-addr 127.0.0.1 -m vericcl_b200.models.tuner --out tuning.json

The engine picks a path per collective and size: the one-shot flag-in-data
kernel, the opt-in two-shot kernel, or the synthesized schedule on the
interpreter (with NVLS multicast or peer pulls for AllGather).  Its default
size thresholds were measured on B200s of one pool; this tuner measures the
candidates on the GPUs it runs on (device time, back-to-back launches, max
over ranks) over sizes 64 KiB … 64 MiB per rank in powers of 2 and derives:

* ``oneshot_max_bytes`` — the largest size up to which the one-shot path is
  the fastest at every size (AllReduce and AllGather together);
* ``twoshot_max_bytes`` — the largest size above that up to which the
  two-shot AllReduce beats the interpreter at every size (0: never);
* ``ag_nvls_max_bytes`` — the smallest size from which peer pulls beat NVLS
  multicast for AllGather (kept at the default without NVLS);
* ``bulk_windows`` — per collective kind (``allgather``, ``other``), the
  longest run of consecutive sizes at which the TMA-staged instance beat the
  vector path by at least 1 % on pull plans (``[first, last]`` bytes per
  rank, or absent), which then replaces the built-in windows.

The result is a small JSON table keyed by rank count, GPU name and driver;
``CollectiveEngine(tuning=load_tuning(path, comm))`` applies it.
"""
from __future__ import annotations

import argparse
import json
import os
import sys
from pathlib import Path

DEFAULT_SIZES = tuple(1 << k for k in range(16, 27))      # 64 KiB … 64 MiB per rank
ONESHOT_PROBE_MAX = 8 << 20     # the flag-in-data paths double the bytes on the wire: no point probing beyond
TWOSHOT_PROBE_MAX = 32 << 20


def derive_thresholds(times: dict, *, default_ag_nvls: int) -> dict:
    """Thresholds from ``times[(collective, path)][size] = µs``.

    Paths: ("allreduce"|"allgather", "oneshot"), ("allreduce", "twoshot"),
    ("allreduce"|"allgather", "interp"), ("allgather", "interp_p2p").
    Missing entries count as unavailable.
    """
    def t(coll, path, size):
        return times.get((coll, path), {}).get(size)

    sizes = sorted({s for series in times.values() for s in series})
    oneshot = 0
    for size in sizes:
        wins = []
        for coll in ("allreduce", "allgather"):
            mine, other = t(coll, "oneshot", size), t(coll, "interp", size)
            if mine is not None and other is not None:
                wins.append(mine < other)
        if wins and all(wins):
            oneshot = size
        else:
            break
    twoshot = 0
    for size in sizes:
        if size <= oneshot:
            continue
        mine, other = t("allreduce", "twoshot", size), t("allreduce", "interp", size)
        if mine is not None and other is not None and mine < other:
            twoshot = size
        else:
            break
    ag_nvls = default_ag_nvls
    if times.get(("allgather", "interp_p2p")):
        ag_nvls = max(sizes) * 2 if sizes else default_ag_nvls
        for size in sizes:
            pull, mc = t("allgather", "interp_p2p", size), t("allgather", "interp", size)
            if pull is not None and mc is not None and pull < mc:
                ag_nvls = size
                break
    table = {"oneshot_max_bytes": oneshot, "twoshot_max_bytes": twoshot, "ag_nvls_max_bytes": ag_nvls}
    windows = {}
    for kind, coll in (("allgather", "allgather"), ("other", "allreduce")):
        if times.get((coll, "pull_vector")) and times.get((coll, "pull_staged")):
            window = staged_window(times[(coll, "pull_vector")], times[(coll, "pull_staged")])
            if window is not None:
                windows[kind] = window
    if any((c, "pull_staged") in times for c in ("allgather", "allreduce")):
        table["bulk_windows"] = windows
    return table


def staged_window(vector: dict, staged: dict, *, margin: float = 0.01):
    """``[first, last]``: the longest run of consecutive measured sizes at which the staged time is at least
    ``margin`` below the vector time (None when there is none)."""
    sizes = sorted(set(vector) & set(staged))
    best, run = None, []
    for size in sizes:
        if staged[size] < vector[size] * (1.0 - margin):
            run.append(size)
            if best is None or len(run) > len(best):
                best = list(run)
        else:
            run = []
    return None if not best else [best[0], best[-1]]


def machine_key(world: int) -> str:
    try:
        import torch
        name = torch.cuda.get_device_name(0) if torch.cuda.is_available() else "cpu"
    except Exception:
        name = "unknown"
    driver = ""
    try:
        import pynvml
        pynvml.nvmlInit()
        try:
            drv = pynvml.nvmlSystemGetDriverVersion()
            driver = drv.decode() if isinstance(drv, bytes) else drv
        finally:
            pynvml.nvmlShutdown()
    except Exception:
        pass
    return "%d|%s|%s" % (world, name, driver)


def save_tuning(path, key: str, table: dict) -> None:
    from vericcl_b200.utils.jsonio import atomic_write_json
    path = Path(path)
    data = json.loads(path.read_text()) if path.exists() else {}
    data[key] = table
    atomic_write_json(path, data)


def load_tuning(path, comm) -> dict | None:
    """The table measured for this rank count and machine, or None."""
    path = Path(path)
    if not path.exists():
        return None
    return json.loads(path.read_text()).get(machine_key(comm.world))


def measure_paths(comm, sizes=DEFAULT_SIZES, *, iters: int = 20, warmup: int = 5, dtype=None) -> dict:
    """Device time (µs, max over ranks) of every candidate path at every size."""
    import torch
    from vericcl_b200.models.collectives import CollectiveEngine
    dtype = dtype or torch.bfloat16
    esize = torch.tensor([], dtype=dtype).element_size()
    world = comm.world
    stream = torch.cuda.current_stream()
    big = max(sizes)
    engines = {
        "oneshot": CollectiveEngine(comm, oneshot_max_bytes=min(big, ONESHOT_PROBE_MAX), twoshot_max_bytes=0),
        "twoshot": CollectiveEngine(comm, oneshot_max_bytes=0, twoshot_max_bytes=min(big, TWOSHOT_PROBE_MAX)),
        "interp": CollectiveEngine(comm, oneshot_max_bytes=0, twoshot_max_bytes=0, ag_nvls_max_bytes=2 * big),
        "interp_p2p": CollectiveEngine(comm, oneshot_max_bytes=0, twoshot_max_bytes=0, ag_nvls_max_bytes=0),
    }
    out = {}

    def timed(fn):
        for _ in range(warmup):
            fn()
        torch.cuda.synchronize()
        comm.barrier()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record(stream)
        for _ in range(iters):
            fn()
        e.record(stream)
        torch.cuda.synchronize()
        t = torch.tensor([s.elapsed_time(e) / iters * 1e3], dtype=torch.float64)
        if world > 1:
            import torch.distributed as dist
            dist.all_reduce(t, op=dist.ReduceOp.MAX, group=comm.control_group)
        return float(t.item())

    vector_or_staged = {"pull_vector": 0, "pull_staged": 1}
    for size in sizes:
        count = size // esize
        buf = comm.empty(count, dtype)
        inp = comm.empty(count, dtype)
        gout = comm.empty(count * world, dtype)
        buf.normal_()
        inp.normal_()
        for name, eng in engines.items():
            for coll in ("allreduce", "allgather"):
                if (coll, name) in (("allgather", "twoshot"), ("allreduce", "interp_p2p")):
                    continue
                if name == "twoshot" and (world < 2 or size % (8 * world) or size > TWOSHOT_PROBE_MAX):
                    continue
                if name == "oneshot" and (world < 2 or size > ONESHOT_PROBE_MAX):
                    continue
                plan = eng.plan(coll, count, dtype, inplace=coll == "allreduce")
                if coll == "allreduce":
                    fn = (lambda p=plan: comm.run(p, buf, buf))
                else:
                    fn = (lambda p=plan: comm.run(p, inp, gout))
                out.setdefault((coll, name), {})[size] = timed(fn)
                comm.check_status()
        # the staged instance against the vector path on pull plans (AllGather pulls; AllReduce without NVLS)
        for coll, eng in (("allgather", engines["interp_p2p"]), ("allreduce", engines["interp"])):
            plan = eng.plan(coll, count, dtype, inplace=coll == "allreduce")
            if world < 2 or plan.kind == "oneshot" or plan.multicast:
                continue
            saved = comm.bulk
            try:
                for label, mode in vector_or_staged.items():
                    comm.bulk = mode
                    if coll == "allreduce":
                        fn = (lambda p=plan: comm.run(p, buf, buf))
                    else:
                        fn = (lambda p=plan: comm.run(p, inp, gout))
                    out.setdefault((coll, label), {})[size] = timed(fn)
                    comm.check_status()
            finally:
                comm.bulk = saved
        for t in (buf, inp, gout):
            comm.free(t)
    return out


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="vericcl_b200.models.tuner")
    ap.add_argument("--out", required=True)
    ap.add_argument("--min-bytes", type=int, default=1 << 16)
    ap.add_argument("--max-bytes", type=int, default=1 << 26)
    args = ap.parse_args(argv)
    import torch
    import torch.distributed as dist
    from vericcl_b200.models.collectives import AG_NVLS_MAX_BYTES
    from vericcl_b200.parallel import Communicator
    local = int(os.environ.get("LOCAL_RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("cpu:gloo,cuda:nccl", device_id=torch.device("cuda", local))
    sizes = []
    s = args.min_bytes
    while s <= args.max_bytes:
        sizes.append(s)
        s *= 2
    # buffers of the largest size plus the flag-in-data regions of both probe limits
    comm = Communicator(heap_bytes=args.max_bytes * (world + 3) + (1 << 30), multicast=world >= 4)
    times = measure_paths(comm, sizes)
    table = derive_thresholds(times, default_ag_nvls=AG_NVLS_MAX_BYTES)
    if comm.rank == 0:
        key = machine_key(world)
        save_tuning(args.out, key, dict(table, measured={"%s/%s" % k: v for k, v in times.items()}))
        print(json.dumps({"key": key, **table}))
    comm.close()
    if world > 1:
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
