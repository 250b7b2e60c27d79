"""Multi-GPU correctness worker (launched by torchrun, one process per GPU).

For every case: synthesize the schedule, compile it for this rank, run it
through the sm_100a interpreter on heap buffers filled with seeded data, and
compare with an fp64 host reference computed from every rank's (regenerated)
inputs.  Prints one JSON line per case on rank 0 and exits non-zero on any
mismatch.  Used by tests/test_gpu_multi.py.
"""
import json
import os
import sys
import zlib

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from vericcl_b200.parallel import Communicator  # noqa: E402
from vericcl_b200.synthesis import schedule_xml  # noqa: E402

TOL = {torch.float32: 1e-4, torch.bfloat16: 3e-2, torch.float16: 5e-3}


def inputs_for(rank, count, dtype, seed):
    g = torch.Generator().manual_seed(seed * 1000 + rank)
    return torch.randn(count, generator=g, dtype=torch.float64).to(dtype)


def reference(coll, world, count, dtype, seed, op, rank):
    xs = [inputs_for(r, count, dtype, seed).double() for r in range(world)]
    if coll == "allreduce":
        if op == "max":
            return torch.stack(xs).max(dim=0).values
        if op == "min":
            return torch.stack(xs).min(dim=0).values
        total = sum(xs)
        if op == "avg":
            total = total / world
        return total
    if coll == "allgather":
        return torch.cat(xs)
    if coll == "reduce_scatter":
        total = sum(xs)
        part = count // world
        return total[rank * part:(rank + 1) * part]
    raise ValueError(coll)


def main():
    dist.init_process_group("cpu:gloo,cuda:nccl", device_id=torch.device("cuda", int(os.environ["LOCAL_RANK"])))
    rank, world = dist.get_rank(), dist.get_world_size()
    torch.cuda.set_device(int(os.environ["LOCAL_RANK"]))
    quick = os.environ.get("VB_QUICK") == "1"
    comm = Communicator(heap_bytes=1 << 30, multicast=os.environ.get("VERICCL_NVLS", "0") == "1", timeout_s=5.0)
    failures = 0
    cases = []
    if rank == 0:
        print(json.dumps({"multicast": comm.multicast, "world": world}), flush=True)
    for coll in ("allreduce", "allgather", "reduce_scatter"):
        for dtype in (torch.float32, torch.bfloat16):
            for inplace in (False, True):
                for slices in ((1, world) if coll != "reduce_scatter" else (world,)):
                    for lanes, iters in ((1, 1), (4, 2), (16, 1)):
                        for count in ((world * 4096, world * 1 << 18) if not quick else (world * 4096,)):
                            cases.append((coll, dtype, inplace, slices, lanes, iters, count, False))
    # push steps (stores into the receiver's heap buffer) on the plain-transfer collectives, no NVLS
    for coll in ("allgather", "allreduce"):
        for inplace in (False, True):
            for lanes, iters in ((1, 1), (8, 2)):
                cases.append((coll, torch.float32, inplace, world if coll == "allreduce" else 1, lanes, iters,
                              world * 4096, True))
    for coll, dtype, inplace, slices, lanes, iters, count, push in cases:
        dname = str(dtype).split(".")[-1]
        xml = schedule_xml(coll, world, slices, inplace=inplace, datatype=dname)
        op = "avg" if coll == "allreduce" and lanes == 4 else "sum"
        # VERICCL_MERGE=0: every XML thread block on CTAs of its own (the unmerged device program)
        plan = comm.compile(xml, nlanes=lanes, niters=iters, push=push, merge=os.environ.get("VERICCL_MERGE") != "0",
                            multicast=comm.multicast and not push and coll in ("allreduce", "allgather"))
        seed = zlib.crc32(repr((coll, dname, inplace, slices, lanes, iters, count)).encode()) % 100000
        x = inputs_for(rank, count, dtype, seed).cuda()
        out_n = count * world if coll == "allgather" else count // world if coll == "reduce_scatter" else count
        if inplace:
            buf = comm.empty(max(count, out_n), dtype)
            if coll == "allgather":
                buf[rank * count:(rank + 1) * count].copy_(x)
                inp, out = buf[rank * count:(rank + 1) * count], buf
            elif coll == "reduce_scatter":
                buf[:count].copy_(x)
                inp, out = buf[:count], buf[rank * out_n:(rank + 1) * out_n]
            else:
                buf.copy_(x)
                inp, out = buf, buf
        else:
            inp = comm.empty(count, dtype)
            out = comm.empty(out_n, dtype)
            inp.copy_(x)
            out.fill_(float("nan"))
        torch.cuda.synchronize()
        dist.barrier()
        if inplace:
            # in-place programs address one buffer for both roles
            comm.run(plan, buf, buf, op=op, count_per_rank=count)
        else:
            comm.run(plan, inp, out, op=op, count_per_rank=count)
        torch.cuda.synchronize()
        comm.check_status()
        ref = reference(coll, world, count, dtype, seed, op, rank)
        if inplace and coll == "reduce_scatter":
            got = buf[rank * out_n:(rank + 1) * out_n]
        else:
            got = out if not inplace or coll != "allreduce" else buf
        got = got.double().cpu()
        err = (got - ref).abs().max().item() if got.numel() else 0.0
        scale = max(1.0, ref.abs().max().item())
        ok = err <= TOL[dtype] * scale * (world if coll != "allgather" else 1) and torch.isfinite(got).all().item()
        if not ok:
            failures += 1
        if rank == 0 or not ok:
            print(json.dumps({"rank": rank, "coll": coll, "dtype": dname, "inplace": inplace, "slices": slices,
                              "lanes": lanes, "iters": iters, "count": count, "op": op, "push": push,
                              "max_err": err, "ok": ok}), flush=True)
        dist.barrier()
        for t in ([buf] if inplace else [inp, out]):
            comm.free(t)
    # one-shot flag-in-data path: every case three times in a row (both LL region halves are reused), AllReduce and
    # AllGather interleaved so they share the launch counter
    from vericcl_b200.models import CollectiveEngine
    from vericcl_b200.models.collectives import ONESHOT_MAX_BYTES
    # an explicit threshold routes to the one-shot kernel at any world size, so it is checked wherever this runs
    eng = CollectiveEngine(comm, oneshot_max_bytes=ONESHOT_MAX_BYTES)
    oneshot = []
    for dtype in (torch.float32, torch.bfloat16, torch.float16):
        esize = torch.tensor([], dtype=dtype).element_size()
        for nbytes in (8, 1024, 65536, eng.oneshot_max_bytes):
            count = nbytes // esize
            for op in ("sum", "avg", "max"):
                oneshot.append(("allreduce", dtype, op, count, op == "avg"))
            oneshot.append(("allgather", dtype, "sum", count, False))
    for coll, dtype, op, count, inplace in oneshot:
        dname = str(dtype).split(".")[-1]
        plan = eng.plan(coll, count, dtype, inplace=inplace, op=op)
        assert plan.kind == "oneshot", plan
        seed = zlib.crc32(repr(("oneshot", coll, dname, op, count)).encode()) % 100000
        x = inputs_for(rank, count, dtype, seed).cuda()
        out_n = count * world if coll == "allgather" else count
        inp = comm.empty(count, dtype)
        out = inp if inplace else comm.empty(out_n, dtype)
        ref = reference(coll, world, count, dtype, seed, op, rank)
        worst, ok = 0.0, True
        for rep in range(3):
            inp.copy_(x)
            if not inplace:
                out.fill_(float("nan"))
            torch.cuda.synchronize()
            comm.run(plan, inp, out, op=op)
            torch.cuda.synchronize()
            comm.check_status()
            got = out.double().cpu()
            err = (got - ref).abs().max().item()
            worst = max(worst, err)
            scale = max(1.0, ref.abs().max().item())
            ok = ok and err <= TOL[dtype] * scale * (world if coll != "allgather" else 1) and \
                torch.isfinite(got).all().item()
        if not ok:
            failures += 1
        if rank == 0 or not ok:
            print(json.dumps({"rank": rank, "coll": coll, "path": "oneshot", "dtype": dname, "op": op,
                              "count": count, "inplace": inplace, "max_err": worst, "ok": ok}), flush=True)
        comm.free(inp)
        if not inplace:
            comm.free(out)
    cases += oneshot
    # two-shot AllReduce (opt-in path): run only when asked
    if os.environ.get("VB_TWOSHOT") == "1":
        two = CollectiveEngine(comm, twoshot_max_bytes=4 << 20)
        twoshot = []
        for dtype in (torch.float32, torch.bfloat16):
            esize = torch.tensor([], dtype=dtype).element_size()
            for nbytes in (2 << 20, 4 << 20):
                for op in ("sum", "avg"):
                    twoshot.append((dtype, nbytes // esize, op))
        for dtype, count, op in twoshot:
            dname = str(dtype).split(".")[-1]
            plan = two.plan("allreduce", count, dtype, inplace=True, op=op)
            assert plan.collective == "allreduce_twoshot", plan
            seed = zlib.crc32(repr(("twoshot", dname, op, count)).encode()) % 100000
            x = inputs_for(rank, count, dtype, seed).cuda()
            buf = comm.empty(count, dtype)
            ref = reference("allreduce", world, count, dtype, seed, op, rank)
            worst, ok = 0.0, True
            for rep in range(3):
                buf.copy_(x)
                torch.cuda.synchronize()
                comm.run(plan, buf, buf, op=op)
                torch.cuda.synchronize()
                comm.check_status()
                err = (buf.double().cpu() - ref).abs().max().item()
                worst = max(worst, err)
                ok = ok and err <= TOL[dtype] * max(1.0, ref.abs().max().item()) * world
            failures += 0 if ok else 1
            if rank == 0 or not ok:
                print(json.dumps({"rank": rank, "coll": "allreduce", "path": "twoshot", "dtype": dname, "op": op,
                                  "count": count, "max_err": worst, "ok": ok}), flush=True)
            comm.free(buf)
        cases += twoshot
    # broadcast / reduce (non-zero roots) and all-to-all through the engine, on non-heap tensors
    extra = [("broadcast", world - 1), ("reduce", world - 1), ("reduce", 0), ("alltoall", 0)]
    for coll, root in extra:
        n = world * 8192
        seed = zlib.crc32(repr(("engine", coll, root)).encode()) % 100000
        x = inputs_for(rank, n, torch.float32, seed).cuda()
        out = torch.full((n,), float("nan"), device="cuda")
        if coll == "broadcast":
            eng.broadcast(x, out, root=root)
        elif coll == "reduce":
            eng.reduce(x, out, root=root)
        else:
            eng.all_to_all(x, out)
        torch.cuda.synchronize()
        comm.check_status()
        xs = [inputs_for(r, n, torch.float32, seed).double() for r in range(world)]
        if coll == "broadcast":
            ref = xs[root]
        elif coll == "reduce":
            ref = sum(xs) if rank == root else None
        else:
            part = n // world
            ref = torch.cat([xs[s][rank * part:(rank + 1) * part] for s in range(world)])
        if ref is None:
            ok, err = True, 0.0                              # non-root output is unspecified
        else:
            err = (out.double().cpu() - ref).abs().max().item()
            ok = err <= 1e-4 * world * max(1.0, ref.abs().max().item())
        failures += 0 if ok else 1
        if rank == 0 or not ok:
            print(json.dumps({"rank": rank, "coll": coll, "root": root, "path": "engine", "max_err": err, "ok": ok}),
                  flush=True)
    cases += extra
    # push AllGather (every rank stores into every peer's heap output), three calls in a row per size
    push_eng = CollectiveEngine(comm)
    push_eng.ag_push_min_bytes = 0
    for dt, n, fanout in ((torch.float32, 1 << 16, False), (torch.bfloat16, (1 << 16) + 8, False),
                          (torch.float16, 24, False), (torch.float32, 1 << 16, True), (torch.bfloat16, 4104, True)):
        push_eng.ag_push_fanout = fanout
        x = inputs_for(rank, n, dt, 777).cuda()
        ref = torch.cat([inputs_for(r, n, dt, 777) for r in range(world)]).cuda()
        out = comm.empty(n * world, dt)
        for call in range(3):
            out.fill_(float("nan"))
            torch.cuda.synchronize()
            comm.barrier()
            push_eng.all_gather(x, out)
            torch.cuda.synchronize()
            comm.check_status()
            ok = bool(torch.equal(out, ref))
            failures += 0 if ok else 1
            if rank == 0 or not ok:
                print(json.dumps({"rank": rank, "coll": "allgather", "path": "push", "dtype": str(dt), "n": n,
                                  "fanout": fanout, "call": call, "ok": ok}), flush=True)
        comm.free(out)
    # block-scaled FP8 AllGather through the engine: the fused kernel (three calls in a row, so both staging
    # parities are reused) against the three-pass path and against the fp64 inputs
    for dt, n in ((torch.float32, 1 << 14), (torch.bfloat16, (1 << 14) + 48), (torch.float16, 4096)):
        x = inputs_for(rank, n, dt, 4242).cuda()
        ref = torch.cat([inputs_for(r, n, dt, 4242) for r in range(world)]).cuda().float()
        slow = torch.empty(n * world, device="cuda", dtype=dt)
        eng.all_gather_fp8(x, slow, fused=False)
        for call in range(3):
            out = torch.full((n * world,), float("nan"), device="cuda", dtype=dt)
            eng.all_gather_fp8(x, out, fused=True)
            torch.cuda.synchronize()
            comm.check_status()
            amax = torch.nn.functional.pad(ref.view(world, n), (0, (-n) % 128)).view(-1, 128).abs().amax(dim=1)
            amax = amax.repeat_interleave(128).view(world, -1)[:, :n].reshape(-1)
            rel = ((out.float() - ref).abs() / amax.clamp_min(1e-6)).max().item()
            same = (out.float() - slow.float()).abs().max().item() <= 1e-2 * float(amax.max()) / 448
            ok = rel < 0.07 and same and not torch.isnan(out.float()).any().item()
            failures += 0 if ok else 1
            if rank == 0 or not ok:
                print(json.dumps({"rank": rank, "coll": "allgather_fp8", "dtype": str(dt), "n": n, "call": call,
                                  "path": "fused", "max_rel_err": rel, "matches_three_pass": same, "ok": ok}),
                      flush=True)
    total = torch.tensor([failures])
    dist.all_reduce(total, group=comm.control_group)
    comm.close()
    dist.destroy_process_group()
    if rank == 0:
        print(json.dumps({"summary": True, "cases": len(cases), "failures": int(total.item())}), flush=True)
    sys.exit(1 if total.item() else 0)


if __name__ == "__main__":
    main()
