"""User-facing collectives bound to a :class:`Communicator`.

``CollectiveEngine`` synthesizes a verified schedule once per (collective,
rank count, slice count, layout, dtype), compiles it for this rank, picks a
launch geometry for the message size (lanes × pipeline iterations over the
co-resident CTA budget), and runs it with the sm_100a interpreter.  Payloads
of at most ``oneshot_max_bytes`` per rank (AllReduce, AllGather) run the
one-shot flag-in-data kernel instead, whose latency is one NVLink trip.  Buffers in
the communicator's heap run zero-copy; other tensors are staged through heap
buffers (a local device copy on each side).
"""
from __future__ import annotations

import os

import torch

from vericcl_b200.errors import RuntimeFailure
from vericcl_b200.synthesis import schedule_xml

ONESHOT_MAX_BYTES = 1 << 20          # per-rank payloads up to this size take the one-shot flag-in-data path
# world sizes whose one-shot / two-shot runs have passed the multi-GPU fp64 checks on B200s; other sizes take the
# interpreter unless VERICCL_ONESHOT_ANY_WORLD=1 (or an explicit threshold) says otherwise
ONESHOT_VERIFIED_WORLDS = frozenset({2, 4, 8})
AG_NVLS_MAX_BYTES = 8 << 20          # larger AllGathers pull from peers (measured faster than multicast stores)
PIECE_MIN_BYTES = 8 * 1024          # smallest useful piece per CTA per iteration
PIECE_TARGET_BYTES = 512 * 1024     # pipeline a lane's work in pieces of about this size
MAX_ITERS = 8


def _pitched(tensor: torch.Tensor) -> bool:
    """A 2D CUDA view with contiguous rows and a larger row pitch (a column slice of a matrix, for example)."""
    return (tensor.is_cuda and tensor.dim() == 2 and tensor.size(0) > 1 and tensor.stride(1) == 1
            and tensor.stride(0) >= tensor.size(1))


class CollectiveEngine:
    def __init__(self, comm, *, method: str = "hierarchy", slices_per_rank: int | None = None,
                 max_lanes: int | None = None, oneshot_max_bytes: int | None = None,
                 twoshot_max_bytes: int | None = None, ag_nvls_max_bytes: int | None = None,
                 tuning: dict | None = None, cta_budget: int | None = None):
        self.comm = comm
        # interpreter CTAs per GPU this engine may launch (None: every co-resident CTA); the rest of the
        # SMs stay free for compute that overlaps the collective (a data-parallel backward pass)
        self.cta_budget = cta_budget
        self.method = method
        self.slices_per_rank = slices_per_rank
        explicit = {"oneshot_max_bytes": oneshot_max_bytes, "twoshot_max_bytes": twoshot_max_bytes,
                    "ag_nvls_max_bytes": ag_nvls_max_bytes}
        # an explicit threshold (argument or environment) is the caller's choice at any world size
        self._explicit_oneshot = (oneshot_max_bytes is not None or twoshot_max_bytes is not None or
                                  "VERICCL_ONESHOT_MAX" in os.environ or "VERICCL_TWOSHOT_MAX" in os.environ)
        if oneshot_max_bytes is None:
            oneshot_max_bytes = int(os.environ.get("VERICCL_ONESHOT_MAX", ONESHOT_MAX_BYTES))
        self.oneshot_max_bytes = oneshot_max_bytes
        if twoshot_max_bytes is None:
            twoshot_max_bytes = int(os.environ.get("VERICCL_TWOSHOT_MAX", 0))
        self.twoshot_max_bytes = twoshot_max_bytes
        self.ag_nvls_max_bytes = AG_NVLS_MAX_BYTES if ag_nvls_max_bytes is None else ag_nvls_max_bytes
        self.ag_push_min_bytes = None      # push AllGather threshold (None: off); VERICCL_AG_PUSH_MIN overrides
        self.ag_push_fanout = False        # push kernel stores each loaded vector to every rank; VERICCL_AG_PUSH_FANOUT
        self.push_collectives = frozenset()   # interpreter collectives compiled with push steps
        if tuning is not None:
            # thresholds measured on this machine (vericcl_b200.models.tuner); explicit arguments still win
            for name, given in explicit.items():
                if given is None and name in tuning:
                    setattr(self, name, int(tuning[name]))
            self._explicit_oneshot |= "oneshot_max_bytes" in tuning or "twoshot_max_bytes" in tuning
            if "bulk_windows" in tuning and getattr(comm, "bulk", None) is None:
                # the staged instance's measured windows on this machine replace the built-in ones
                comm.bulk_windows = {k: tuple(v) for k, v in tuning["bulk_windows"].items()}
        self._max_ctas = comm._mod.max_ctas(512)
        self.max_lanes = max_lanes or self._max_ctas
        self._staging: dict = {}

    # -- geometry ---------------------------------------------------------------
    def geometry(self, plan_blocks: int, chunk_bytes: int):
        cap = self._max_ctas if self.cta_budget is None else max(1, min(self._max_ctas, self.cta_budget))
        lanes = max(1, min(self.max_lanes, 256, cap // max(1, plan_blocks)))
        lanes = max(1, min(lanes, chunk_bytes // PIECE_MIN_BYTES))
        iters = max(1, min(MAX_ITERS, chunk_bytes // (lanes * PIECE_TARGET_BYTES)))
        if os.environ.get("VERICCL_LANES"):
            lanes = int(os.environ["VERICCL_LANES"])
        if os.environ.get("VERICCL_ITERS"):
            iters = int(os.environ["VERICCL_ITERS"])
        return lanes, iters

    def use_multicast(self, collective: str, op: str, nbytes: int = 0) -> bool:
        """NVLS pays off from 4 ranks up (it cuts AllReduce NVLink traffic from 2(P-1)/P·M to about (1+1/P)·M).

        AllGather moves (P-1)·M into every GPU either way; from ``ag_nvls_max_bytes``
        per rank (default ``AG_NVLS_MAX_BYTES``), peer pulls in rotated order (rank r
        reads r+1, r+2, … first) were faster than owner multicast stores on 4 B200s
        (16 MiB: 117 vs 132 µs; 64 MiB: 364 vs 423 µs), so large AllGathers use them.
        """
        if not self.comm.multicast or self.comm.world < 4:
            return False
        if collective == "allreduce":
            return op in ("sum", "avg")
        limit = int(os.environ.get("VERICCL_AG_NVLS_MAX", self.ag_nvls_max_bytes))
        return collective == "allgather" and nbytes < limit

    def _oneshot_world_ok(self) -> bool:
        return (self.comm.world in ONESHOT_VERIFIED_WORLDS or self._explicit_oneshot
                or os.environ.get("VERICCL_ONESHOT_ANY_WORLD") == "1")

    def use_oneshot(self, collective: str, count: int, dtype) -> bool:
        """Small AllReduce / AllGather payloads go through the one-shot kernel (one NVLink trip, no barrier)."""
        nbytes = count * torch.tensor([], dtype=dtype).element_size()
        return (collective in ("allreduce", "allgather") and self.comm.world > 1 and 0 < nbytes
                <= self.oneshot_max_bytes and nbytes % 8 == 0 and self._oneshot_world_ok())

    def use_twoshot(self, collective: str, count: int, dtype) -> bool:
        """Mid-size AllReduce (above the one-shot range, up to ``twoshot_max_bytes``; off unless set)."""
        nbytes = count * torch.tensor([], dtype=dtype).element_size()
        world = self.comm.world
        return (collective == "allreduce" and world > 1 and self.oneshot_max_bytes < nbytes <= self.twoshot_max_bytes
                and nbytes % (8 * world) == 0 and self._oneshot_world_ok())

    def plan(self, collective: str, count: int, dtype, *, inplace: bool, op: str = "sum", root: int = 0):
        world = self.comm.world
        if self.use_oneshot(collective, count, dtype):
            return self.comm.oneshot_plan(collective, self.oneshot_max_bytes,
                                          multicast=self.comm.multicast and world > 2)
        if self.use_twoshot(collective, count, dtype):
            return self.comm.oneshot_plan("allreduce_twoshot", self.twoshot_max_bytes,
                                          multicast=self.comm.multicast and world > 2)
        default = 1 if collective in ("allgather", "broadcast") else world
        slices = self.slices_per_rank or default
        if collective in ("reduce_scatter", "alltoall") and slices % world:
            slices = world
        dname = str(dtype).split(".")[-1]
        xml = schedule_xml(collective, world, slices, inplace=inplace, datatype=dname, method=self.method,
                           root=root if collective in ("broadcast", "reduce") else 0)
        nbytes = count * torch.tensor([], dtype=dtype).element_size()
        merge = self.merge_blocks(collective, nbytes)
        multicast = self.use_multicast(collective, op, nbytes)
        push = not multicast and self.push_steps(collective, nbytes)
        probe = self.comm.compile(xml, nlanes=1, niters=1, merge=merge, push=push)
        esize = torch.tensor([], dtype=dtype).element_size()
        runtime = count * (world if collective == "allgather" else 1)
        nchunks = slices * (world if collective == "allgather" else 1)
        chunk_bytes = runtime * esize // nchunks
        lanes, iters = self.geometry(probe.device_plan.nblocks, chunk_bytes)
        share = tuple(int(v) for v in os.environ.get("VERICCL_MC_SHARE", "1/1").split("/"))
        return self.comm.compile(xml, nlanes=lanes, niters=iters, multicast=multicast, mc_share=share,
                                 merge=merge, push=push)

    def push_steps(self, collective: str, nbytes: int) -> bool:
        """Compile plain transfers as pushes (stores into the receiver) instead of pulls.

        Pushes keep read requests off the links, which matters when every GPU
        sends and receives at once.  ``VERICCL_PUSH=1`` turns it on for every
        interpreter collective, ``VERICCL_PUSH=0`` off; the default follows
        ``push_collectives``, empty because push steps measured slower than
        pulls at every size from 1 to 256 MiB on two B200s.
        """
        env = os.environ.get("VERICCL_PUSH")
        if env is not None:
            return env not in ("0", "")
        return self.comm.world > 1 and collective in self.push_collectives

    def merge_blocks(self, collective: str, nbytes: int) -> bool:
        """Run a rank's steps as one CTA group in one order (default) or each XML block on its own CTAs.

        ``VERICCL_MERGE=0`` keeps the XML blocks apart: an AllGather then pulls
        from every peer at once, each peer's chunk on its own share of the CTAs.
        """
        env = os.environ.get("VERICCL_MERGE")
        return True if env is None else env not in ("0", "")

    def _copy_in(self, flat: torch.Tensor, tensor: torch.Tensor) -> None:
        """``flat`` (contiguous) ← ``tensor`` in row-major order; pitched 2D views go through the native copy."""
        if tensor.is_contiguous():
            flat.copy_(tensor.view(-1))
        elif _pitched(tensor):
            self.comm._mod.strided_copy(flat.view(tensor.shape), tensor)
        else:
            flat.view(tensor.shape).copy_(tensor)

    def _copy_out(self, tensor: torch.Tensor, flat: torch.Tensor) -> None:
        """``tensor`` ← ``flat`` (contiguous, row-major)."""
        if tensor.is_contiguous():
            tensor.view(-1).copy_(flat)
        elif _pitched(tensor):
            self.comm._mod.strided_copy(tensor, flat.view(tensor.shape))
        else:
            tensor.copy_(flat.view(tensor.shape))

    def _heap_copy(self, tensor: torch.Tensor, tag: str) -> torch.Tensor:
        key = (tag, tensor.numel(), tensor.dtype)
        buf = self._staging.get(key)
        if buf is None:
            buf = self.comm.empty(tensor.numel(), tensor.dtype)
            self._staging[key] = buf
        return buf

    # -- collectives ---------------------------------------------------------
    def all_reduce(self, tensor: torch.Tensor, *, op: str = "sum", scale: float | None = None) -> torch.Tensor:
        """In-place AllReduce of ``tensor`` (fused reduction, cast and scale); strided views are staged."""
        n = tensor.numel()
        pad = self._padding(n, tensor.dtype, self.slices_per_rank or self.comm.world)
        if tensor.is_contiguous() and self.comm.in_heap(tensor.view(-1)) and pad == 0:
            flat = tensor.view(-1)
            plan = self.plan("allreduce", n, flat.dtype, inplace=True, op=op)
            self.comm.run(plan, flat, flat, op=op, scale=scale)
            return tensor
        count = n + pad
        buf = self._heap_copy(torch.empty(count, dtype=tensor.dtype, device="meta"), "ar")
        self._copy_in(buf[:n], tensor)
        if pad:
            buf[n:].zero_()
        plan = self.plan("allreduce", count, tensor.dtype, inplace=True, op=op)
        self.comm.run(plan, buf, buf, op=op, scale=scale)
        self._copy_out(tensor, buf[:n])
        return tensor

    def use_push(self, nbytes: int) -> bool:
        """AllGathers of at least ``VERICCL_AG_PUSH_MIN`` bytes per rank run the push kernel (off unless set)."""
        env = os.environ.get("VERICCL_AG_PUSH_MIN")
        limit = self.ag_push_min_bytes if env is None else int(env)
        return self.comm.world > 1 and limit is not None and nbytes >= limit and nbytes % 16 == 0

    def _push_all_gather(self, inp: torch.Tensor, out: torch.Tensor) -> None:
        """Every rank stores its chunk into every peer's heap output (csrc/cuda/push.cu)."""
        mod = self.comm._mod
        flags = self._staging.get("push-flags")
        if flags is None:
            ctas = max(1, min(mod.push_allgather_max_ctas(), 148))
            flags = (self.comm.empty(4 * (ctas + 1), torch.float16), ctas)
            flags[0].zero_()
            torch.cuda.synchronize()
            self.comm.barrier()
            self._staging["push-flags"] = flags
        region, ctas = flags
        env = os.environ.get("VERICCL_AG_PUSH_FANOUT")
        fanout = self.ag_push_fanout if env is None else env not in ("0", "")
        mod.push_allgather(self.comm.heap, inp.data_ptr(), self.comm.offset_of(out), inp.numel() * inp.element_size(),
                           self.comm.offset_of(region), ctas, self.comm.timeout_s, fanout)

    def all_gather(self, inp: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
        world = self.comm.world
        if out.numel() != inp.numel() * world:
            raise RuntimeFailure("all_gather output must hold world × input elements")
        nbytes = inp.numel() * inp.element_size()
        if self.use_push(nbytes) and inp.is_contiguous() and out.is_contiguous():
            dst = out.view(-1) if self.comm.in_heap(out.view(-1)) else self._heap_copy(out, "ag-push-out")
            self._push_all_gather(inp.view(-1), dst)
            if dst.data_ptr() != out.data_ptr():
                self._copy_out(out, dst)
            return out
        if inp.is_contiguous() and out.is_contiguous() and self.comm.in_heap(inp) and self.comm.in_heap(out):
            plan = self.plan("allgather", inp.numel(), inp.dtype, inplace=False)
            self.comm.run(plan, inp.view(-1), out.view(-1))
            return out
        src = self._staged(inp, "ag-in", True)
        dst = self._staged(out, "ag-out", False)
        plan = self.plan("allgather", inp.numel(), inp.dtype, inplace=False)
        self.comm.run(plan, src, dst)
        self._unstage(out, dst)
        return out

    def all_gather_fp8(self, inp: torch.Tensor, out: torch.Tensor, *, block: int = 128,
                       fused: bool | None = None) -> torch.Tensor:
        """AllGather with block-scaled FP8 (e4m3) payloads.

        Each rank's input is quantized with one fp32 scale per ``block``
        elements; only the e4m3 bytes and the scales cross NVLink (about a
        quarter of an fp32, half of a bf16 AllGather's bytes) and every rank's
        part of ``out`` is dequantized; values carry e4m3 precision and every
        rank, the owner included, sees the same values.

        With 128-element blocks and a multiple of 16 elements per rank one
        fused kernel does it all (quantize into the heap, per-CTA ready flags,
        pull and dequantize straight into ``out``: ``fp8_allgather`` in
        csrc/cuda/fp8.cu).  Otherwise (or with ``fused=False``) three passes
        run: a quantize kernel, the synthesized AllGather of the packed
        payload bytes, a dequantize kernel per rank.
        """
        world = self.comm.world
        n = inp.numel()
        if out.numel() != n * world:
            raise RuntimeFailure("all_gather_fp8 output must hold world × input elements")
        can_fuse = block == 128 and n % 16 == 0 and inp.dtype in (torch.float32, torch.bfloat16, torch.float16) \
            and out.dtype == inp.dtype
        if fused is None:
            fused = can_fuse
        if fused:
            if not can_fuse:
                raise RuntimeFailure("the fused fp8 AllGather needs 128-element blocks and 16-element multiples")
            return self._fp8_fused(inp, out)
        nblocks = -(-n // block)
        packed = -(-(n + 4 * nblocks) // 16) * 16        # bytes per rank, 16-byte aligned
        key = ("fp8", n, block)
        bufs = self._staging.get(key)
        if bufs is None:
            src = self.comm.empty(packed // 2, torch.bfloat16)
            dst = self.comm.empty(packed // 2 * world, torch.bfloat16)
            bufs = (src, dst)
            self._staging[key] = bufs
        src, dst = bufs
        raw = src.view(torch.uint8)
        self.comm._mod.quantize_fp8(inp.contiguous().view(-1), raw[:n], raw[n:n + 4 * nblocks].view(torch.float32),
                                    block)
        plan = self.plan("allgather", packed // 2, torch.bfloat16, inplace=False)
        self.comm.run(plan, src, dst)
        gathered = dst.view(torch.uint8).view(world, packed)
        flat_out = out.view(world, n)
        for r in range(world):
            part = gathered[r]
            self.comm._mod.dequantize_fp8(part[:n], part[n:n + 4 * nblocks].view(torch.float32), flat_out[r], block)
        return out

    def _fp8_fused(self, inp: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
        mod, n = self.comm._mod, inp.numel()
        key = ("fp8-fused", n)
        regions = self._staging.get(key)
        if regions is None:
            blocks = -(-n // 128)
            ctas = max(1, min(mod.fp8_allgather_max_ctas(), 4 * 148, -(-blocks // 16)))
            # heap tensors are float-typed; the regions are raw bytes
            stage = self.comm.empty(mod.fp8_stage_bytes(n), torch.float16)          # 2 parities = 2 x bytes / 2
            flags = self.comm.empty(4 * ctas, torch.float16)                         # ctas x 8 bytes
            flags.zero_()
            torch.cuda.synchronize()
            self.comm.barrier()            # every rank's flags are zero before any launch reads them
            regions = (stage, flags, ctas)
            self._staging[key] = regions
        stage, flags, ctas = regions
        src = inp.contiguous().view(-1)
        dst = out if out.is_contiguous() else torch.empty_like(out)
        mod.fp8_allgather(self.comm.heap, src, dst.view(-1), self.comm.offset_of(stage), self.comm.offset_of(flags),
                          ctas, self.comm.timeout_s)
        if dst is not out:
            out.copy_(dst)
        return out

    def reduce_scatter(self, inp: torch.Tensor, out: torch.Tensor, *, op: str = "sum",
                       scale: float | None = None) -> torch.Tensor:
        world = self.comm.world
        if inp.numel() != out.numel() * world:
            raise RuntimeFailure("reduce_scatter input must hold world × output elements")
        src, dst = self._staged(inp, "rs-in", True), self._staged(out, "rs-out", False)
        plan = self.plan("reduce_scatter", inp.numel(), inp.dtype, inplace=False)
        self.comm.run(plan, src, dst, op=op, scale=scale, count_per_rank=inp.numel())
        self._unstage(out, dst)
        return out

    def _staged(self, tensor: torch.Tensor, tag: str, copy_in: bool) -> torch.Tensor:
        """The heap tensor to run on: ``tensor`` itself when it is contiguous in the heap, else a staging buffer."""
        if tensor.is_contiguous() and self.comm.in_heap(tensor.view(-1)):
            return tensor.view(-1)
        buf = self._heap_copy(torch.empty(tensor.numel(), dtype=tensor.dtype, device="meta"), tag)
        if copy_in:
            self._copy_in(buf, tensor)
        return buf

    def _unstage(self, tensor: torch.Tensor, flat: torch.Tensor) -> None:
        """Copy a staged result back unless ``flat`` is ``tensor``'s own storage."""
        if not (tensor.is_contiguous() and flat.data_ptr() == tensor.data_ptr()):
            self._copy_out(tensor, flat)

    def broadcast(self, inp: torch.Tensor, out: torch.Tensor, *, root: int = 0) -> torch.Tensor:
        """``out`` on every rank = ``inp`` of rank ``root`` (other ranks' ``inp`` is not read)."""
        if inp.numel() != out.numel():
            raise RuntimeFailure("broadcast input and output must have the same size")
        src, dst = self._staged(inp, "bc-in", True), self._staged(out, "bc-out", False)
        plan = self.plan("broadcast", inp.numel(), inp.dtype, inplace=False, root=root)
        self.comm.run(plan, src, dst)
        self._unstage(out, dst)
        return out

    def reduce(self, inp: torch.Tensor, out: torch.Tensor, *, root: int = 0, op: str = "sum",
               scale: float | None = None) -> torch.Tensor:
        """``out`` on rank ``root`` = op over every rank's ``inp`` (fused scale).

        The schedule may use other ranks' ``out`` as intermediate storage, so
        its contents there are unspecified afterwards.
        """
        if inp.numel() != out.numel():
            raise RuntimeFailure("reduce input and output must have the same size")
        src, dst = self._staged(inp, "rd-in", True), self._staged(out, "rd-out", False)
        plan = self.plan("reduce", inp.numel(), inp.dtype, inplace=False, op=op, root=root)
        self.comm.run(plan, src, dst, op=op, scale=scale)
        self._unstage(out, dst)
        return out

    def all_to_all(self, inp: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
        """Part ``d`` of rank ``s``'s ``inp`` (world equal parts) becomes part ``s`` of rank ``d``'s ``out``."""
        world = self.comm.world
        if inp.numel() != out.numel() or inp.numel() % world:
            raise RuntimeFailure("all_to_all needs equal input/output sizes divisible by the world size")
        src, dst = self._staged(inp, "a2a-in", True), self._staged(out, "a2a-out", False)
        plan = self.plan("alltoall", inp.numel(), inp.dtype, inplace=False)
        self.comm.run(plan, src, dst)
        self._unstage(out, dst)
        return out

    def _padding(self, count: int, dtype, slices: int) -> int:
        esize = torch.tensor([], dtype=dtype).element_size()
        unit = slices * (16 // esize)
        return (-count) % unit
