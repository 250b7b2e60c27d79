"""Communicator: one process per GPU, a symmetric peer-mapped heap, compiled plans.

Bootstrap uses ``torch.distributed`` for the host-side plumbing only (a gloo
group carries the session token and the barriers between the collective
set-up phases); every collective byte then moves through this package's own
kernels over NVLink.  Heap set-up phases: create + export (each rank), import
and map every peer, add the device to the NVLS multicast object, bind and map
the multicast range (reference counterpart: NCCL's bootstrap and P2P
transport, third_party/msccl/src/bootstrap.cc and src/transport/p2p.cc).

Buffers handed to a plan must live in the heap at the same offset on every
rank (allocate them in the same order on every rank with :meth:`empty`); the
offsets of each (input, output, scratch) triple are checked across ranks the
first time a plan sees them.
"""
from __future__ import annotations

import os
import secrets
import threading
from dataclasses import dataclass

import torch

from vericcl_b200.errors import RuntimeFailure
from vericcl_b200.ops import native
from vericcl_b200.program.device import REDOPS, REDUCING

DTYPE_CODES = {torch.float32: 0, torch.bfloat16: 1, torch.float16: 2}
TORCH_DTYPES = {"float32": torch.float32, "bfloat16": torch.bfloat16, "float16": torch.float16}
DEFAULT_HEAP_BYTES = 1 << 30
TIMELINE_SLOTS = 256      # launch timeline slots (matches the device-side constant)


def _bulk_mode(value) -> int:
    """The staged-instance mode: 0 off, 1 TMA loads, 3 TMA loads and (for local plain copies) TMA stores."""
    if value in (None, "", "0", "false", "False"):
        return 0
    if value in ("true", "True"):
        return 1
    mode = int(value)
    if mode not in (1, 3):
        raise ValueError("VERICCL_BULK must be 0, 1 or 3, not %r" % value)
    return mode


# Per rank count, the per-rank payload windows (bytes, inclusive) in which the TMA-staged instance measured
# faster than the vector path on B200s, after passing the fp64 collective checks on that many GPUs:
#   2 ranks: AllGather 16-256 MiB +3-27 %; pull AllReduce 64-256 MiB +2-5 %, 16-25 MiB level or 0.5 % slower.
#   4 ranks: AllGather 16-256 MiB +3-5 %, 1 GiB 14 % slower (pull reductions not measured).
#   8 ranks: AllGather 16 MiB +6.6 %, 64 MiB 1.8 % slower, 256 MiB-1 GiB 6-28 % slower; the window stops at 32 MiB
#            because the crossover between 16 and 64 MiB is not measured.
BULK_WINDOWS = {
    2: {"allgather": (16 << 20, 256 << 20), "other": (64 << 20, 256 << 20)},
    4: {"allgather": (16 << 20, 256 << 20)},
    8: {"allgather": (16 << 20, 32 << 20)},
}


def _env_flag(name: str, default: bool) -> bool:
    value = os.environ.get(name)
    if value is None:
        return default
    return value not in ("0", "false", "False", "")


@dataclass
class PlanHandle:
    device_plan: object
    xml: str
    collective: str
    nlanes: int
    niters: int
    slots: tuple
    checked: set
    multicast: bool = False
    kind: str = "interp"


@dataclass
class OneShotPlan:
    """Small-message AllReduce / AllGather with the one-shot flag-in-data kernel (no device program)."""
    collective: str
    max_bytes: int
    checked: set
    kind: str = "oneshot"
    nlanes: int = 0
    niters: int = 1
    multicast: bool = False
    xml: str | None = None
    device_plan: object = None


ONESHOT_COLLS = {"allreduce": 0, "allgather": 1, "allreduce_twoshot": 2}


class Communicator:
    """A set of ranks (one GPU each) sharing a symmetric heap."""

    def __init__(self, group=None, *, heap_bytes: int | None = None, multicast: bool | None = None,
                 device: int | None = None, timeout_s: float = 10.0):
        import torch.distributed as dist
        self._dist = dist if dist.is_available() and dist.is_initialized() else None
        if self._dist is not None:
            self.rank = dist.get_rank(group)
            self.world = dist.get_world_size(group)
            backend = dist.get_backend(group)
            self.control_group = group if backend == "gloo" else dist.new_group(
                ranks=dist.get_process_group_ranks(group) if group is not None else None, backend="gloo")
        else:
            self.rank, self.world, self.control_group = 0, 1, None
        if device is None:
            device = int(os.environ.get("LOCAL_RANK", self.rank)) % max(1, torch.cuda.device_count())
        torch.cuda.set_device(device)
        self.device = device
        self.timeout_s = timeout_s
        heap_bytes = int(heap_bytes or os.environ.get("VERICCL_HEAP_BYTES", DEFAULT_HEAP_BYTES))
        multicast = _env_flag("VERICCL_NVLS", False) if multicast is None else multicast
        token = [secrets.token_hex(6) if self.rank == 0 else None]
        if self._dist is not None and self.world > 1:
            self._dist.broadcast_object_list(token, src=self._global(0), group=self.control_group)
        self.session = "%s.%d" % (token[0], os.getpid() if self.world == 1 else 0)
        mod = native.cuda()
        self._mod = mod
        self.heap = self._build_heap(heap_bytes, bool(multicast))
        if multicast and not self.heap_multicast_everywhere():
            # NVLS could not be set up on every rank: rebuild the heap without it on all ranks
            self.heap.destroy()
            self.barrier()
            self.session += ".u"
            self.heap = self._build_heap(heap_bytes, False)
        self._allocs: dict[int, int] = {}
        self._bound: dict = {}
        self._plans: dict = {}
        self._scratch: dict = {}
        self._ll = None              # (offset, bytes per source) of the one-shot LL region
        # Sum/avg launches use the register-lean interpreter instance when VERICCL_LEAN=1, and by default on a
        # single rank, where every step is a one-source copy (its copies keep eight vectors in flight per thread)
        self.lean = _env_flag("VERICCL_LEAN", self.world == 1)
        # copy and reduce steps stage their sources in shared memory with TMA bulk copies (VERICCL_BULK=1); with
        # VERICCL_BULK=3 staged plain copies into local memory are written back by TMA too (a bit mask, 0..3).
        # Unset (None): chosen per launch by bulk_for()
        env = os.environ.get("VERICCL_BULK")
        self.bulk = None if env is None else _bulk_mode(env)
        # per-machine staged windows from a tuning table ({"allgather": [lo, hi], "other": [lo, hi]}); None: the
        # built-in BULK_WINDOWS of this rank count
        self.bulk_windows = None
        self._lock = threading.Lock()
        self._closed = False

    def _build_heap(self, heap_bytes: int, multicast: bool):
        heap = self._mod.Heap(self.rank, self.world, self.device, heap_bytes, self.session, multicast)
        self.barrier()
        heap.exchange(60.0)
        self.barrier()
        error = None
        try:
            heap.bind_multicast()
        except RuntimeError as exc:       # a failed bind leaves the heap usable for peer access
            error = str(exc)
        self.setup_error = error
        self.barrier()
        heap.finish()
        return heap

    def heap_multicast_everywhere(self) -> bool:
        flags = self.all_gather_object(bool(self.heap.multicast))
        return all(flags)

    # -- host control plane ------------------------------------------------
    def _global(self, rank: int) -> int:
        if self._dist is None or self.control_group is None:
            return rank
        return self._dist.get_global_rank(self.control_group, rank)

    def barrier(self) -> None:
        if self._dist is not None and self.world > 1:
            self._dist.barrier(group=self.control_group)

    def all_gather_object(self, value):
        if self._dist is None or self.world == 1:
            return [value]
        out = [None] * self.world
        self._dist.all_gather_object(out, value, group=self.control_group)
        return out

    @property
    def multicast(self) -> bool:
        return bool(self.heap.multicast)

    # -- memory --------------------------------------------------------------
    def empty(self, numel: int, dtype=torch.float32) -> torch.Tensor:
        """Allocate a heap tensor (collective: every rank allocates in the same order)."""
        code = DTYPE_CODES[dtype]
        nbytes = numel * torch.tensor([], dtype=dtype).element_size()
        offset = self.heap.alloc(max(nbytes, 16))
        tensor = self.heap.tensor(offset, numel, code)
        self._allocs[tensor.data_ptr()] = offset
        return tensor

    def free(self, tensor: torch.Tensor) -> None:
        ptr = tensor.data_ptr()
        self._bound = {k: v for k, v in self._bound.items() if ptr not in k[1:4]}
        offset = self._allocs.pop(ptr, None)
        if offset is not None:
            self.heap.free(offset)

    def offset_of(self, tensor: torch.Tensor) -> int:
        return self.heap.offset_of(tensor)

    def in_heap(self, tensor: torch.Tensor) -> bool:
        try:
            self.heap.offset_of(tensor)
            return True
        except RuntimeError:
            return False

    # -- plans ----------------------------------------------------------------
    def compile(self, xml: str, *, nlanes: int = 1, niters: int = 1, elide: bool = True, fuse: bool = True,
                multicast: bool = False, mc_share: tuple = (1, 1), merge: bool = True,
                push: bool = False) -> PlanHandle:
        """Compile ``xml`` for this rank (cached).  ``push``: plain send/receive pairs become stores by the sender
        into the receiver's heap buffer instead of pulls (see csrc/plan/compile.cc)."""
        import re
        if multicast and not self.multicast:
            raise RuntimeFailure("multicast mapping requested but this communicator's heap has no NVLS binding")
        coll = re.search(r'coll="([a-z_]+)"', xml)
        collective = coll.group(1) if coll else "allreduce"
        key = (xml, nlanes, niters, elide, fuse, multicast, tuple(mc_share), merge, push)
        with self._lock:
            if key in self._plans:
                return self._plans[key]
            plan = self._mod.DevicePlan(xml, self.rank, nlanes, niters, elide, fuse, multicast,
                                        collective in REDUCING, int(mc_share[0]), int(mc_share[1]), merge, push)
            handle = PlanHandle(plan, xml, collective, nlanes, niters, tuple(plan.slots()), set(), multicast)
            self._plans[key] = handle
            return handle

    def scratch_for(self, plan: PlanHandle, count_per_rank: int, dtype, copies: int = 1) -> int:
        code = DTYPE_CODES[dtype]
        chunk, _ = plan.device_plan.geometry(count_per_rank, code)
        esize = torch.tensor([], dtype=dtype).element_size()
        need = max(16, plan.slots[2] * chunk * esize * copies)
        key = id(plan)
        with self._lock:
            have = self._scratch.get(key)
            if have is None or have[1] < need:
                if have is not None:
                    # launches already enqueued may still use the old scratch, and bound launches name it
                    torch.cuda.synchronize()
                    self.heap.free(have[0])
                    self._bound = {k: v for k, v in self._bound.items() if k[0] != key}
                self._scratch[key] = (self.heap.alloc(need), need)
            return self._scratch[key][0]

    # -- one-shot small-message path ---------------------------------------------
    def oneshot_plan(self, collective: str, max_bytes: int, *, multicast: bool = False) -> OneShotPlan:
        """Plan handle for the one-shot kernel; reserves the LL region on first use (collective call).

        With ``multicast`` (and an NVLS-bound heap) each line is pushed once
        through the multicast address instead of once per peer.
        """
        if collective not in ONESHOT_COLLS:
            raise RuntimeFailure("the one-shot path covers allreduce and allgather, not %s" % collective)
        if collective == "allreduce_twoshot":
            # both areas of the two-shot AllReduce (4 · bytes of lines) must fit one region half
            self._ensure_ll(-(-4 * max_bytes // (16 * self.world)) * 16)
        else:
            self._ensure_ll(-(-max_bytes // 8) * 16)
        multicast = bool(multicast and self.multicast)
        key = ("oneshot", collective, multicast)
        plan = self._plans.get(key)
        if plan is None or plan.max_bytes < max_bytes:
            plan = OneShotPlan(collective, max_bytes, set(), multicast=multicast)
            self._plans[key] = plan
        return plan

    def _ensure_ll(self, need: int) -> None:
        """LL region of two halves with ``need`` bytes of lines per source (grows, never shrinks)."""
        if self._ll is not None and self._ll[1] >= need:
            return
        if self._ll is not None:
            # a larger region replaces the old one; nothing may still be using it
            torch.cuda.synchronize()
            self.barrier()
            self.heap.free(self._ll[0])
        total = 2 * self.world * need
        offset = self.heap.alloc(total)
        self.heap.tensor(offset, total // 4, 0).zero_()
        torch.cuda.synchronize()
        self.barrier()
        self._ll = (offset, need)
        self._bound = {k: v for k, v in self._bound.items() if k[0] != "oneshot"}

    def _run_oneshot(self, plan: OneShotPlan, inp, out, op, scale, stream, count_per_rank) -> None:
        key = ("oneshot", id(plan), inp.data_ptr(), out.data_ptr(), count_per_rank, inp.dtype, op, scale,
               inp.numel())
        bound = self._bound.get(key)
        if bound is None:
            if inp.dtype != out.dtype:
                raise RuntimeFailure("input and output dtypes differ")
            count = inp.numel() if count_per_rank is None else count_per_rank
            nbytes = count * inp.element_size()
            if nbytes > plan.max_bytes:
                raise RuntimeFailure("one-shot plan holds %d bytes per rank, call has %d" % (plan.max_bytes, nbytes))
            if plan.collective == "allreduce_twoshot" and nbytes % (8 * self.world):
                raise RuntimeFailure("two-shot AllReduce needs a payload of whole 8-byte units per rank")
            need_out = count * (self.world if plan.collective == "allgather" else 1)
            if inp.numel() < count or out.numel() < need_out:
                raise RuntimeFailure("one-shot %s needs %d input and %d output elements, got %d and %d"
                                     % (plan.collective, count, need_out, inp.numel(), out.numel()))
            in_off, out_off = self.offset_of(inp), self.offset_of(out)
            offsets = (in_off, out_off, nbytes)
            if offsets not in plan.checked:
                got = self.all_gather_object(offsets)
                if any(o != offsets for o in got):
                    raise RuntimeFailure("one-shot buffers are not symmetric across ranks: %s" % (got,))
                plan.checked.add(offsets)
            factor = 1.0 / self.world if op == "avg" else 1.0
            if scale is not None:
                factor *= scale
            redop = REDOPS["sum" if op == "avg" else op]
            bound = self._mod.bind_oneshot(self.heap, in_off, out_off, self._ll[0], self._ll[1], nbytes,
                                           DTYPE_CODES[inp.dtype], redop, ONESHOT_COLLS[plan.collective],
                                           float(factor), factor != 1.0, self.timeout_s,
                                           plan.multicast and self.multicast)
            self._bound[key] = bound
        bound.launch((torch.cuda.current_stream() if stream is None else stream).cuda_stream)

    def run(self, plan: PlanHandle, inp: torch.Tensor, out: torch.Tensor, *, op: str = "sum",
            scale: float | None = None, stream=None, count_per_rank: int | None = None, nbatch: int = 1,
            in_stride: int = 0, out_stride: int = 0, trace: torch.Tensor | None = None,
            timeline: torch.Tensor | None = None) -> None:
        """Launch ``plan`` on heap tensors ``inp`` → ``out`` on ``stream`` (asynchronous).

        With ``nbatch > 1`` one launch runs the plan ``nbatch`` times back to back on
        buffers ``in_stride`` / ``out_stride`` elements apart (for example every
        gradient bucket of a flat buffer); the instances pipeline through the same
        persistent CTAs and only the last one waits for peers at the end.
        ``timeline`` (from :meth:`timeline_buffer`) records kernel entry and
        exit times per launch on this GPU (:meth:`launch_gaps` reads them).
        """
        if plan.kind == "oneshot":
            if nbatch != 1 or trace is not None:
                raise RuntimeFailure("the one-shot path runs one instance without tracing")
            self._run_oneshot(plan, inp, out, op, scale, stream, count_per_rank)
            return
        tl_ptr = 0 if timeline is None else timeline.data_ptr()
        bulk = 0 if tl_ptr else self.bulk_for(plan, (inp.numel() if count_per_rank is None else count_per_rank)
                                              * inp.element_size())
        bound_key = (id(plan), inp.data_ptr(), out.data_ptr(), count_per_rank, inp.numel(), out.numel(), inp.dtype,
                     op, scale, nbatch, in_stride, out_stride, tl_ptr, bulk, self.lean)
        if trace is None:
            fast = self._bound.get(bound_key)
            if fast is not None:
                fast.launch((torch.cuda.current_stream() if stream is None else stream).cuda_stream)
                return
        if inp.dtype != out.dtype:
            raise RuntimeFailure("input and output dtypes differ")
        count = inp.numel() if count_per_rank is None else count_per_rank
        in_off, out_off = self.offset_of(inp), self.offset_of(out)
        esize = inp.element_size()
        scr_off = self.scratch_for(plan, count, inp.dtype, copies=nbatch)
        chunk, _ = plan.device_plan.geometry(count, DTYPE_CODES[inp.dtype])
        if inp.numel() < plan.slots[0] * chunk or out.numel() < plan.slots[1] * chunk:
            raise RuntimeFailure("%s plan reads %d and writes %d elements per instance; tensors hold %d and %d"
                                 % (plan.collective, plan.slots[0] * chunk, plan.slots[1] * chunk, inp.numel(),
                                    out.numel()))
        scr_stride = plan.slots[2] * chunk * esize
        strides = [in_stride * esize, out_stride * esize, scr_stride]
        key = (in_off, out_off, scr_off, count, nbatch, tuple(strides))
        if key not in plan.checked:
            offsets = self.all_gather_object(key)
            if any(o != key for o in offsets):
                raise RuntimeFailure("plan buffers are not symmetric across ranks: %s" % (offsets,))
            plan.checked.add(key)
        if plan.multicast and op not in ("sum", "avg"):
            raise RuntimeFailure("a multicast-mapped plan only reduces with sum/avg; compile without multicast")
        factor = 1.0 / self.world if op == "avg" else 1.0
        if scale is not None:
            factor *= scale
        stream = torch.cuda.current_stream() if stream is None else stream
        trace_ptr, trace_stride = 0, 0
        if trace is not None:
            trace_stride = plan.niters * nbatch * plan.device_plan.max_steps()
            need = plan.device_plan.nblocks * plan.nlanes * trace_stride * 3
            if trace.dtype != torch.int64 or trace.numel() < need or not trace.is_cuda:
                raise RuntimeFailure("trace buffer needs %d int64 elements on the device" % need)
            trace.zero_()
            trace_ptr = trace.data_ptr()
        if trace is None:
            if timeline is not None and (timeline.dtype != torch.int64 or timeline.numel() < 2 * TIMELINE_SLOTS
                                         or not timeline.is_cuda):
                raise RuntimeFailure("timeline buffer needs %d int64 elements on the device" % (2 * TIMELINE_SLOTS))
            lean = self.lean and REDOPS[op] == 0
            bound = plan.device_plan.bind(self.heap, in_off, out_off, scr_off, count, DTYPE_CODES[inp.dtype],
                                          REDOPS[op], float(factor), self.timeout_s, 512, nbatch, strides, tl_ptr,
                                          lean, bulk)
            self._bound[bound_key] = bound
            bound.launch(stream.cuda_stream)
            return
        plan.device_plan.run(self.heap, in_off, out_off, scr_off, count, DTYPE_CODES[inp.dtype], REDOPS[op],
                             float(factor), stream.cuda_stream, self.timeout_s, 512, nbatch, strides, trace_ptr,
                             trace_stride)

    def bulk_for(self, plan, nbytes: int) -> int:
        """Interpreter instance mode for one launch: the explicit ``bulk`` setting, else TMA-staged loads (1) when
        the plan has no multicast steps (the staged path covers copy and reduce steps only) and the per-rank
        payload lies in this rank count's measured window (``bulk_windows`` from a tuning table, else
        ``BULK_WINDOWS``), else the vector path (0)."""
        if self.bulk is not None:
            return int(self.bulk)
        windows = BULK_WINDOWS.get(self.world, {}) if getattr(self, "bulk_windows", None) is None \
            else self.bulk_windows
        window = windows.get("allgather" if getattr(plan, "collective", "") == "allgather" else "other")
        if window is not None and not plan.multicast and window[0] <= nbytes <= window[1]:
            return 1
        return 0

    def timeline_buffer(self) -> torch.Tensor:
        return torch.zeros(2 * TIMELINE_SLOTS, dtype=torch.int64, device="cuda")

    def launch_gaps(self, timeline: torch.Tensor, launches: int) -> dict:
        """Kernel durations and the idle gaps between consecutive launches (µs) of the last ``launches``."""
        epoch = int(self.status()["epoch"])
        tl = timeline.view(TIMELINE_SLOTS, 2).cpu().tolist()
        spans = []
        for e in range(max(1, epoch - launches), epoch):
            entry, exit_ = tl[e % TIMELINE_SLOTS]
            if entry and exit_:
                spans.append((entry, exit_))
        durations = [(b - a) / 1e3 for a, b in spans]
        gaps = [(spans[i + 1][0] - spans[i][1]) / 1e3 for i in range(len(spans) - 1)]
        med = (lambda v: sorted(v)[len(v) // 2] if v else None)
        return {"launches": len(spans), "kernel_us_median": med(durations), "gap_us_median": med(gaps),
                "kernel_us": durations, "gap_us": gaps}

    def trace_buffer(self, plan: PlanHandle, nbatch: int = 1) -> torch.Tensor:
        n = plan.device_plan.nblocks * plan.nlanes * plan.niters * nbatch * plan.device_plan.max_steps() * 3
        return torch.zeros(n, dtype=torch.int64, device="cuda")

    def clock_samples(self, count: int = 16):
        """(host_before_ns, gpu_globaltimer_ns, host_after_ns) bracketing samples of this rank's GPU."""
        import time as _time
        buf = torch.zeros(1, dtype=torch.int64, device="cuda")
        out = []
        for _ in range(count):
            torch.cuda.synchronize()
            t0 = _time.time_ns()
            self._mod.read_timer(buf)
            torch.cuda.synchronize()
            t1 = _time.time_ns()
            out.append((t0, int(buf.item()), t1))
        return out

    def status(self) -> dict:
        return self.heap.status()

    def check_status(self) -> None:
        st = self.heap.status()
        if st["status"] != 0:
            raise RuntimeFailure("device status %d (rank, block, lane, wait) = %s" % (st["status"], st["detail"]))

    def close(self) -> None:
        if self._closed:
            return
        self._closed = True
        torch.cuda.synchronize()
        self.barrier()
        self._plans.clear()
        self.heap.destroy()
        self.barrier()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()
