"""Data-parallel gradient synchronisation with bucketed, scaled AllReduce.

Gradients live in one flat buffer of the communicator's symmetric heap, cut
into fixed-size buckets (25 MiB by default).  One AllReduce schedule is
synthesized for the bucket shape and replayed for every bucket; the gradient
scale (for example 1/world for averaging, or a loss-scale correction) is fused
into the final store of each reduced slice, so no separate elementwise pass
runs.  A partial last bucket is padded inside the buffer so every bucket uses
the same compiled plan geometry (the padding holds zeros).

All buckets run in one persistent launch by default.  On an NVLS plan the
launch keeps to ``NVLS_BUCKET_CTAS`` CTAs per GPU, which measured as fast as
every SM, so a backward pass can overlap it; ``cta_budget`` sets another
budget.  ``sync_from_host`` takes the gradients from pinned host memory and
overlaps their host-to-device copy, group of buckets by group, with the
AllReduce of the groups already copied.
"""
from __future__ import annotations

import torch

from vericcl_b200.models.collectives import CollectiveEngine

DEFAULT_BUCKET_BYTES = 25 * 1024 * 1024
# CTAs per GPU of an NVLS (multicast) bucket plan when no budget is given: the switch does the reduction, and on
# 4 and 8 B200s 16, 32, 64 and 148 CTAs synced 16 GB of 25 MiB buckets in the same time (within 0.7 %), so the
# sync keeps 32 and leaves the other SMs to overlapping compute
NVLS_BUCKET_CTAS = 32


def bucket_groups(buckets: int, groups: int) -> list:
    """``[(first, end), ...]``: ``buckets`` consecutive buckets cut into at most ``groups`` runs of equal length
    (the last may be shorter), in order."""
    if buckets < 1:
        return []
    groups = max(1, min(groups, buckets))
    per = -(-buckets // groups)
    return [(b0, min(buckets, b0 + per)) for b0 in range(0, buckets, per)]


class GradBucketAllReduce:
    def __init__(self, comm, numel: int, *, dtype=torch.bfloat16, bucket_bytes: int = DEFAULT_BUCKET_BYTES,
                 scale: float | None = None, slices_per_rank: int | None = None, cta_budget: int | None = None):
        """``cta_budget``: CTAs per GPU for the sync (None: ``NVLS_BUCKET_CTAS`` on an NVLS plan, else every SM)."""
        self.comm = comm
        self.dtype = dtype
        self.numel = numel
        esize = torch.tensor([], dtype=dtype).element_size()
        world = comm.world
        slices = slices_per_rank or world
        unit = slices * (16 // esize)
        self.bucket_elems = max(unit, (bucket_bytes // esize) // unit * unit)
        self.buckets = -(-numel // self.bucket_elems)
        self.scale = 1.0 / world if scale is None else scale
        self.grads = comm.empty(self.buckets * self.bucket_elems, dtype)
        self.grads[numel:].zero_()
        self.engine = CollectiveEngine(comm, slices_per_rank=slices, cta_budget=cta_budget)
        self.plan = self.engine.plan("allreduce", self.bucket_elems, dtype, inplace=True)
        if cta_budget is None and self.plan.kind != "oneshot" and self.plan.multicast:
            self.plan = self.plan_with_budget(NVLS_BUCKET_CTAS)

    def plan_with_budget(self, ctas: int):
        """The bucket plan launched on about ``ctas`` CTAs per GPU, leaving the other SMs to overlapping compute.

        The grid is (thread blocks of the schedule) × lanes, so a budget below the
        schedule's block count still launches one lane per block.
        """
        eng = CollectiveEngine(self.comm, slices_per_rank=self.engine.slices_per_rank, cta_budget=ctas)
        return eng.plan("allreduce", self.bucket_elems, self.dtype, inplace=True)

    @staticmethod
    def ctas_of(plan) -> int:
        """CTAs per GPU one launch of ``plan`` occupies (one-shot plans report their own grid)."""
        if plan.device_plan is None:
            return int(getattr(plan, "nlanes", 0) or 0)
        return plan.device_plan.nblocks * plan.nlanes

    @property
    def flat(self) -> torch.Tensor:
        """The gradient buffer (first ``numel`` elements are the real gradients)."""
        return self.grads[:self.numel]

    def bucket(self, i: int) -> torch.Tensor:
        return self.grads[i * self.bucket_elems:(i + 1) * self.bucket_elems]

    def sync(self, stream=None, *, batched: bool = True, plan=None) -> None:
        """AllReduce every bucket in place with the fused scale (asynchronous on ``stream``).

        By default all buckets run in one persistent launch (the bucket index is an
        outer pipeline dimension of the replayed schedule); ``batched=False`` issues one
        launch per bucket.  Buckets small enough for the one-shot path are launched one by
        one (that kernel has no batched form; each launch is a few microseconds).
        ``plan`` replaces the default bucket plan (for example one from :meth:`plan_with_budget`).
        """
        plan = plan or self.plan
        if batched and plan.kind != "oneshot":
            b = self.bucket(0)
            self.comm.run(plan, b, b, op="sum", scale=self.scale, stream=stream, nbatch=self.buckets,
                          in_stride=self.bucket_elems, out_stride=self.bucket_elems)
            return
        for i in range(self.buckets):
            b = self.bucket(i)
            self.comm.run(plan, b, b, op="sum", scale=self.scale, stream=stream)

    def sync_from_host(self, host: torch.Tensor, stream=None, *, groups: int = 8, copy_stream=None) -> int:
        """Copy the gradients in from pinned host memory and AllReduce them, the two overlapped.

        The buckets are cut into ``groups`` consecutive groups.  Group g is copied
        host→device on ``copy_stream`` (a side stream by default) while the
        AllReduce of group g-1 runs on ``stream``; each group's AllReduce waits
        for its own copy only (an event).  The copy stream first waits for the
        work already queued on ``stream``, so a previous step's readers of the
        buffer finish before it is overwritten.  Returns the number of
        AllReduce launches issued.  ``host`` holds ``numel`` elements of the
        buffer's dtype; pinned memory makes the copies asynchronous.
        """
        if host.numel() != self.numel or host.dtype != self.dtype or host.is_cuda:
            raise ValueError("host gradients must be a CPU tensor of %d %s elements" % (self.numel, self.dtype))
        stream = torch.cuda.current_stream() if stream is None else stream
        if copy_stream is None:
            copy_stream = getattr(self, "_copy_stream", None)
            if copy_stream is None:
                copy_stream = self._copy_stream = torch.cuda.Stream()
        copy_stream.wait_stream(stream)
        launches = 0
        for b0, b1 in bucket_groups(self.buckets, groups):
            lo, hi = b0 * self.bucket_elems, min(self.numel, b1 * self.bucket_elems)
            with torch.cuda.stream(copy_stream):
                self.grads[lo:hi].copy_(host[lo:hi], non_blocking=True)
                landed = torch.cuda.Event()
                landed.record(copy_stream)
            stream.wait_event(landed)
            first = self.bucket(b0)
            if self.plan.kind != "oneshot":
                self.comm.run(self.plan, first, first, op="sum", scale=self.scale, stream=stream, nbatch=b1 - b0,
                              in_stride=self.bucket_elems, out_stride=self.bucket_elems)
                launches += 1
            else:
                for i in range(b0, b1):
                    b = self.bucket(i)
                    self.comm.run(self.plan, b, b, op="sum", scale=self.scale, stream=stream)
                    launches += 1
        return launches

    @property
    def launches_per_sync(self) -> int:
        return self.buckets if self.plan.kind == "oneshot" else 1

    def bus_bytes_per_rank(self) -> float:
        """NCCL-convention bus bytes of one full sync (2(P-1)/P × bytes; P=1 counts the bytes once)."""
        world = self.comm.world
        nbytes = self.numel * self.grads.element_size()
        return nbytes * (2.0 * (world - 1) / world if world > 1 else 1.0)

    def nvlink_bytes_per_rank(self) -> float:
        """Bytes one GPU sends (and receives) over NVLink in one full sync, for the path the plan takes.

        Peer pulls (reduce-scatter, then all-gather of the reduced slices) move
        2(P-1)/P × bytes each way.  The NVLS path reads every GPU's copy of each
        slice once through the switch (multimem.ld_reduce, bytes out of every GPU)
        and multicasts each reduced slice once (bytes/P into the switch per GPU,
        bytes out of the switch into every GPU): about (1 + 1/P) × bytes each way.
        One GPU moves nothing over NVLink.
        """
        world = self.comm.world
        nbytes = self.numel * self.grads.element_size()
        if world == 1:
            return 0.0
        if self.plan.kind != "oneshot" and self.plan.multicast:
            return nbytes * (1.0 + 1.0 / world)
        return nbytes * 2.0 * (world - 1) / world
