"""Engine routing on the host: which collectives and sizes take the one-shot path."""
from types import SimpleNamespace

import torch

from vericcl_b200.models.collectives import ONESHOT_MAX_BYTES, CollectiveEngine


class _Comm:
    def __init__(self, world):
        self.world = world
        self.multicast = world >= 4
        self._mod = SimpleNamespace(max_ctas=lambda threads=512: 148)
        self.requests = []

    def oneshot_plan(self, collective, max_bytes, multicast=False):
        self.requests.append((collective, max_bytes))
        return SimpleNamespace(kind="oneshot", collective=collective, max_bytes=max_bytes)


def test_small_allreduce_and_allgather_take_the_oneshot_path():
    comm = _Comm(8)
    eng = CollectiveEngine(comm, oneshot_max_bytes=ONESHOT_MAX_BYTES)
    assert eng.use_oneshot("allreduce", 512, torch.bfloat16)
    assert eng.use_oneshot("allgather", ONESHOT_MAX_BYTES // 4, torch.float32)
    assert not eng.use_oneshot("allgather", ONESHOT_MAX_BYTES // 4 + 2, torch.float32)
    assert not eng.use_oneshot("reduce_scatter", 512, torch.bfloat16)
    assert not eng.use_oneshot("allreduce", 3, torch.bfloat16)          # 6 bytes: not whole 8-byte units
    plan = eng.plan("allreduce", 512, torch.bfloat16, inplace=True)
    assert plan.kind == "oneshot" and comm.requests == [("allreduce", ONESHOT_MAX_BYTES)]


def test_single_rank_and_disabled_threshold_use_the_interpreter():
    assert not CollectiveEngine(_Comm(1)).use_oneshot("allreduce", 512, torch.bfloat16)
    assert not CollectiveEngine(_Comm(8), oneshot_max_bytes=0).use_oneshot("allreduce", 512, torch.bfloat16)


def test_large_allgathers_pull_from_peers():
    from vericcl_b200.models.collectives import AG_NVLS_MAX_BYTES
    eng = CollectiveEngine(_Comm(8))
    assert eng.use_multicast("allreduce", "sum", 1 << 30)
    assert eng.use_multicast("allgather", "sum", AG_NVLS_MAX_BYTES - 16)
    assert not eng.use_multicast("allgather", "sum", AG_NVLS_MAX_BYTES)
    assert not CollectiveEngine(_Comm(2)).use_multicast("allreduce", "sum", 1 << 20)


def test_twoshot_window_is_opt_in():
    comm = _Comm(8)
    off = CollectiveEngine(comm)
    assert off.twoshot_max_bytes == 0 and not off.use_twoshot("allreduce", 1 << 21, torch.bfloat16)
    on = CollectiveEngine(comm, twoshot_max_bytes=8 << 20)
    assert on.use_twoshot("allreduce", 1 << 21, torch.bfloat16)            # 4 MiB
    assert not on.use_twoshot("allreduce", 1 << 19, torch.bfloat16)        # 1 MiB: one-shot range
    assert not on.use_twoshot("allgather", 1 << 21, torch.bfloat16)
    plan = on.plan("allreduce", 1 << 21, torch.bfloat16, inplace=True)
    assert plan.collective == "allreduce_twoshot" and comm.requests[-1] == ("allreduce_twoshot", 8 << 20)


def test_cta_budget_caps_the_interpreter_grid():
    """A budget of B CTAs gives at most max(1, B // blocks) lanes per schedule block; no budget fills the GPU."""
    full = CollectiveEngine(_Comm(8))
    assert full.geometry(8, 64 << 20)[0] == 148 // 8
    small = CollectiveEngine(_Comm(8), cta_budget=32)
    assert small.geometry(8, 64 << 20)[0] == 4
    assert small.geometry(64, 64 << 20)[0] == 1            # below the block count: one lane per block
    assert CollectiveEngine(_Comm(8), cta_budget=4096).geometry(8, 64 << 20)[0] == 148 // 8


def test_tma_staged_instance_is_chosen_inside_the_measured_windows():
    import pytest
    from vericcl_b200.parallel.comm import BULK_WINDOWS, Communicator, _bulk_mode
    ag = SimpleNamespace(multicast=False, collective="allgather")
    ar = SimpleNamespace(multicast=False, collective="allreduce")
    nvls = SimpleNamespace(multicast=True, collective="allreduce")
    mib = 1 << 20

    def pick(world, plan, nbytes, bulk=None):
        return Communicator.bulk_for(SimpleNamespace(bulk=bulk, world=world), plan, nbytes)

    assert [pick(2, ag, n * mib) for n in (4, 16, 256, 1024)] == [0, 1, 1, 0]
    assert [pick(2, ar, n * mib) for n in (16, 25, 64, 256, 512)] == [0, 0, 1, 1, 0]
    assert [pick(4, ag, n * mib) for n in (16, 256, 1024)] == [1, 1, 0]
    assert pick(4, ar, 128 * mib) == 0                          # pull reductions on four ranks: not measured
    assert [pick(8, ag, n * mib) for n in (8, 16, 32, 64)] == [0, 1, 1, 0]
    assert pick(2, nvls, 128 * mib) == 0                        # multimem steps are not staged
    assert pick(1, ag, 64 * mib) == 0 and pick(16, ag, 64 * mib) == 0
    assert pick(1, ag, 16, bulk=3) == 3                         # an explicit setting wins
    assert set(BULK_WINDOWS) == {2, 4, 8}
    assert [_bulk_mode(v) for v in (None, "0", "1", "3", "true")] == [0, 0, 1, 3, 1]
    with pytest.raises(ValueError):
        _bulk_mode("2")
