"""Threshold derivation of the engine tuner from measured path times."""
from types import SimpleNamespace

from vericcl_b200.models.tuner import derive_thresholds, save_tuning

KiB, MiB = 1 << 10, 1 << 20
SIZES = [64 * KiB, 256 * KiB, 1 * MiB, 4 * MiB, 16 * MiB, 64 * MiB]


def _series(fn):
    return {s: fn(s) for s in SIZES}


def test_thresholds_follow_the_crossovers():
    times = {
        ("allreduce", "oneshot"): _series(lambda s: 5 + s / 100e3),          # wins up to 1 MiB
        ("allgather", "oneshot"): _series(lambda s: 5 + s / 120e3),
        ("allreduce", "interp"): _series(lambda s: 20 + s / 400e3),
        ("allgather", "interp"): _series(lambda s: 20 + s / 300e3),            # NVLS
        ("allreduce", "twoshot"): _series(lambda s: 10 + s / 300e3),           # beats interp up to 4 MiB
        ("allgather", "interp_p2p"): _series(lambda s: 25 + s / 400e3),        # pulls win from 16 MiB
    }
    table = derive_thresholds(times, default_ag_nvls=8 * MiB)
    assert table["oneshot_max_bytes"] == 1 * MiB
    assert table["twoshot_max_bytes"] == 4 * MiB
    assert table["ag_nvls_max_bytes"] == 16 * MiB


def test_missing_paths_keep_safe_defaults(tmp_path):
    times = {("allreduce", "interp"): _series(lambda s: 1.0), ("allgather", "interp"): _series(lambda s: 1.0)}
    table = derive_thresholds(times, default_ag_nvls=8 * MiB)
    assert table == {"oneshot_max_bytes": 0, "twoshot_max_bytes": 0, "ag_nvls_max_bytes": 8 * MiB}
    path = tmp_path / "tuning.json"
    save_tuning(path, "8|B200|580", table)
    save_tuning(path, "4|B200|580", dict(table, oneshot_max_bytes=MiB))
    import json
    data = json.loads(path.read_text())
    assert set(data) == {"8|B200|580", "4|B200|580"} and data["4|B200|580"]["oneshot_max_bytes"] == MiB


class _Comm:
    world, multicast = 8, True
    _mod = SimpleNamespace(max_ctas=lambda threads=512: 148)


def test_engine_applies_a_tuning_table():
    from vericcl_b200.models.collectives import CollectiveEngine
    eng = CollectiveEngine(_Comm(), tuning={"oneshot_max_bytes": 2 * MiB, "twoshot_max_bytes": 8 * MiB,
                                             "ag_nvls_max_bytes": 32 * MiB})
    assert (eng.oneshot_max_bytes, eng.twoshot_max_bytes, eng.ag_nvls_max_bytes) == (2 * MiB, 8 * MiB, 32 * MiB)
    explicit = CollectiveEngine(_Comm(), oneshot_max_bytes=0, tuning={"oneshot_max_bytes": 2 * MiB})
    assert explicit.oneshot_max_bytes == 0


def test_staged_windows_come_from_the_measured_crossovers():
    from vericcl_b200.models.tuner import staged_window
    vector = _series(lambda s: 10 + s / 400e3)
    staged = {s: (vector[s] * 0.9 if 1 * MiB <= s <= 16 * MiB else vector[s] * 1.05) for s in SIZES}
    assert staged_window(vector, staged) == [1 * MiB, 16 * MiB]
    assert staged_window(vector, {s: vector[s] * 0.995 for s in SIZES}) is None      # within the 1 % margin
    times = {("allreduce", "interp"): _series(lambda s: 1.0), ("allgather", "interp"): _series(lambda s: 1.0),
             ("allgather", "pull_vector"): vector, ("allgather", "pull_staged"): staged}
    table = derive_thresholds(times, default_ag_nvls=8 * MiB)
    assert table["bulk_windows"] == {"allgather": [1 * MiB, 16 * MiB]}


def test_engine_installs_measured_staged_windows():
    from vericcl_b200.models.collectives import CollectiveEngine
    from vericcl_b200.parallel.comm import Communicator
    comm = _Comm()
    comm.bulk, comm.bulk_windows = None, None
    CollectiveEngine(comm, tuning={"bulk_windows": {"allgather": [1 * MiB, 16 * MiB]}})
    assert comm.bulk_windows == {"allgather": (1 * MiB, 16 * MiB)}
    ag = SimpleNamespace(multicast=False, collective="allgather")
    assert Communicator.bulk_for(comm, ag, 4 * MiB) == 1
    assert Communicator.bulk_for(comm, ag, 64 * MiB) == 0                # outside the measured window
    ar = SimpleNamespace(multicast=False, collective="allreduce")
    assert Communicator.bulk_for(comm, ar, 4 * MiB) == 0                 # no window measured for reductions
    forced = _Comm()
    forced.bulk, forced.bulk_windows = 0, None                            # an explicit setting keeps priority
    CollectiveEngine(forced, tuning={"bulk_windows": {"allgather": [1, 2]}})
    assert forced.bulk_windows is None
