"""Generate complete request documents for common cases.

``example_documents`` returns the four JSON documents (topology, sketch,
atom, runtime) for one collective on an NVSwitch B200 domain, with every
budget and tolerance the resolver requires filled in (reference:
tools/generate_examples.py, used by its README).  ``write_documents`` stores
them as ``<dir>/<name>.json``.
"""
from __future__ import annotations

from pathlib import Path

from vericcl_b200.topology.nvswitch import nvswitch_topology
from vericcl_b200.utils.jsonio import atomic_write_json


def example_documents(operator: str = "allreduce", method: str = "hierarchy", ranks: int = 8, *,
                      total_size_bytes: int = 1 << 20, slice_size_bytes: int | None = 1 << 18,
                      datatype: str = "float32", inplace: bool = False, topology: dict | None = None,
                      alpha_us: float | None = None, link_gbps: float | None = None, max_channels: int = 1,
                      tuning_rounds: int = 0, scratch_bytes: int = 1 << 30, calibration: bool = False,
                      per_model_timeout_s: float = 60.0, reduction_op: str | None = None,
                      scale: float | None = None, root: int = 0) -> dict:
    kw = {}
    if alpha_us is not None:
        kw["alpha_us"] = alpha_us
    if link_gbps is not None:
        kw["link_gbps"] = link_gbps
    topo = topology if topology is not None else nvswitch_topology(ranks, **kw)
    collective = {"operator": operator, "datatype": datatype, "inplace": inplace}
    if operator in ("allreduce", "reduce", "reduce_scatter"):
        collective["reduction_op"] = reduction_op or "sum"
        if scale is not None:
            collective["scale"] = scale
    if operator in ("broadcast", "reduce"):
        collective["root"] = root
    sketch = {
        "collective": collective,
        "hyperparameters": {"total_size_bytes": total_size_bytes, "slice_size_bytes": slice_size_bytes},
        "solver": {"backend": "highs", "per_model_timeout_s": per_model_timeout_s, "cpu_budget": 4,
                   "max_threads_per_model": 1, "max_parallel_models": 1, "max_channels": max_channels},
        "budgets": {"max_initial_synthesis_s": 600, "max_offline_validation_per_round_s": 300,
                    "max_offline_validation_total_s": 900, "max_repair_per_round_s": 300,
                    "max_repair_total_s": 900, "max_tuning_rounds": tuning_rounds, "cleanup_reserve_s": 5,
                    "max_online_validation_per_round_s": 600, "max_online_validation_total_s": 1800,
                    "max_run_wall_s": 3600},
        "tolerances": {"absolute": 1e-3, "relative": 1e-3},
        "calibration": {"enabled": calibration, "max_relative_fit_error": 0.1, "job_timeout_s": 300},
        "trace_and_measure": {"enabled": False, "job_timeout_s": 300, "trace_capacity_bytes": 1 << 24},
    }
    atom = {"synthesis_method": method, "M_switch": 1 << 24}
    # eight GPUs per host: ranks beyond the first eight go to further (named) hosts
    hosts = ["localhost" if topo["ranks"] <= 8 else "node-%d" % (r // 8) for r in range(topo["ranks"])]
    runtime = {"rank_map": [{"rank": r, "host": hosts[r], "device": r % 8} for r in range(topo["ranks"])],
               "environment": {"NCCL_BUFFSIZE": str(1 << 26)},
               "scratch_bytes_per_rank": scratch_bytes,
               "control": {"bind_address": "127.0.0.1", "port": 24950}}
    return {"topology": topo, "sketch": sketch, "atom": atom, "runtime": runtime}


def write_documents(directory, documents: dict) -> dict:
    directory = Path(directory)
    files = {}
    for name in ("topology", "sketch", "atom", "runtime"):
        files[name] = atomic_write_json(directory / (name + ".json"), documents[name])
    return files
