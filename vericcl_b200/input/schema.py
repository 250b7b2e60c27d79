"""Declarative schema of the four request documents and its normaliser.

The field set, defaults, bounds and enabling rules follow the reference's
public contract (vericcl/input/schema.py:78-174, docs/input-schema.md:18-227):
topology.json, sketch.json, atom.json and runtime.json.  The DSL here is a
small tree of :class:`Node` records; ``normalize`` walks a document against it,
rejects unknown keys and out-of-range values, fills defaults and records the
provenance of every value in ``value_sources``.  ``json_schema`` exports the
same tree as JSON Schema (draft 2020-12) for the published schema files.

One deliberate difference: ``sketch.solver.backend`` accepts ``"highs"`` (the
default here, the MILP engine shipped with SciPy) as well as ``"scip"`` which
is accepted as an alias because PySCIPOpt is not available on the B200 image.
"""
from __future__ import annotations

import copy
import math
from dataclasses import dataclass, field
from typing import Any

from vericcl_b200.errors import InputValidationError

INT_MAX = 2 ** 63 - 1
_ABSENT = object()

DATATYPE_BYTES = {"float16": 2, "float32": 4, "float64": 8, "bfloat16": 2, "int8": 1, "uint8": 1,
                  "int32": 4, "uint32": 4, "int64": 8, "uint64": 8, "float8_e4m3": 1}
OPERATORS = ("broadcast", "reduce", "allgather", "allreduce", "alltoall", "reduce_scatter")
MANUAL_OPERATORS = ("broadcast", "reduce", "scatter", "gather", "allgather", "allreduce", "alltoall",
                    "reduce_scatter")
OPERATOR_ALIASES = {"all_gather": "allgather", "all_reduce": "allreduce", "all_to_all": "alltoall",
                    "reducescatter": "reduce_scatter"}
REDUCTIONS = ("sum", "prod", "min", "max", "avg")
ENVIRONMENT_KEYS = ("CUDA_HOME", "CUDA_PATH", "CUDA_VISIBLE_DEVICES", "LD_LIBRARY_PATH", "MSCCL_ROOT",
                    "MSCCL_XML_FILES", "NCCL_ALGO", "NCCL_BUFFSIZE", "NCCL_DEBUG", "NCCL_DEBUG_SUBSYS",
                    "NCCL_IB_GID_INDEX", "NCCL_IB_HCA", "NCCL_P2P_DISABLE", "NCCL_PROTO", "NCCL_SHM_DISABLE",
                    "NCCL_SOCKET_IFNAME", "NCCL_TESTS_ROOT", "NCCL_NVLS_ENABLE", "OMPI_MCA_btl",
                    "OMPI_MCA_btl_tcp_if_include", "OMPI_MCA_oob_tcp_if_include", "OMPI_MCA_pml",
                    "OMP_NUM_THREADS", "PATH", "PYTHONPATH", "UCX_NET_DEVICES", "UCX_TLS",
                    "VERICCL_TRACE_ENABLE", "VERICCL_NVLS")


@dataclass
class Node:
    """One schema node: a scalar, an object or an array."""

    kind: str                      # integer | number | string | boolean | object | array
    default: Any = _ABSENT
    enum: tuple | None = None
    minimum: float | None = None
    maximum: float | None = None
    exclusive_minimum: float | None = None
    properties: dict = field(default_factory=dict)
    required: tuple = ()
    items: "Node | None" = None
    min_items: int = 0
    max_items: int | None = None
    doc: str = ""
    open_map: bool = False         # object whose keys come from ``enum`` (environment)


def integer(minimum=0, maximum=INT_MAX, default=_ABSENT, doc=""):
    return Node("integer", default=default, minimum=minimum, maximum=maximum, doc=doc)


def number(default=_ABSENT, minimum=None, maximum=None, exclusive_minimum=None, doc=""):
    return Node("number", default=default, minimum=minimum, maximum=maximum,
                exclusive_minimum=exclusive_minimum, doc=doc)


def positive(default=_ABSENT, doc=""):
    return number(default=default, exclusive_minimum=0, doc=doc)


def string(default=_ABSENT, enum=None, doc=""):
    return Node("string", default=default, enum=None if enum is None else tuple(enum), doc=doc)


def boolean(default=False, doc=""):
    return Node("boolean", default=default, doc=doc)


def obj(properties, required=(), default=_ABSENT, doc=""):
    return Node("object", properties=properties, required=tuple(required), default=default, doc=doc)


def section(properties, doc=""):
    return obj(properties, default={}, doc=doc)


def array(items, default=_ABSENT, min_items=0, max_items=None, doc=""):
    return Node("array", items=items, default=default, min_items=min_items, max_items=max_items, doc=doc)


COST = obj({"alpha_us": number(minimum=0, doc="Fixed service overhead per operation, in microseconds."),
            "beta_us_per_byte": positive(doc="Service cost per byte, in microseconds per byte.")},
           required=("alpha_us", "beta_us_per_byte"))

TOPOLOGY = obj({
    "name": string(default="unspecified", doc="Topology name, used only for identification."),
    "ranks": integer(minimum=1, doc="Number of logical ranks."),
    "nodes": array(obj({"id": integer(doc="Node identifier."),
                        "ranks": array(integer(), min_items=1, doc="Ranks of this node."),
                        "gateways": array(integer(), default=[], doc="Ranks that connect this node externally.")},
                       required=("id", "ranks")), min_items=1, doc="Node groups covering every rank."),
    "directed_links": array(obj({
        "src": integer(doc="Sending rank."), "dst": integer(doc="Receiving rank."),
        "alpha_us": number(minimum=0, doc="Fixed service overhead per operation, in microseconds."),
        "beta_us_per_byte": positive(doc="Service cost per byte; bandwidth is its reciprocal."),
        "max_channels": integer(minimum=1, maximum=16, default=16, doc="Maximum channel count."),
        "resources": array(string(), default=[], doc="Shared resources used by this link."),
        "physical_path": array(string(), default=[], doc="Physical path of the abstract link.")},
        required=("src", "dst", "alpha_us", "beta_us_per_byte")), doc="Directed links."),
    "shared_resources": array(obj({
        "id": string(doc="Resource identifier."),
        "capacity_bytes_per_us": positive(doc="Total effective bandwidth in bytes per microsecond."),
        "links": array(array(integer(), min_items=2, max_items=2), default=[], doc="Member links [src,dst]."),
        "kind": string(default="other", enum=("nic", "pcie", "switch_port", "link", "nvlink_port", "nvls",
                                             "other"), doc="Resource category.")},
        required=("id", "capacity_bytes_per_us")), default=[], doc="Shared bottlenecks."),
    "groups": array(array(integer(), min_items=1), default=[], doc="Candidate groups for hierarchy."),
    "multicast_groups": array(array(integer(), min_items=2), default=[],
                              doc="Rank sets that share an NVLS multicast object (NVSwitch in-switch reduction)."),
    "local_costs": array(obj({"rank": integer(), "copy": COST, "reduce": COST}, required=("rank",)),
                         default=[], doc="Initial local copy/reduce costs."),
    "provenance": obj({
        "legacy_format": string(enum=("taccl_topology_v2",), doc="Format of the converted source."),
        "reference_slice_bytes": integer(minimum=1, doc="Chunk size the source durations refer to."),
        "source_topology": string(doc="Canonical JSON of the source topology."),
        "source_sketch": string(doc="Canonical JSON of the source sketch.")},
        required=("legacy_format", "reference_slice_bytes", "source_topology", "source_sketch"),
        doc="Sources of a topology converted from another format (topology/legacy.py)."),
}, required=("ranks", "nodes", "directed_links"))

BUDGETS = {k: positive() for k in (
    "max_initial_synthesis_s", "max_online_validation_per_round_s", "max_online_validation_total_s",
    "max_offline_validation_per_round_s", "max_offline_validation_total_s", "max_repair_per_round_s",
    "max_repair_total_s", "max_run_wall_s", "cleanup_reserve_s")}
BUDGETS["max_tuning_rounds"] = integer()

SKETCH = obj({
    "collective": obj({
        "operator": string(enum=OPERATORS, doc="Collective operator."),
        "datatype": string(default="float32", enum=tuple(DATATYPE_BYTES), doc="Element datatype."),
        "root": integer(doc="Root for broadcast/reduce."),
        "reduction_op": string(enum=REDUCTIONS, doc="Reduction operation."),
        "inplace": boolean(False, doc="Use the in-place buffer layout."),
        "scale": positive(doc="Optional factor applied to every reduced output (fused into the final store)."),
    }, required=("operator",)),
    "hyperparameters": obj({
        "total_size_bytes": integer(minimum=1, doc="Input bytes M per rank."),
        "slice_size_bytes": Node("integer", default=None, minimum=1, maximum=INT_MAX, doc="Slice size S."),
        "reference_slice_size_bytes": Node("integer", default=None, minimum=1, maximum=INT_MAX,
                                           doc="Reference partition for slice_id constraints."),
    }, required=("total_size_bytes",)),
    "solver": section({
        "backend": string(default="highs", enum=("highs", "scip"), doc="MILP backend (scip is an alias)."),
        "per_model_timeout_s": positive(), "cpu_budget": integer(minimum=1),
        "max_threads_per_model": integer(minimum=1, default=12), "max_parallel_models": integer(minimum=1),
        "max_channels": integer(minimum=1, maximum=16, default=7), "solver_seed": integer(default=0),
        "mip_gap": number(minimum=0, maximum=1, default=0), "require_proven_optimal": boolean(False),
        "bdd_backend": string(default="native", enum=("native", "cudd", "autoref")),
    }),
    "budgets": section(BUDGETS),
    "tolerances": section({"absolute": number(minimum=0), "relative": number(minimum=0)}),
    "calibration": section({
        "enabled": boolean(True), "launches": integer(minimum=1, default=20),
        "warmup_iterations": integer(default=5), "timed_iterations": integer(minimum=1, default=20),
        "max_rounds": integer(minimum=1, default=3), "max_cv": positive(default=0.05),
        "max_relative_fit_error": number(minimum=0), "job_timeout_s": positive(),
        "payload_sizes": array(integer(minimum=1), default=[]),
        "probe_scope": string(default="every_link", enum=("every_link", "link_classes"),
                              doc="every_link probes each directed link; link_classes probes two links of every "
                                  "class of interchangeable links (same α, β, placement and shared-resource kinds) "
                                  "and one rank per node, and gives the fit to the whole class"),
    }),
    "trace_and_measure": section({
        "enabled": boolean(False), "pairs": integer(minimum=1, default=20),
        "warmup_iterations": integer(default=5), "timed_iterations": integer(minimum=1, default=20),
        "max_rounds": integer(minimum=1, default=3), "max_cv": positive(default=0.05),
        "min_relative_gain": number(minimum=0, maximum=1, default=0),
        "task_alpha": number(exclusive_minimum=0, maximum=0.05, default=0.05),
        "single_attempt_alpha_cap": number(exclusive_minimum=0, maximum=0.05, default=0.05),
        "seed": integer(default=0), "job_timeout_s": positive(), "trace_capacity_bytes": integer(minimum=1),
    }),
    "repair": section({"mode": string(default="strategy_first", enum=("strategy_first", "joint")),
                       "candidate_batch_size": integer(minimum=1, default=4),
                       "analysis_batch_size": integer(minimum=1, default=16)}),
    "runtime_compatibility": section({"enabled": boolean(True)}),
    "history": section({
        "schedule_reuse": boolean(False), "calibration_reuse": boolean(False),
        "relative_bandwidth_tolerance": number(minimum=0), "max_schedule_candidates": integer(minimum=1),
        "calibration_max_age_s": positive(), "schedule_index": string(), "calibration_index": string(),
    }),
}, required=("collective", "hyperparameters"))

STATE = obj({"rank": integer(), "offset": integer(), "contributors": array(integer())},
            required=("rank", "offset", "contributors"))
ATOM = obj({
    "synthesis_method": string(default="auto", enum=("auto", "hierarchy", "constructive_trees")),
    "M_switch": integer(minimum=1),
    "stage_num": Node("integer", default=None, minimum=1, maximum=INT_MAX),
    "forbidden_transfers": array(array(integer(), min_items=4, max_items=4), default=[]),
    "strategies": section({"symmetry": boolean(False), "shortest_paths": boolean(False),
                           "batching": boolean(False),
                           "objective_mode": Node("string", default=None,
                                                  enum=("latency", "throughput", "auto"))}),
    "manual": section({
        "enabled": boolean(False),
        "nodes": array(obj({
            "id": string(), "stage_id": integer(), "operator": string(enum=MANUAL_OPERATORS),
            "group": array(integer(), min_items=1), "root": integer(),
            "relay_ranks": array(integer(), default=[]),
            "atoms": array(obj({"slice_ids": array(integer(), min_items=1),
                                "src_ranks": array(integer(), min_items=1),
                                "dst_ranks": array(integer(), min_items=1)},
                               required=("slice_ids", "src_ranks", "dst_ranks")), default=[]),
            "depends_on": array(string(), default=[]),
            "input_states": array(STATE), "output_states": array(STATE),
        }, required=("id", "stage_id", "operator", "group")), default=[]),
    }),
})

ENVIRONMENT = Node("object", properties={k: string() for k in ENVIRONMENT_KEYS}, open_map=False,
                   required=("NCCL_BUFFSIZE",))
RUNTIME = obj({
    "rank_map": array(obj({"rank": integer(), "host": string(), "device": integer()},
                          required=("rank", "host", "device")), min_items=1),
    "environment": ENVIRONMENT,
    "paths": section({k: string() for k in ("cuda_home", "mpi_bin", "msccl_root", "nccl_tests_root",
                                            "vericcl_driver", "vericcl_native")}),
    "device_memory_budget_bytes": integer(default=0),
    "protocol": string(default="Simple", enum=("Simple",)),
    "scratch_bytes_per_rank": integer(),
    "limits": section({"steps_per_tb": integer(minimum=1, maximum=256, default=256),
                       "tbs_per_rank": integer(minimum=1, maximum=216, default=216),
                       "send_tbs_per_channel": integer(minimum=1, maximum=32, default=32),
                       "recv_tbs_per_channel": integer(minimum=1, maximum=32, default=32),
                       "dependency_id": integer(maximum=127, default=127),
                       "buffer_offset": integer(maximum=32767, default=32767)}),
    "tb_layout": string(default="separate", enum=("separate", "fused")),
    "control": section({"bind_address": string(), "port": integer(minimum=1, maximum=65535)}),
}, required=("rank_map", "environment", "scratch_bytes_per_rank"))

SCHEMAS = {"topology": TOPOLOGY, "sketch": SKETCH, "atom": ATOM, "runtime": RUNTIME}


def _type_ok(node: Node, value) -> bool:
    if node.kind == "integer":
        return isinstance(value, int) and not isinstance(value, bool)
    if node.kind == "number":
        return isinstance(value, (int, float)) and not isinstance(value, bool) and math.isfinite(value)
    if node.kind == "string":
        return isinstance(value, str) and len(value) >= 1
    if node.kind == "boolean":
        return isinstance(value, bool)
    if node.kind == "object":
        return isinstance(value, dict)
    if node.kind == "array":
        return isinstance(value, list)
    raise InputValidationError("unknown schema node kind " + node.kind)


def normalize(node: Node, value, path: str, sources: dict, origin: str):
    """Validate ``value`` against ``node``; return a new normalised value.

    Absent/null members take their default (recorded as ``default`` in
    ``sources``); members without a default stay absent so that enabling rules
    can report them.  Provided values are recorded with ``origin``.
    """
    if not _type_ok(node, value):
        raise InputValidationError("%s must be of type %s" % (path, node.kind))
    if node.kind in ("integer", "number"):
        if node.minimum is not None and value < node.minimum:
            raise InputValidationError("%s must be >= %s" % (path, node.minimum))
        if node.maximum is not None and value > node.maximum:
            raise InputValidationError("%s must be <= %s" % (path, node.maximum))
        if node.exclusive_minimum is not None and value <= node.exclusive_minimum:
            raise InputValidationError("%s must be > %s" % (path, node.exclusive_minimum))
        return value
    if node.kind == "string":
        if node.enum is not None and value not in node.enum:
            raise InputValidationError("%s must be one of %s" % (path, ", ".join(node.enum)))
        return value
    if node.kind == "boolean":
        return value
    if node.kind == "array":
        if len(value) < node.min_items or (node.max_items is not None and len(value) > node.max_items):
            raise InputValidationError("%s has an invalid number of items" % path)
        return [normalize(node.items, item, "%s[%d]" % (path, i), sources, origin) for i, item in enumerate(value)]
    result = {}
    unknown = set(value) - set(node.properties)
    if unknown:
        raise InputValidationError("%s has unknown fields: %s" % (path, ", ".join(sorted(unknown))))
    for key, child in node.properties.items():
        child_path = path + "." + key
        present = key in value and value[key] is not None
        if present:
            result[key] = normalize(child, value[key], child_path, sources, origin)
            sources.setdefault(child_path, {"kind": "input", "file": origin})
        elif key in node.required:
            raise InputValidationError("%s is required" % child_path)
        elif child.default is not _ABSENT:
            default = copy.deepcopy(child.default)
            if child.kind == "object" and isinstance(default, dict):
                default = normalize(child, default, child_path, sources, "default")
            result[key] = default
            sources.setdefault(child_path, {"kind": "default"})
    return result


def json_schema(node: Node, title: str | None = None) -> dict:
    """Export ``node`` as a JSON Schema document."""
    out: dict = {}
    if title:
        out["$schema"] = "https://json-schema.org/draft/2020-12/schema"
        out["title"] = title
    out["type"] = node.kind
    if node.doc:
        out["description"] = node.doc
    if node.default is not _ABSENT:
        out["default"] = node.default
    if node.enum is not None:
        out["enum"] = list(node.enum)
    for key, attr in (("minimum", "minimum"), ("maximum", "maximum"), ("exclusiveMinimum", "exclusive_minimum")):
        if getattr(node, attr) is not None:
            out[key] = getattr(node, attr)
    if node.kind == "object":
        out["properties"] = {k: json_schema(v) for k, v in node.properties.items()}
        out["required"] = list(node.required)
        out["additionalProperties"] = False
    if node.kind == "array":
        out["items"] = json_schema(node.items)
        out["minItems"] = node.min_items
        if node.max_items is not None:
            out["maxItems"] = node.max_items
    return out


def field_rows(node: Node, path: str):
    """Yield (path, node) for documentation tables."""
    yield path, node
    if node.kind == "object":
        for key, child in node.properties.items():
            yield from field_rows(child, path + "." + key)
    elif node.kind == "array" and node.items is not None and node.items.kind in ("object", "array"):
        yield from field_rows(node.items, path + "[]")
