"""Load, migrate, override and resolve the four request documents.

Behaviour follows the reference loader (vericcl/input/loader.py:26 and
vericcl/input/schema.py:390-470): strict JSON, schema normalisation with value
provenance, ``--set FIELD=JSON`` overrides that may only fill unspecified
values unless ``override_input`` is given, cross-field arithmetic (M divisible
by S, whole elements), enabling rules per purpose, automatic method selection
through ``M_switch`` and a size-accounting record.
"""
from __future__ import annotations

import copy
from pathlib import Path

from vericcl_b200.errors import InputValidationError
from vericcl_b200.input import schema as S
from vericcl_b200.input.models import (AtomConstraints, ForbiddenTransfer, Hyperparameters, ResolvedInput,
                                       SolverConfig)
from vericcl_b200.semantics.collective import CollectiveKind, CollectiveSpec, validate_problem
from vericcl_b200.utils.hashing import digest
from vericcl_b200.utils.jsonio import strict_load, strict_loads

DOCUMENTS = ("topology", "sketch", "atom", "runtime")
PURPOSES = ("solve", "verify", "calibrate")


def parse_override(text: str):
    """Parse ``a.b.c=JSON`` into (path tuple, value)."""
    if "=" not in text:
        raise InputValidationError("override must look like FIELD=JSON: " + text)
    key, raw = text.split("=", 1)
    parts = tuple(part for part in key.strip().split(".") if part)
    if len(parts) < 2 or parts[0] not in DOCUMENTS:
        raise InputValidationError("override field must start with topology/sketch/atom/runtime: " + key)
    return parts, strict_loads(raw)


def migrate(documents: dict) -> dict:
    """Apply the supported legacy migrations in place; return their origins.

    Operator aliases are normalised (docs/input-schema.md:11); atom-level
    ``symmetry/shortest_paths/batching/objective_mode`` move under
    ``atom.strategies``.  A field present in both its old and new locations
    is an error even when the values agree.
    """
    origins = {}
    collective = documents["sketch"].get("collective")
    if isinstance(collective, dict) and isinstance(collective.get("operator"), str):
        op = collective["operator"].lower()
        collective["operator"] = S.OPERATOR_ALIASES.get(op, op)
    atom = documents["atom"]
    for key in ("symmetry", "shortest_paths", "batching", "objective_mode"):
        if key in atom:
            strategies = atom.setdefault("strategies", {})
            if not isinstance(strategies, dict):
                raise InputValidationError("atom.strategies must be an object")
            if key in strategies:
                raise InputValidationError("atom.%s is present in both its old and new locations" % key)
            strategies[key] = atom.pop(key)
            origins["atom.strategies." + key] = "migrated from atom." + key
    manual = atom.get("manual")
    if isinstance(manual, dict):
        for node in manual.get("nodes") or []:
            if isinstance(node, dict) and isinstance(node.get("operator"), str):
                op = node["operator"].lower()
                node["operator"] = S.OPERATOR_ALIASES.get(op, op)
    return origins


def _apply_overrides(documents, overrides, override_input, sources):
    for text in overrides or ():
        parts, value = parse_override(text) if isinstance(text, str) else text
        target = documents[parts[0]]
        for part in parts[1:-1]:
            if target.get(part) is None:
                target[part] = {}
            target = target[part]
            if not isinstance(target, dict):
                raise InputValidationError("override path crosses a non-object: " + ".".join(parts))
        leaf = parts[-1]
        existing = target.get(leaf)
        if existing is not None and existing != value and not override_input:
            raise InputValidationError("override changes a specified value; pass --override-input: " + ".".join(parts))
        target[leaf] = value
        sources[".".join(parts)] = {"kind": "override", "replaced": existing is not None}


def _required(section: dict, key: str, prefix: str):
    if section.get(key) is None:
        raise InputValidationError("%s.%s is required for this request" % (prefix, key))
    return section[key]


def _validate_topology(topology, runtime):
    ranks = topology["ranks"]
    covered = [r for node in topology["nodes"] for r in node["ranks"]]
    if sorted(covered) != list(range(ranks)):
        raise InputValidationError("topology.nodes must cover every rank exactly once")
    if len({node["id"] for node in topology["nodes"]}) != len(topology["nodes"]):
        raise InputValidationError("topology.nodes ids must be unique")
    for node in topology["nodes"]:
        if not set(node["gateways"]) <= set(node["ranks"]):
            raise InputValidationError("a node gateway must belong to its node")
    resource_ids = [item["id"] for item in topology["shared_resources"]]
    if len(set(resource_ids)) != len(resource_ids):
        raise InputValidationError("duplicate shared resource id")
    links = set()
    for edge in topology["directed_links"]:
        pair = (edge["src"], edge["dst"])
        if max(pair) >= ranks or pair[0] == pair[1] or pair in links:
            raise InputValidationError("invalid or duplicate directed link %s" % (pair,))
        if not set(edge["resources"]) <= set(resource_ids):
            raise InputValidationError("directed link references an unknown shared resource")
        links.add(pair)
    for resource in topology["shared_resources"]:
        if not {tuple(edge) for edge in resource["links"]} <= links:
            raise InputValidationError("shared resource %s references an unknown link" % resource["id"])
    for group in topology["groups"] + topology["multicast_groups"]:
        if len(set(group)) != len(group) or max(group) >= ranks:
            raise InputValidationError("invalid topology group")
    for cost in topology["local_costs"]:
        if cost["rank"] >= ranks:
            raise InputValidationError("local cost names an unknown rank")
    mapping = runtime["rank_map"]
    if sorted(item["rank"] for item in mapping) != list(range(ranks)):
        raise InputValidationError("runtime.rank_map must contain every rank exactly once")
    if len({(item["host"], item["device"]) for item in mapping}) != ranks:
        raise InputValidationError("runtime.rank_map must use a distinct device per rank on each host")
    raw = runtime["environment"]["NCCL_BUFFSIZE"]
    if not raw.isascii() or not raw.isdigit() or not 8 <= int(raw) <= 2 ** 31 - 1:
        raise InputValidationError("NCCL_BUFFSIZE must be an integer byte count from 8 to 2147483647")


def _validate_enabled(config, purpose):
    sketch = config["sketch"]
    budgets, solver = sketch["budgets"], sketch["solver"]
    for key in ("per_model_timeout_s", "cpu_budget"):
        _required(solver, key, "sketch.solver")
    for key in ("cleanup_reserve_s", "max_offline_validation_per_round_s", "max_offline_validation_total_s"):
        _required(budgets, key, "sketch.budgets")
    if purpose == "solve":
        for key in ("max_initial_synthesis_s", "max_tuning_rounds"):
            _required(budgets, key, "sketch.budgets")
        if budgets["max_tuning_rounds"]:
            for key in ("max_repair_per_round_s", "max_repair_total_s"):
                _required(budgets, key, "sketch.budgets")
    calibration, measured = sketch["calibration"], sketch["trace_and_measure"]
    if calibration["enabled"] or measured["enabled"] or purpose == "calibrate":
        for key in ("max_online_validation_per_round_s", "max_online_validation_total_s"):
            _required(budgets, key, "sketch.budgets")
    if calibration["enabled"] or purpose == "calibrate":
        for key in ("max_relative_fit_error", "job_timeout_s"):
            _required(calibration, key, "sketch.calibration")
    if measured["pairs"] % 2 or measured["pairs"] < 2:
        raise InputValidationError("sketch.trace_and_measure.pairs must be even and at least two")
    if measured["max_rounds"] > 3 or measured["max_cv"] > .05 or measured["min_relative_gain"] >= 1:
        raise InputValidationError("trace_and_measure needs max_rounds <= 3, max_cv <= .05, min_relative_gain < 1")
    if measured["enabled"]:
        for key in ("job_timeout_s", "trace_capacity_bytes"):
            _required(measured, key, "sketch.trace_and_measure")
    history = sketch["history"]
    if history["schedule_reuse"]:
        for key in ("relative_bandwidth_tolerance", "max_schedule_candidates", "schedule_index"):
            _required(history, key, "sketch.history")
    if history["calibration_reuse"]:
        for key in ("calibration_max_age_s", "calibration_index"):
            _required(history, key, "sketch.history")


def expanded_forbidden_transfers(atom: dict):
    """Expand manual ``atoms`` variable groups plus explicit forbidden transfers.

    Each group ``{slice_ids, src_ranks, dst_ranks}`` of a manual node expands to
    the cross product with the node's stage (README.md "Atom variable groups").
    Duplicates are removed; the result is sorted.
    """
    values = {tuple(item) for item in atom["forbidden_transfers"]}
    if atom["manual"]["enabled"]:
        for node in atom["manual"]["nodes"]:
            group = set(node["group"])
            for item in node["atoms"]:
                for slice_id in item["slice_ids"]:
                    for src in item["src_ranks"]:
                        for dst in item["dst_ranks"]:
                            if src == dst or src not in group or dst not in group:
                                raise InputValidationError("manual atom edge must join two distinct group ranks")
                            values.add((slice_id, src, dst, node["stage_id"]))
    return tuple(sorted(values))


def resolve_documents(documents: dict, *, origins=None, overrides=None, override_input=False,
                      purpose="solve") -> ResolvedInput:
    """Resolve already-parsed documents (``{name: dict}``) into a request."""
    if purpose not in PURPOSES:
        raise InputValidationError("invalid request purpose " + repr(purpose))
    if set(documents) != set(DOCUMENTS):
        raise InputValidationError("request needs exactly topology, sketch, atom and runtime")
    documents = {k: copy.deepcopy(v) for k, v in documents.items()}
    for name, value in documents.items():
        if not isinstance(value, dict):
            raise InputValidationError(name + " must be a JSON object")
    migrated = migrate(documents)
    sources: dict = {key: {"kind": "migrated", "detail": value} for key, value in migrated.items()}
    _apply_overrides(documents, overrides, override_input, sources)
    origins = origins or {}
    config = {name: S.normalize(S.SCHEMAS[name], documents[name], name, sources, origins.get(name, name))
              for name in DOCUMENTS}
    topology, sketch, atom, runtime = (config[k] for k in DOCUMENTS)
    _validate_topology(topology, runtime)
    ranks = topology["ranks"]
    collective = sketch["collective"]
    kind = CollectiveKind(collective["operator"])
    rooted = kind in (CollectiveKind.BROADCAST, CollectiveKind.REDUCE)
    reducing = kind in (CollectiveKind.REDUCE, CollectiveKind.ALL_REDUCE, CollectiveKind.REDUCE_SCATTER)
    for key, applies, default in (("root", rooted, 0), ("reduction_op", reducing, "sum")):
        if applies and key not in collective:
            collective[key] = default
            sources["sketch.collective." + key] = {"kind": "default"}
        elif not applies and key in collective:
            raise InputValidationError("collective.%s is not applicable to %s" % (key, kind.value))
        elif not applies:
            collective[key] = None
    if "scale" in collective and not reducing:
        raise InputValidationError("collective.scale only applies to reducing collectives")
    spec = CollectiveSpec(kind, collective["datatype"], collective["reduction_op"], collective["root"],
                          collective["inplace"], collective.get("scale"))
    hyper = sketch["hyperparameters"]
    size, slice_size = hyper["total_size_bytes"], hyper["slice_size_bytes"]
    reference = hyper["reference_slice_size_bytes"]
    element = S.DATATYPE_BYTES[spec.datatype]
    if size % element:
        raise InputValidationError("total_size_bytes must contain whole datatype elements")
    for value in (slice_size, reference):
        if value is not None and (value % element or size % value):
            raise InputValidationError("slice size must divide total_size_bytes and hold whole elements")
    slice_count = None if slice_size is None else size // slice_size
    validate_problem(spec, ranks, slice_count if slice_count is not None else size // element)
    if reducing and spec.datatype in ("float16", "float32", "float64", "bfloat16", "float8_e4m3"):
        for key in ("absolute", "relative"):
            _required(sketch["tolerances"], key, "sketch.tolerances")
    method = atom["synthesis_method"]
    if atom["manual"]["enabled"]:
        if method == "constructive_trees":
            raise InputValidationError("manual stage plans require synthesis_method=hierarchy or auto")
        if sketch["history"]["schedule_reuse"]:
            raise InputValidationError("manual stage plans require history.schedule_reuse=false")
        method = "hierarchy"
    elif method == "auto":
        threshold = _required(atom, "M_switch", "atom")
        method = "hierarchy" if size < threshold else "constructive_trees"
        sources["derived.selected_synthesis_method"] = {"kind": "derived", "expression": "M < M_switch",
                                                        "value": method}
    if method == "constructive_trees" and atom["strategies"]["shortest_paths"]:
        raise InputValidationError("shortest_paths is only an initial hierarchy option")
    forbidden = []
    values = expanded_forbidden_transfers(atom)
    if values:
        if reference is None and slice_size is not None:
            reference = slice_size
            hyper["reference_slice_size_bytes"] = reference
            sources["sketch.hyperparameters.reference_slice_size_bytes"] = {
                "kind": "derived", "expression": "explicit slice_size_bytes", "value": reference}
        if reference is None:
            raise InputValidationError("reference_slice_size_bytes is required to bind slice_id constraints")
        for slice_id, src, dst, stage in values:
            if (slice_id >= ranks * (size // reference) or max(src, dst) >= ranks or src == dst
                    or (atom["stage_num"] is not None and stage >= atom["stage_num"])):
                raise InputValidationError("forbidden transfer is outside its partition/rank/stage domain")
            forbidden.append(ForbiddenTransfer(slice_id, src, dst, stage))
    _validate_enabled(config, purpose)
    solver = sketch["solver"]
    if kind is CollectiveKind.ALL_GATHER:
        output = size * ranks
    elif kind is CollectiveKind.REDUCE_SCATTER:
        output = size // ranks
    else:
        output = size
    accounting = {"input_bytes_per_rank": size, "slice_size_bytes": slice_size, "slices_per_rank": slice_count,
                  "valid_output_bytes": output, "element_bytes": element,
                  "output_ranks": [spec.root] if kind is CollectiveKind.REDUCE else list(range(ranks)),
                  "nccl_tests_size_bytes": size * ranks if kind is CollectiveKind.ALL_GATHER else size}
    request_config = {name: config[name] for name in DOCUMENTS}
    return ResolvedInput(
        collective=spec,
        hyperparameters=Hyperparameters(size, slice_size, reference),
        solver=SolverConfig(solver["backend"], float(solver["per_model_timeout_s"]), solver["cpu_budget"],
                            solver["max_threads_per_model"], solver.get("max_parallel_models") or 1,
                            solver["max_channels"], solver["solver_seed"], float(solver["mip_gap"]),
                            solver["require_proven_optimal"]),
        atom_constraints=AtomConstraints(atom["stage_num"], tuple(forbidden)),
        rank_count=ranks,
        selected_synthesis_method=method,
        input_sha256=digest(request_config),
        request_config=request_config,
        value_sources=dict(sorted(sources.items())),
        size_accounting=accounting,
        purpose=purpose,
    )


def load_request(files, overrides=None, *, override_input=False, purpose="solve") -> ResolvedInput:
    """Load ``{"topology": path, "sketch": path, "atom": path, "runtime": path}``."""
    if not isinstance(files, dict) or set(files) != set(DOCUMENTS):
        raise InputValidationError("request files must name topology, sketch, atom and runtime")
    documents, origins = {}, {}
    for name in DOCUMENTS:
        path = Path(files[name])
        if not path.is_file():
            raise InputValidationError("%s file does not exist: %s" % (name, path))
        documents[name] = strict_load(path)
        origins[name] = str(path.resolve())
    return resolve_documents(documents, origins=origins, overrides=overrides, override_input=override_input,
                             purpose=purpose)
