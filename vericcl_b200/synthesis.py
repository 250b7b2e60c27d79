"""One-call synthesis front end: request → checked candidate bundle.

``synthesize`` runs the initial pipeline the workflow uses for one (S, C)
choice: plan (direct, hierarchy or manual), demands, route MILP,
composition, storage plan, native lowering, XML emission, the eight
admission checks and the exact T_pred (reference call stack:
vericcl/workflow_v5.py:193 initial_candidates → xml/v5_lower.py:338
lower_and_check).  ``schedule_xml`` is the shortcut the runtime API uses to
obtain a verified XML for a collective on an NVSwitch domain.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from functools import lru_cache

from vericcl_b200.composer import compose_routes
from vericcl_b200.errors import SemanticError
from vericcl_b200.performance.initial import initial_cost_model, model_context
from vericcl_b200.planner.direct import build_direct_plan
from vericcl_b200.program.native import build_executable, lower_program
from vericcl_b200.program.storage import build_storage_plan
from vericcl_b200.program.xmlio import emit_xml
from vericcl_b200.solver.demands import build_demands
from vericcl_b200.solver.routing import choose_trees
from vericcl_b200.topology import load_topology


@dataclass
class CandidateBundle:
    request: object
    plan: object
    network: object
    storage: object
    program: object
    xml: str
    executable: object
    prediction: object
    checks: dict = field(default_factory=dict)
    origin: str = "direct"
    timing: dict | None = None        # seed vs solver-timed T_pred when the timing MILP ran

    @property
    def t_pred_us(self):
        return None if self.prediction is None else self.prediction.t_pred_us

    @property
    def can_execute(self) -> bool:
        required = ("semantic", "storage", "endpoint", "deadlock", "xml", "launch", "prediction")
        return all(self.checks.get(k, {}).get("status") == "valid" for k in required) and \
            self.checks.get("compatibility", {}).get("status") in ("valid", "not_run")


def plan_for(request, topology):
    method = request.selected_synthesis_method
    if request.request_config["atom"]["manual"]["enabled"]:
        from vericcl_b200.planner.manual import plan_manual
        return plan_manual(request, topology)
    if method == "hierarchy":
        from vericcl_b200.planner.hierarchy import plan_hierarchy
        return plan_hierarchy(request, topology)
    return build_direct_plan(request, topology, reason="constructive_trees_seed")


def lower_candidate(request, topology, network, model=None, *, plan=None, origin="direct") -> CandidateBundle:
    from vericcl_b200.program.checks import evaluate_program
    from vericcl_b200.performance.simulation import predict
    storage = build_storage_plan(network, request)
    program = lower_program(storage, request)
    xml = emit_xml(program)
    model = model or initial_cost_model(request)
    executable = build_executable(program, storage, request, topology, model_context(request))
    prediction = predict(executable, model, exact=True)
    bundle = CandidateBundle(request, plan, network, storage, program, xml, executable, prediction, origin=origin)
    bundle.checks = evaluate_program(bundle, topology)
    return bundle


def synthesize(request, model=None, *, channels: int = 1, timing: bool = True, plan=None) -> CandidateBundle:
    """Synthesize, lower, check and predict one candidate (``plan``: a given stage plan, else the method's)."""
    topology = load_topology(request)
    if request.hyperparameters.slice_count is None:
        raise SemanticError("synthesize needs a resolved slice size; use the parameter domain first")
    slice_bytes = request.hyperparameters.slice_size_bytes
    if request.selected_synthesis_method == "constructive_trees" and \
            not request.request_config["atom"]["manual"]["enabled"]:
        from vericcl_b200.solver.trees.construct import construct_network
        network = construct_network(request, topology, model or initial_cost_model(request), channels=channels)
        return lower_candidate(request, topology, network, model, origin="constructive_trees")
    plan = plan if plan is not None else plan_for(request, topology)
    demands = build_demands(plan, topology, slice_bytes)
    trees = choose_trees(demands, topology, slice_bytes, time_limit=request.solver.per_model_timeout_s)
    network = compose_routes(plan, demands, trees, topology, slice_bytes, channels=channels, origin=plan.mode.value)
    from vericcl_b200.solver.timing import keep_better, optimize_fixed_routes
    seed = lower_candidate(request, topology, network, model, plan=plan, origin=plan.mode.value)
    if channels > 1:
        # channels chosen for the whole schedule at once instead of round-robin per link
        from vericcl_b200.solver.global_scheduler import assign_channels
        global_net = assign_channels(network, topology, channels,
                                     max_blocks_per_rank=request.request_config["runtime"]["limits"]["tbs_per_rank"])
        try:
            alt = lower_candidate(request, topology, global_net, model, plan=plan, origin=global_net.origin)
        except SemanticError:
            alt = None
        if alt is not None and keep_better(seed, alt) is alt:
            seed, network = alt, global_net
    if not timing:
        return seed
    timed_network = optimize_fixed_routes(network, topology, time_limit=min(3.0, request.solver.per_model_timeout_s))
    if timed_network is network:
        return seed
    try:
        timed = lower_candidate(request, topology, timed_network, model, plan=plan,
                                origin=seed.origin + "+timing")
    except SemanticError as error:
        # the re-timed order can need more scratch than the budget holds: the seed stands
        seed.timing = {"seed_t_pred_us": seed.t_pred_us, "timed_t_pred_us": None, "kept": "seed",
                       "network_origin": timed_network.origin, "timed_failed": str(error)[:200]}
        return seed
    best = keep_better(seed, timed)
    best.timing = {"seed_t_pred_us": seed.t_pred_us, "timed_t_pred_us": timed.t_pred_us,
                   "kept": "timed" if best is timed else "seed", "network_origin": timed_network.origin}
    return best


def allgather_request_for(request):
    """The AllGather request over the same slices (same slice size, 1/P the bytes) of a ReduceScatter or an
    AllReduce request."""
    import json
    from vericcl_b200.input.loader import resolve_documents
    p = request.rank_count
    n = request.hyperparameters.slice_count
    if n is None or n % p:
        raise SemanticError("the slice count must be a multiple of the rank count")
    docs = json.loads(json.dumps(dict(request.request_config), default=dict))
    coll = docs["sketch"]["collective"]
    coll["operator"] = "allgather"
    for key in ("reduction_op", "scale", "root"):
        coll.pop(key, None)
    hyper = docs["sketch"]["hyperparameters"]
    hyper["total_size_bytes"] = request.hyperparameters.total_size_bytes // p
    hyper["slice_size_bytes"] = request.hyperparameters.slice_size_bytes
    hyper.pop("reference_slice_size_bytes", None)
    return resolve_documents(docs, purpose=request.purpose)


def synthesize_reduce_scatter_dual(request, model=None, *, channels: int = 1) -> CandidateBundle:
    """A ReduceScatter candidate made by reversing the AllGather schedule of the same slices.

    The AllGather is synthesized for the same topology, slice size and
    method; every broadcast tree is reversed into a reduction tree
    (``composer/dual.py``); the result is lowered, checked and predicted
    like any ReduceScatter candidate.
    """
    from vericcl_b200.composer.dual import reverse_allgather
    if request.collective.kind.value != "reduce_scatter":
        raise SemanticError("the AllGather dual builds ReduceScatter candidates only")
    topology = load_topology(request)
    # the AllGather's own cost context (no reduction); routes come from the topology, and the reversed
    # schedule is predicted under ``model`` below
    ag = synthesize(allgather_request_for(request), None, channels=channels)
    network = reverse_allgather(ag.network, topology, origin="dual:" + ag.origin)
    return lower_candidate(request, topology, network, model, origin="allgather_dual")


def synthesize_allreduce_rs_ag(request, model=None, *, channels: int = 1) -> CandidateBundle:
    """An AllReduce candidate: the reversed AllGather schedule (a ReduceScatter) then the AllGather itself."""
    from vericcl_b200.composer.dual import allreduce_from_allgather
    if request.collective.kind.value != "allreduce":
        raise SemanticError("the ReduceScatter + AllGather composition builds AllReduce candidates only")
    topology = load_topology(request)
    ag = synthesize(allgather_request_for(request), None, channels=channels)
    network = allreduce_from_allgather(ag.network, topology, origin="rs_ag:" + ag.origin)
    return lower_candidate(request, topology, network, model, origin="reduce_scatter_allgather")


@lru_cache(maxsize=256)
def schedule_xml(collective: str, ranks: int, slices_per_rank: int, *, inplace: bool = False,
                 datatype: str = "float32", method: str = "hierarchy", channels: int = 1, root: int = 0) -> str:
    """Verified XML for ``collective`` over ``ranks`` GPUs of one NVSwitch domain.

    The XML is size independent (its chunks scale with the runtime buffer);
    the request uses a nominal 64 KiB slice so the partition is exact.
    """
    from vericcl_b200.examples import example_documents
    from vericcl_b200.input.loader import resolve_documents
    elem = {"float32": 4, "bfloat16": 2, "float16": 2}.get(datatype, 4)
    slice_bytes = 64 * 1024 // elem * elem
    docs = example_documents(collective, method, ranks, total_size_bytes=slice_bytes * slices_per_rank,
                             slice_size_bytes=slice_bytes, datatype=datatype, inplace=inplace,
                             max_channels=channels, scratch_bytes=slice_bytes * slices_per_rank * ranks,
                             root=root)
    request = resolve_documents(docs)
    # the runtime path skips the timing MILP: on one NVSwitch domain it never beat the list schedule's
    # T_pred (every link is uncontended and the ports are shared symmetrically) and costs seconds per shape
    bundle = synthesize(request, channels=channels, timing=False)
    if not bundle.can_execute:
        failed = {k: v for k, v in bundle.checks.items() if v.get("status") not in ("valid", "not_run")}
        raise SemanticError("synthesized schedule failed admission checks: %s" % failed)
    return bundle.xml


class Lowerer:
    """Callable that lowers, checks and predicts network candidates under one model."""

    def __init__(self, request, topology, model):
        self.request = request
        self.topology = topology
        self.model = model

    def __call__(self, network) -> CandidateBundle:
        return lower_candidate(self.request, self.topology, network, self.model, origin=network.origin)
