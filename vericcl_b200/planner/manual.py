"""Manual stage plans from ``atom.manual.nodes``.

Each manual node names a stage, a local collective, a group, optional relay
ranks, dependencies and optional input/output state contracts
(``{rank, offset, contributors}``).  When contracts are omitted they are
derived from the collective semantics of the node over its group.  Atom
variable groups become forbidden directed edges bound to original slice ids
(reference: vericcl/planner/manual.py:11 and README "manual-generate").
"""
from __future__ import annotations

from vericcl_b200.errors import InputValidationError
from vericcl_b200.planner.model import PlanDAG, PlanEdge, PlanNode, PlanningMode, StageInterface
from vericcl_b200.semantics.collective import CollectiveKind, OutputSlot

REDUCING = {CollectiveKind.REDUCE, CollectiveKind.REDUCE_SCATTER, CollectiveKind.ALL_REDUCE}


def _states(items):
    return StageInterface({OutputSlot(s["rank"], s["offset"]): frozenset(s["contributors"]) for s in items})


def plan_manual(request, topology) -> PlanDAG:
    atom = request.request_config["atom"]
    if not atom["manual"]["enabled"]:
        raise InputValidationError("atom.manual.enabled is false")
    p = request.rank_count
    n = request.hyperparameters.slice_count
    nodes, edges = [], []
    ids = set()
    for item in atom["manual"]["nodes"]:
        kind = CollectiveKind(item["operator"])
        group = tuple(item["group"])
        if not set(group) <= set(range(p)):
            raise InputValidationError("manual node %s uses a rank outside the task" % item["id"])
        relays = tuple(item.get("relay_ranks") or ())
        if not set(relays) <= set(group):
            raise InputValidationError("manual relay ranks must belong to the node's group")
        if "input_states" not in item or "output_states" not in item:
            raise InputValidationError("manual node %s needs input_states and output_states" % item["id"])
        forbidden = set()
        for atom_group in item.get("atoms", ()):
            for sid in atom_group["slice_ids"]:
                for a in atom_group["src_ranks"]:
                    for b in atom_group["dst_ranks"]:
                        forbidden.add((sid, a, b))
        root = item.get("root")
        inputs, outputs = _states(item["input_states"]), _states(item["output_states"])
        if root is None:
            root = min(s.rank for s in (outputs.values if kind in REDUCING else inputs.values))
        node_kind = CollectiveKind.REDUCE if kind in REDUCING else CollectiveKind.BROADCAST
        if kind in REDUCING and len(outputs.values) > 1:
            raise InputValidationError("manual reducing nodes must have one output state; split them per slot")
        nodes.append(PlanNode(item["id"], item["stage_id"], node_kind, group, root, inputs, outputs, relays,
                              frozenset(forbidden)))
        ids.add(item["id"])
    for item in atom["manual"]["nodes"]:
        for dep in item.get("depends_on", ()):
            if dep not in ids:
                raise InputValidationError("manual node %s depends on unknown node %s" % (item["id"], dep))
            edges.append(PlanEdge(dep, item["id"]))
    return PlanDAG(request.collective, p, n, tuple(nodes), tuple(edges), PlanningMode.MANUAL, "manual")


def manual_nodes_from_plan(plan: PlanDAG) -> list:
    """Editable manual-node documents for an existing plan (README manual-generate)."""
    def states(iface):
        return [{"rank": s.rank, "offset": s.offset, "contributors": sorted(v)} for s, v in iface.values.items()]
    out = []
    for node in plan.nodes:
        out.append({"id": node.node_id, "stage_id": node.stage_id, "operator": node.kind.value, "root": node.root,
                    "group": list(node.group), "relay_ranks": list(node.group),
                    "depends_on": plan.predecessors(node.node_id), "input_states": states(node.logical_input),
                    "output_states": states(node.logical_output), "atoms": []})
    return out
