"""Schedule sidecar (``schedule.json``, schema 5): everything verify needs.

The XML holds the native program; the sidecar adds what the XML cannot
express: the slice partition, the logical values (contributor sets) with
their producers, the slot addresses, the instruction dependency graph and
channels, the origin of the candidate and the model context it was predicted
under.  ``bundle_from_sidecar`` rebuilds a candidate bundle from XML +
sidecar and re-runs the eight checks and the exact prediction (reference:
vericcl/xml/v5_lower.py:327-359).
"""
from __future__ import annotations

from vericcl_b200.errors import SemanticError
from vericcl_b200.program.model import Address, Instruction, StoragePlan, Value
from vericcl_b200.utils.hashing import sha256_hex

SIDECAR_SCHEMA = 5


def to_sidecar(bundle) -> dict:
    st = bundle.storage
    req = bundle.request
    return {
        "schema_version": SIDECAR_SCHEMA,
        "xml_sha256": sha256_hex(bundle.xml),
        "origin": bundle.origin,
        "collective": {"operator": req.collective.kind.value, "datatype": req.collective.datatype,
                       "reduction_op": req.collective.reduction_op, "root": req.collective.root,
                       "inplace": req.collective.inplace},
        "partition": {"total_size_bytes": req.hyperparameters.total_size_bytes,
                      "slice_size_bytes": req.hyperparameters.slice_size_bytes,
                      "slice_count": req.hyperparameters.slice_count, "rank_count": req.rank_count},
        "values": [{"id": v.state_id, "rank": v.rank, "index": v.index, "contributors": sorted(v.contributors),
                    "producer": v.producer} for v in st.values.values()],
        "initial": list(st.initial_ids),
        "addresses": {k: [a.rank, a.buffer, a.offset] for k, a in st.addresses.items()},
        "instructions": [{"id": i.operation_id, "kind": i.kind, "inputs": list(i.inputs), "output": i.output,
                          "rank": i.rank, "peer": i.peer, "channel": i.channel, "stage": i.stage_id,
                          "dependencies": sorted(i.dependencies), "priority": i.priority_time}
                         for i in st.instructions],
        "outputs": [[slot.rank, slot.offset, sid] for slot, sid in st.outputs.items()],
        "slots": {"input": {str(k): v for k, v in st.input_slots.items()},
                  "output": {str(k): v for k, v in st.output_slots.items()},
                  "scratch": {str(k): v for k, v in st.scratch_slots.items()}},
        "reuse": list(st.reuse),
        "step_operations": {"%d:%d" % (b.rank, b.tb_id): [x.operation_id for x in b.steps]
                            for b in bundle.program.blocks},
        "prediction": None if bundle.prediction is None else {
            "t_pred_us": bundle.prediction.t_pred_us, "model_version": bundle.prediction.model_version,
            "exact_ratio": bundle.prediction.exact_completion_ratio},
        "checks": bundle.checks,
    }


def storage_from_sidecar(doc: dict) -> StoragePlan:
    from vericcl_b200.semantics.collective import OutputSlot
    if doc.get("schema_version") != SIDECAR_SCHEMA:
        raise SemanticError("unsupported sidecar schema %r" % doc.get("schema_version"))
    values = {v["id"]: Value(v["id"], v["rank"], v["index"], frozenset(v["contributors"]), v["producer"])
              for v in doc["values"]}
    addresses = {k: Address(*a) for k, a in doc["addresses"].items()}
    instructions = tuple(Instruction(i["id"], i["kind"], tuple(i["inputs"]), i["output"], i["rank"], i["peer"],
                                     i["channel"], i["stage"], frozenset(i["dependencies"]), i["priority"])
                         for i in doc["instructions"])
    outputs = {OutputSlot(r, o): sid for r, o, sid in doc["outputs"]}
    slots = doc["slots"]
    conv = lambda d: {int(k): v for k, v in d.items()}
    return StoragePlan(values, tuple(doc["initial"]), instructions, addresses, outputs, conv(slots["input"]),
                       conv(slots["output"]), conv(slots["scratch"]), tuple(doc.get("reuse", ())))


def attach_operations(program, doc):
    """Give parsed XML steps the operation identities recorded in the sidecar."""
    from dataclasses import replace
    ops = doc.get("step_operations", {})
    blocks = []
    for b in program.blocks:
        ids = ops.get("%d:%d" % (b.rank, b.tb_id))
        if ids is None or len(ids) != len(b.steps):
            raise SemanticError("sidecar does not describe TB %d of rank %d" % (b.tb_id, b.rank))
        blocks.append(replace(b, steps=tuple(replace(s, operation_id=i) for s, i in zip(b.steps, ids))))
    return replace(program, blocks=tuple(blocks))


def bundle_from_sidecar(request, topology, xml: str, doc: dict, model=None):
    from vericcl_b200.performance.initial import initial_cost_model, model_context
    from vericcl_b200.performance.simulation import predict
    from vericcl_b200.planner.parameters import bind_artifact_partition
    from vericcl_b200.program.checks import evaluate_program
    from vericcl_b200.program.native import build_executable
    from vericcl_b200.program.xmlio import parse_xml
    from vericcl_b200.synthesis import CandidateBundle
    if sha256_hex(xml) != doc["xml_sha256"]:
        raise SemanticError("sidecar was written for a different XML")
    request = bind_artifact_partition(request, doc["partition"]["slice_size_bytes"])
    storage = storage_from_sidecar(doc)
    program = attach_operations(parse_xml(xml), doc)
    model = model or initial_cost_model(request)
    executable = build_executable(program, storage, request, topology, model_context(request))
    prediction = predict(executable, model, exact=True)
    bundle = CandidateBundle(request, None, None, storage, program, xml, executable, prediction,
                             origin=doc.get("origin", "verify"))
    bundle.checks = evaluate_program(bundle, topology)
    return bundle
