"""Manual stage plans (``atom.manual``): generated from an automatic plan, edited, synthesized and checked."""
import json

import pytest

from vericcl_b200.cli.main import main as cli_main
from vericcl_b200.errors import InputValidationError
from vericcl_b200.examples import example_documents, write_documents
from vericcl_b200.input.loader import load_request
from vericcl_b200.planner.manual import plan_manual
from vericcl_b200.program.xmlio import parse_xml
from vericcl_b200.synthesis import synthesize
from vericcl_b200.topology import load_topology
from vericcl_b200.topology.nvswitch import grouped_topology
from vericcl_b200.verification.chunksim import check_program_numerics


def _inputs(tmp_path, coll, ranks=4, slices=1, topology=None):
    s = 4096
    docs = example_documents(coll, "hierarchy", ranks, total_size_bytes=s * slices * (ranks if coll != "allgather"
                                                                                       else 1),
                             slice_size_bytes=s, topology=topology, scratch_bytes=s * slices * ranks * ranks)
    return write_documents(tmp_path / "in", docs)


def _generate(tmp_path, files, source="direct"):
    argv = ["manual-generate", "--out", str(tmp_path / "manual"), "--from", source]
    for name, path in files.items():
        argv += ["--" + name, str(path)]
    assert cli_main(argv) == 0
    return {name: tmp_path / "manual" / (name + ".json") for name in files}


@pytest.mark.parametrize("coll,source", [("allreduce", "direct"), ("allgather", "direct"),
                                         ("allreduce", "hierarchy"), ("reduce_scatter", "direct")])
def test_generated_manual_plan_synthesizes_a_correct_schedule(tmp_path, capsys, coll, source):
    topo_doc = grouped_topology([2, 2]) if source == "hierarchy" else None
    files = _generate(tmp_path, _inputs(tmp_path, coll, topology=topo_doc), source)
    out = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    assert out["nodes"] == out["planned_nodes"] > 0
    atom = json.loads(files["atom"].read_text())
    assert atom["manual"]["enabled"] and len(atom["manual"]["nodes"]) == out["nodes"]
    request = load_request(files)
    topology = load_topology(request)
    plan = plan_manual(request, topology)
    assert plan.reason == "manual"
    bundle = synthesize(request)
    assert bundle.can_execute, bundle.checks
    ok, err = check_program_numerics(parse_xml(bundle.xml), count_per_rank=request.rank_count * 64, seed=3)
    assert ok, err


def test_atoms_forbid_the_named_edges(tmp_path):
    files = _generate(tmp_path, _inputs(tmp_path, "allgather"))
    atom = json.loads(files["atom"].read_text())
    node = atom["manual"]["nodes"][0]
    # forbid the broadcast root's direct edge to one member: the node must relay around it
    root = node["root"]
    target = [r for r in node["group"] if r != root][0]
    node["atoms"] = [{"slice_ids": sorted({s["offset"] for s in node["input_states"]}), "src_ranks": [root],
                      "dst_ranks": [target]}]
    files["atom"].write_text(json.dumps(atom))
    request = load_request(files)
    plan = plan_manual(request, load_topology(request))
    first = [n for n in plan.nodes if n.node_id == node["id"]][0]
    assert first.forbidden_edges and all(a == root and b == target for _, a, b in first.forbidden_edges)
    bundle = synthesize(request)
    assert bundle.can_execute, bundle.checks
    ok, err = check_program_numerics(parse_xml(bundle.xml), count_per_rank=request.rank_count * 64, seed=5)
    assert ok, err
    # the node's data reaches `target` through a relay, never over the forbidden edge
    carried = {c for st in node["input_states"] for c in st["contributors"]}
    direct = [op for op in bundle.network.operations
              if (op.src_rank, op.dst_rank) == (root, target) and set(op.contributors) & carried]
    assert not direct
    assert any(op.dst_rank == target and set(op.contributors) & carried for op in bundle.network.operations)


@pytest.mark.parametrize("edit,message", [
    (lambda n, nodes: n.update(group=[0, 1, 9]), "outside the task"),
    (lambda n, nodes: n.update(relay_ranks=[n["group"][0], 99]), "relay ranks"),
    (lambda n, nodes: n.update(depends_on=["no-such-node"]), "unknown node"),
    (lambda n, nodes: n.pop("output_states"), "input_states and output_states"),
])
def test_invalid_manual_nodes_are_refused(tmp_path, edit, message):
    files = _generate(tmp_path, _inputs(tmp_path, "allreduce"))
    atom = json.loads(files["atom"].read_text())
    edit(atom["manual"]["nodes"][0], atom["manual"]["nodes"])
    files["atom"].write_text(json.dumps(atom))
    with pytest.raises(InputValidationError, match=message):
        request = load_request(files)
        plan_manual(request, load_topology(request))


def test_vericcl_module_alias_runs_the_same_cli(tmp_path):
    """``python -m vericcl`` (the reference's module name) answers with the same commands."""
    import os
    import subprocess
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    proc = subprocess.run([sys.executable, "-m", "vericcl", "--help"], cwd=root, capture_output=True, text=True,
                          timeout=120)
    assert proc.returncode == 0
    for verb in ("solve", "verify", "calibrate", "inspect", "resume", "manual-generate"):
        assert verb in proc.stdout
