"""AllGather → ReduceScatter duality (vericcl_b200/composer/dual.py)."""
import pytest

from vericcl_b200.composer.dual import reverse_allgather
from vericcl_b200.errors import SemanticError
from vericcl_b200.examples import example_documents
from vericcl_b200.input.loader import resolve_documents
from vericcl_b200.program.xmlio import parse_xml
from vericcl_b200.synthesis import synthesize, synthesize_reduce_scatter_dual
from vericcl_b200.topology import load_topology
from vericcl_b200.topology.nvswitch import multinode_topology
from vericcl_b200.verification.chunksim import check_program_numerics


@pytest.mark.parametrize("p,method,groups", [(4, "hierarchy", 1), (4, "constructive_trees", 1), (8, "hierarchy", 2)])
def test_reversed_allgather_is_a_valid_reduce_scatter(p, method, groups):
    s, q = 1024, 2
    topo = multinode_topology(groups, p // groups, inter_gbps=25.0) if groups > 1 else None
    rs = resolve_documents(example_documents("reduce_scatter", method, p, total_size_bytes=p * q * s,
                                             slice_size_bytes=s, topology=topo, scale=0.5))
    bundle = synthesize_reduce_scatter_dual(rs)
    assert bundle.can_execute, bundle.checks
    assert bundle.origin == "allgather_dual"
    ok, err = check_program_numerics(parse_xml(bundle.xml), count_per_rank=p * q * 16, seed=2)
    assert ok, err
    direct = synthesize(rs)
    # on one NVSwitch both reach the same time; across two groups the reversed hierarchy wins
    assert bundle.t_pred_us <= direct.t_pred_us + 1e-9


def test_reversal_keeps_links_and_channels():
    p, s, q = 4, 1024, 2
    ag = synthesize(resolve_documents(example_documents("allgather", "hierarchy", p, total_size_bytes=q * s,
                                                        slice_size_bytes=s)))
    rs = resolve_documents(example_documents("reduce_scatter", "hierarchy", p, total_size_bytes=p * q * s,
                                             slice_size_bytes=s))
    dual = reverse_allgather(ag.network, load_topology(rs))
    fwd = sorted((op.src_rank, op.dst_rank, op.channel) for op in ag.network.operations)
    back = sorted((op.dst_rank, op.src_rank, op.channel) for op in dual.operations)
    assert fwd == back and all(op.kind == "rrc" for op in dual.operations)
    assert dual.slice_count == p * q


def test_non_tree_schedules_are_refused():
    from dataclasses import replace
    p, s, q = 4, 1024, 1
    ag = synthesize(resolve_documents(example_documents("allgather", "hierarchy", p, total_size_bytes=q * s,
                                                        slice_size_bytes=s)))
    rs = resolve_documents(example_documents("reduce_scatter", "hierarchy", p, total_size_bytes=p * s,
                                             slice_size_bytes=s))
    ops = list(ag.network.operations)
    broken = replace(ag.network, operations=tuple(ops[1:]))
    with pytest.raises(SemanticError):
        reverse_allgather(broken, load_topology(rs))


def test_workflow_offers_the_dual_candidate(tmp_path):
    from vericcl_b200.cli.main import main
    from vericcl_b200.examples import write_documents
    import json
    docs = example_documents("reduce_scatter", "hierarchy", 8, total_size_bytes=8 * 2 * 1024, slice_size_bytes=1024,
                             topology=multinode_topology(2, 4, inter_gbps=25.0), calibration=False)
    write_documents(tmp_path / "in", docs)
    args = ["solve", "--project-root", str(tmp_path), "--case", "d", "--run-id", "s"]
    for k in ("topology", "sketch", "atom", "runtime"):
        args += ["--" + k, str(tmp_path / "in" / (k + ".json"))]
    assert main(args) == 0
    meta = json.loads((tmp_path / "examples" / "d" / "output" / "s" / "run.json").read_text())
    assert meta["best"]["origin"] == "allgather_dual"


@pytest.mark.parametrize("groups,p", [(1, 4), (2, 8)])
def test_allreduce_from_reduce_scatter_then_allgather(groups, p):
    from vericcl_b200.synthesis import synthesize_allreduce_rs_ag
    s, q = 1024, 2
    topo = multinode_topology(groups, p // groups, inter_gbps=25.0) if groups > 1 else None
    ar = resolve_documents(example_documents("allreduce", "hierarchy", p, total_size_bytes=p * q * s,
                                             slice_size_bytes=s, topology=topo, scale=0.25))
    bundle = synthesize_allreduce_rs_ag(ar)
    assert bundle.can_execute, bundle.checks
    ok, err = check_program_numerics(parse_xml(bundle.xml), count_per_rank=p * q * 16, seed=5)
    assert ok, err
    kinds = [op.kind for op in bundle.network.operations]
    assert kinds.count("rrc") == kinds.count("send") > 0


@pytest.mark.parametrize("groups,p", [(1, 4), (2, 8)])
def test_reduce_scatter_reverses_into_an_allgather_and_round_trips(groups, p):
    from vericcl_b200.composer.dual import reverse_reduce_scatter
    from vericcl_b200.performance.initial import initial_cost_model
    from vericcl_b200.synthesis import Lowerer
    s, q = 1024, 2
    topo_doc = multinode_topology(groups, p // groups, inter_gbps=25.0) if groups > 1 else None
    ag_req = resolve_documents(example_documents("allgather", "hierarchy", p, total_size_bytes=q * s,
                                                 slice_size_bytes=s, topology=topo_doc))
    rs_req = resolve_documents(example_documents("reduce_scatter", "hierarchy", p, total_size_bytes=p * q * s,
                                                 slice_size_bytes=s, topology=topo_doc))
    topo = load_topology(ag_req)
    rs = synthesize(rs_req)
    back = Lowerer(ag_req, topo, initial_cost_model(ag_req))(reverse_reduce_scatter(rs.network, topo))
    assert back.can_execute, back.checks
    ok, err = check_program_numerics(parse_xml(back.xml), count_per_rank=q * 16, seed=3)
    assert ok, err
    # AllGather → ReduceScatter → AllGather keeps every edge and channel
    ag = synthesize(ag_req)
    again = reverse_reduce_scatter(reverse_allgather(ag.network, load_topology(rs_req)), topo)
    key = lambda ops: sorted((o.src_rank, o.dst_rank, o.channel, min(o.contributors)) for o in ops)
    assert key(again.operations) == key(ag.network.operations)


def test_reduce_scatter_cycle_among_non_owners_is_refused():
    """Two non-owner ranks that reduce a slice into each other never reach the owner."""
    from dataclasses import replace
    from vericcl_b200.composer.dual import reverse_reduce_scatter
    p, s = 4, 1024
    req = resolve_documents(example_documents("reduce_scatter", "hierarchy", p, total_size_bytes=p * s,
                                              slice_size_bytes=s))
    rs = synthesize(req).network
    ops = list(rs.operations)
    # slice 0 is owned by rank 0; send rank 1's and rank 2's contributions to each other instead
    for i, op in enumerate(ops):
        if op.index == 0 and op.src_rank in (1, 2):
            ops[i] = replace(op, dst_rank=2 if op.src_rank == 1 else 1)
    with pytest.raises(SemanticError, match="not connected to its owner"):
        reverse_reduce_scatter(replace(rs, operations=tuple(ops)), load_topology(req))
