"""Hierarchy search (vericcl_b200/planner/group_search.py): partitions, rails, gateway plans, streaming."""
import pytest

from vericcl_b200.composer import compose_routes
from vericcl_b200.examples import example_documents
from vericcl_b200.input.loader import resolve_documents
from vericcl_b200.planner.group_search import (CandidateStream, discover_rails, gateway_rails,
                                               partition_candidates)
from vericcl_b200.program.xmlio import parse_xml
from vericcl_b200.solver.demands import build_demands
from vericcl_b200.solver.routing import choose_trees
from vericcl_b200.synthesis import lower_candidate, synthesize
from vericcl_b200.topology import load_topology
from vericcl_b200.topology.nvswitch import grouped_topology, multinode_topology
from vericcl_b200.verification.chunksim import check_program_numerics

S = 16 * 1024


def _request(coll, topo_doc, slices, ranks):
    docs = example_documents(coll, "hierarchy", ranks, total_size_bytes=S * slices, slice_size_bytes=S,
                             datatype="float32", scratch_bytes=S * slices * ranks, topology=topo_doc)
    return resolve_documents(docs)


def _lower(req, topo, plan):
    demands = build_demands(plan, topo)
    trees = choose_trees(demands, topo, S)
    net = compose_routes(plan, demands, trees, topo, S, origin="hierarchy")
    return lower_candidate(req, topo, net, plan=plan)


@pytest.mark.parametrize("coll,slices", [("allreduce", 8), ("allgather", 1)])
@pytest.mark.parametrize("sizes", [(5, 3), (3, 3, 2)])
def test_unequal_groups_give_valid_plans_of_both_families(coll, slices, sizes):
    ranks = sum(sizes)
    req = _request(coll, grouped_topology(list(sizes)), slices, ranks)
    topo = load_topology(req)
    assert sorted(len(g) for g in partition_candidates(topo)[0]) == sorted(sizes)
    modes, runnable = set(), 0
    for plan in CandidateStream(req, topo):
        modes.add(plan.metadata["rail_mode"])
        bundle = _lower(req, topo, plan)
        failed = {k: v for k, v in bundle.checks.items() if v.get("status") not in ("valid", "not_run")}
        # the schedule itself is always correct; the device compiler may still refuse a merged order
        # whose cross-rank waits form a cycle (then the workflow drops the candidate)
        assert set(failed) <= {"compatibility"}, failed
        runnable += bundle.can_execute
        per_rank = (slices if coll == "allreduce" else 1) * 16
        ok, err = check_program_numerics(parse_xml(bundle.xml), count_per_rank=per_rank, seed=5)
        assert ok, err
    assert modes == {"rails", "gateways"} and runnable >= 1


def test_rails_follow_the_cheap_links():
    """Only ranks 3 and 4 own the inter-group links: every rail must cross through them."""
    doc = grouped_topology([4, 4], gateways=[[3], [4]])
    req = _request("allreduce", doc, 8, 8)
    topo = load_topology(req)
    groups = partition_candidates(topo)[0]
    rails = discover_rails(topo, groups, range(8))
    for owner, members in rails.items():
        other = members[1] if owner < 4 else members[0]
        assert other == (4 if owner < 4 else 3)
    assert gateway_rails(topo, groups, range(8))[0] == (3, 4)


def test_stream_yields_plans_in_coarse_score_order_and_the_workflow_uses_the_best():
    req = _request("allgather", multinode_topology(2, 4, inter_gbps=25.0), 1, 8)
    topo = load_topology(req)
    scores = [plan.metadata["coarse_score_us"] for plan in CandidateStream(req, topo)]
    assert scores == sorted(scores) and len(scores) == 2
    bundle = synthesize(req, timing=False)
    assert "rails" in bundle.plan.reason


def test_partitions_of_a_three_level_topology():
    """Two cost levels inside the box (fast pairs, slower quads) and a slow inter-group link give nested partitions."""
    doc = grouped_topology([4, 4], inter_gbps=25.0)
    for edge in doc["directed_links"]:
        same_pair = edge["src"] // 2 == edge["dst"] // 2
        same_quad = edge["src"] // 4 == edge["dst"] // 4
        if same_quad and not same_pair:
            edge["beta_us_per_byte"] *= 2
    req = _request("allreduce", doc, 8, 8)
    parts = partition_candidates(load_topology(req))
    assert ((0, 1, 2, 3), (4, 5, 6, 7)) in parts
    assert ((0, 1), (2, 3), (4, 5), (6, 7)) in parts


def test_resynthesis_offers_the_other_groupings_of_the_hierarchy():
    from vericcl_b200.tuning.resynthesis import branches, resynthesize_branch
    from vericcl_b200.performance.initial import initial_cost_model
    req = _request("allreduce", multinode_topology(2, 4, inter_gbps=25.0), 8, 8)
    bundle = synthesize(req, timing=False)
    alts = [b for b in branches(req, bundle) if b.plan_reason is not None]
    assert alts and all(b.plan_reason != bundle.plan.reason for b in alts)
    other = resynthesize_branch(req, alts[0], initial_cost_model(req))
    assert other is not None and other.can_execute and other.plan.reason == alts[0].plan_reason
