"""Global channel assignment (vericcl_b200/solver/global_scheduler.py)."""
from vericcl_b200.composer import compose_routes
from vericcl_b200.examples import example_documents
from vericcl_b200.input.loader import resolve_documents
from vericcl_b200.program.xmlio import parse_xml
from vericcl_b200.solver.demands import build_demands
from vericcl_b200.solver.global_scheduler import assign_channels
from vericcl_b200.solver.routing import choose_trees
from vericcl_b200.synthesis import lower_candidate, plan_for, synthesize
from vericcl_b200.topology import load_topology
from vericcl_b200.verification.chunksim import check_program_numerics


def _network(coll, ranks, slices, channels):
    s = 4096
    d = example_documents(coll, "hierarchy", ranks, total_size_bytes=s * slices, slice_size_bytes=s,
                          max_channels=channels, scratch_bytes=s * slices * ranks)
    req = resolve_documents(d)
    topo = load_topology(req)
    plan = plan_for(req, topo)
    dem = build_demands(plan, topo, s)
    net = compose_routes(plan, dem, choose_trees(dem, topo, s), topo, s, channels=channels, origin="direct")
    return req, topo, net


def test_channels_balance_and_the_schedule_stays_correct():
    req, topo, net = _network("allreduce", 4, 16, 4)
    glob = assign_channels(net, topo, 4)
    assert glob.origin.endswith("+channels")
    per_conn = {}
    for op in glob.operations:
        assert 0 <= op.channel < 4
        per_conn.setdefault((op.src_rank, op.dst_rank), []).append(op.channel)
    for chans in per_conn.values():
        counts = [chans.count(c) for c in set(chans)]
        assert max(counts) - min(counts) <= max(2, len(chans) // 4)
    a = lower_candidate(req, topo, net)
    b = lower_candidate(req, topo, glob)
    assert b.can_execute, b.checks
    ok, err = check_program_numerics(parse_xml(b.xml), count_per_rank=16 * 16, seed=4)
    assert ok, err
    assert b.t_pred_us <= a.t_pred_us * 1.05


def test_one_channel_is_left_alone_and_synthesis_keeps_the_better_assignment():
    req, topo, net = _network("allgather", 4, 2, 1)
    assert assign_channels(net, topo, 1) is net
    d = example_documents("allreduce", "hierarchy", 4, total_size_bytes=4096 * 16, slice_size_bytes=4096,
                          max_channels=4, scratch_bytes=4096 * 16 * 4)
    bundle = synthesize(resolve_documents(d), channels=4, timing=False)
    assert bundle.can_execute


def _blocks(candidate):
    blocks = {}
    for op in candidate.operations:
        blocks.setdefault(op.src_rank, set()).add((op.dst_rank, "send", op.channel))
        blocks.setdefault(op.dst_rank, set()).add((op.src_rank, "recv", op.channel))
    return blocks


def test_the_thread_block_budget_per_rank_holds():
    req, topo, net = _network("allreduce", 4, 16, 4)
    roomy = _blocks(assign_channels(net, topo, 4))
    assert max(len(b) for b in roomy.values()) > 8                 # without a budget the links use several channels
    capped = assign_channels(net, topo, 4, max_blocks_per_rank=8)
    assert max(len(b) for b in _blocks(capped).values()) <= 8
    b = lower_candidate(req, topo, capped)
    assert b.can_execute, b.checks
    ok, err = check_program_numerics(parse_xml(b.xml), count_per_rank=16 * 16, seed=5)
    assert ok, err


def test_a_budget_below_one_block_per_connection_gives_each_connection_one():
    _, topo, net = _network("allreduce", 4, 16, 4)
    capped = assign_channels(net, topo, 4, max_blocks_per_rank=2)
    blocks = _blocks(capped)
    # each rank talks to 3 peers both ways: 6 blocks is the least any assignment can use
    assert all(len(b) == 6 for b in blocks.values())
