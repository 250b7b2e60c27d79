import pytest

from vericcl_b200.examples import example_documents
from vericcl_b200.input.loader import resolve_documents
from vericcl_b200.program.xmlio import parse_xml
from vericcl_b200.synthesis import synthesize
from vericcl_b200.verification.chunksim import check_program_numerics

CASES = [("allreduce", False), ("allreduce", True), ("allgather", False), ("allgather", True),
         ("reduce_scatter", False), ("reduce_scatter", True), ("broadcast", False), ("reduce", False),
         ("alltoall", False)]


@pytest.mark.parametrize("op,inplace", CASES)
@pytest.mark.parametrize("ranks", [2, 4])
def test_synthesize_checks_and_numerics(op, inplace, ranks):
    slices = ranks
    d = example_documents(op, "hierarchy", ranks, total_size_bytes=slices * 256, slice_size_bytes=256,
                          inplace=inplace)
    req = resolve_documents(d)
    bundle = synthesize(req)
    assert bundle.can_execute, bundle.checks
    assert bundle.t_pred_us > 0
    ok, err = check_program_numerics(parse_xml(bundle.xml), count_per_rank=slices * 64, seed=3)
    assert ok, err


def test_allgather_p8_1mib_hierarchy_on_the_chunk_simulator():
    """P=8 AllGather, hierarchy, fp32, M=1 MiB, S=256 KiB, alpha=2us, beta=1/150 GB/s."""
    d = example_documents("allgather", "hierarchy", 8, total_size_bytes=1 << 20, slice_size_bytes=1 << 18,
                          alpha_us=2.0, link_gbps=150.0, per_model_timeout_s=60)
    req = resolve_documents(d)
    bundle = synthesize(req)
    assert bundle.can_execute, bundle.checks
    # chunk simulator on seeded uniform(-1, 1) fp32 inputs: each output is the concatenation
    ok, err = check_program_numerics(parse_xml(bundle.xml), count_per_rank=(1 << 20) // 4 // 64, seed=7,
                                     distribution="uniform", atol=0, rtol=0)
    assert ok and err == 0.0
    # alpha-beta sanity: 7 direct sends of 4 slices over one port at 150 GB/s
    assert bundle.t_pred_us > (7 * (1 << 20)) / 150e3


def test_emulated_two_groups_use_hierarchy():
    from vericcl_b200.topology.nvswitch import multinode_topology
    topo = multinode_topology(2, 4, inter_gbps=25.0)
    d = example_documents("allreduce", "hierarchy", 8, total_size_bytes=8 * 1024, slice_size_bytes=1024,
                          topology=topo)
    req = resolve_documents(d)
    bundle = synthesize(req)
    assert bundle.can_execute, bundle.checks
    assert bundle.plan.mode.value == "hierarchy"
    ok, _ = check_program_numerics(parse_xml(bundle.xml), count_per_rank=8 * 16)
    assert ok


def test_device_memory_budget_is_checked():
    d = example_documents("allgather", "hierarchy", 4, total_size_bytes=4 * 4096, slice_size_bytes=4096)
    d["runtime"]["device_memory_budget_bytes"] = 1024
    bundle = synthesize(resolve_documents(d))
    assert bundle.checks["storage"]["status"] != "valid" and "device bytes" in str(bundle.checks["storage"])
