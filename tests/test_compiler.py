import numpy as np
import pytest

from vericcl_b200.errors import SemanticError
from vericcl_b200.program.device import compile_xml, run_cpu
from vericcl_b200.synthesis import schedule_xml
from vericcl_b200.verification.chunksim import reference_result


def _run(coll, p, slices, inplace, lanes, iters, fuse, merge, dtype="float32", seed=0):
    xml = schedule_xml(coll, p, slices, inplace=inplace)
    c = compile_xml(xml, nlanes=lanes, niters=iters, fuse=fuse, merge=merge)
    count = p * slices * 8 * 3
    rng = np.random.default_rng(seed)
    ins = [rng.uniform(-1, 1, count).astype(np.float32) for _ in range(p)]
    exp = reference_result(coll, [a.astype(np.float64) for a in ins], rank_count=p)
    outs = run_cpu(c, ins, seed=seed, dtype=dtype)
    tol = 1e-5 if dtype == "float32" else 2e-2 * p
    for r in range(p):
        if exp[r] is not None:
            np.testing.assert_allclose(outs[r][:len(exp[r])], exp[r], atol=tol)
    return c


@pytest.mark.parametrize("coll", ["allreduce", "allgather", "reduce_scatter"])
@pytest.mark.parametrize("inplace", [False, True])
@pytest.mark.parametrize("lanes,iters,fuse,merge", [(1, 1, False, False), (3, 2, True, True), (2, 3, True, False)])
def test_interpreter_matches_reference(coll, inplace, lanes, iters, fuse, merge):
    for seed in range(2):
        _run(coll, 4, 4, inplace, lanes, iters, fuse, merge, seed=seed)


def test_bf16_and_fused_chain():
    c = _run("allreduce", 8, 8, True, 4, 2, True, True, dtype="bfloat16")
    assert c.stats["fused_reduces"] == 8
    assert c.max_blocks == 1


def test_scale_applied_once():
    xml = schedule_xml("allreduce", 4, 4)
    c = compile_xml(xml, nlanes=2)
    ins = [np.full(4 * 8 * 2, r + 1.0, np.float32) for r in range(4)]
    outs = run_cpu(c, ins, scale=0.25)
    np.testing.assert_allclose(outs[0], 2.5)


def test_rejects_unmatched_send():
    xml = """<algo name="x" nchannels="1" nchunksperloop="1" coll="allgather" inplace="0" ngpus="2">
      <gpu id="0" i_chunks="1" o_chunks="2" s_chunks="0">
        <tb id="0" send="1" recv="-1" chan="0"><step s="0" type="s" srcbuf="i" srcoff="0" dstbuf="o" dstoff="0" cnt="1" depid="-1" deps="-1" hasdep="0"/></tb>
      </gpu>
      <gpu id="1" i_chunks="1" o_chunks="2" s_chunks="0"></gpu></algo>"""
    with pytest.raises(SemanticError, match="receives"):
        compile_xml(xml)


def test_rejects_cyclic_schedule():
    xml = """<algo name="x" nchannels="1" nchunksperloop="2" coll="allgather" inplace="0" ngpus="2">
      <gpu id="0" i_chunks="1" o_chunks="2" s_chunks="0">
        <tb id="0" send="-1" recv="1" chan="0"><step s="0" type="r" srcbuf="o" srcoff="1" dstbuf="o" dstoff="1" cnt="1" depid="-1" deps="-1" hasdep="0"/></tb>
        <tb id="1" send="1" recv="-1" chan="0"><step s="0" type="s" srcbuf="i" srcoff="0" dstbuf="o" dstoff="0" cnt="1" depid="-1" deps="-1" hasdep="0"/></tb>
      </gpu>
      <gpu id="1" i_chunks="1" o_chunks="2" s_chunks="0">
        <tb id="0" send="0" recv="0" chan="0">
          <step s="0" type="r" srcbuf="o" srcoff="0" dstbuf="o" dstoff="0" cnt="1" depid="-1" deps="-1" hasdep="0"/>
          <step s="1" type="s" srcbuf="i" srcoff="0" dstbuf="o" dstoff="1" cnt="1" depid="-1" deps="-1" hasdep="0"/>
        </tb>
      </gpu></algo>"""
    # rank 1 receives before it sends; rank 0's receive needs rank 1's send: fine.  Make it cyclic:
    cyclic = xml.replace('<tb id="1" send="1" recv="-1" chan="0"><step s="0" type="s"',
                         '<tb id="1" send="1" recv="-1" chan="0"><step s="0" type="s"').replace(
        'type="s" srcbuf="i" srcoff="0" dstbuf="o" dstoff="0" cnt="1" depid="-1"',
        'type="s" srcbuf="i" srcoff="0" dstbuf="o" dstoff="0" cnt="1" depid="0" deps="0" hasdep="0" x="', 1)
    with pytest.raises(SemanticError):
        compile_xml(cyclic.replace(' x="', ' y="'))


def test_xml_reader_rejects_garbage():
    with pytest.raises(SemanticError):
        compile_xml("<algo ngpus='2'><gpu></algo>")


@pytest.mark.parametrize("coll,inplace", [("allreduce", True), ("allreduce", False), ("allgather", False),
                                          ("allgather", True)])
@pytest.mark.parametrize("p", [4, 8])
@pytest.mark.parametrize("lanes,iters", [(1, 1), (3, 2)])
def test_multicast_programs_match_reference(coll, inplace, p, lanes, iters):
    """NVLS-mapped programs (with idle steps removed) through the CPU oracle's multicast emulation."""
    slices = p if coll == "allreduce" else 1
    xml = schedule_xml(coll, p, slices, inplace=inplace)
    c = compile_xml(xml, nlanes=lanes, niters=iters, multicast=True)
    if not (coll == "allgather" and inplace):       # in-place AllGather has no owner copy to broadcast
        assert c.stats["multicast_ops"] > 0 and c.stats["dropped_nops"] > 0
    count = p * slices * 8 * 3
    for seed in range(2):
        rng = np.random.default_rng(seed)
        ins = [rng.uniform(-1, 1, count).astype(np.float32) for _ in range(p)]
        exp = reference_result(coll, [a.astype(np.float64) for a in ins], rank_count=p)
        outs = run_cpu(c, ins, seed=seed, launches=2 if not inplace else 1)
        for r in range(p):
            np.testing.assert_allclose(outs[r][:len(exp[r])], exp[r], atol=1e-5)


def test_idle_nops_removed_and_waits_renumbered():
    xml = schedule_xml("allreduce", 8, 8, inplace=True)
    plain = compile_xml(xml, nlanes=1)
    assert plain.stats["dropped_nops"] == 48
    text = plain.describe(0)
    assert "nop" not in text and "wait(r1,b0,e2)" in text


@pytest.mark.parametrize("coll,root", [("broadcast", 0), ("broadcast", 2), ("reduce", 0), ("reduce", 3),
                                       ("alltoall", 0)])
@pytest.mark.parametrize("lanes,iters,merge", [(1, 1, False), (3, 2, True)])
def test_rooted_and_alltoall_programs_on_the_oracle(coll, root, lanes, iters, merge):
    p = 4
    slices = p
    xml = schedule_xml(coll, p, slices, inplace=False, root=root)
    c = compile_xml(xml, nlanes=lanes, niters=iters, merge=merge)
    count = p * slices * 8 * 3
    rng = np.random.default_rng(7)
    ins = [rng.uniform(-1, 1, count).astype(np.float32) for _ in range(p)]
    exp = reference_result(coll, [a.astype(np.float64) for a in ins], rank_count=p, root=root)
    outs = run_cpu(c, ins, seed=3)
    for r in range(p):
        if exp[r] is not None:
            np.testing.assert_allclose(outs[r][:len(exp[r])], exp[r], atol=1e-5)


def test_device_blocks_must_fit_the_resident_ctas(monkeypatch):
    from vericcl_b200.examples import example_documents
    from vericcl_b200.input.loader import resolve_documents
    from vericcl_b200.program import checks
    req = resolve_documents(example_documents("allreduce", "hierarchy", 4, total_size_bytes=4 * 1024,
                                              slice_size_bytes=1024))
    from vericcl_b200.synthesis import synthesize
    bundle = synthesize(req)
    assert bundle.checks["compatibility"]["status"] == "valid"
    assert 1 <= bundle.checks["compatibility"]["detail"]["device_blocks"] <= checks.B200_RESIDENT_CTAS
    monkeypatch.setattr(checks, "B200_RESIDENT_CTAS", 0)
    from vericcl_b200.topology import load_topology
    again = checks.evaluate_program(bundle, load_topology(req))
    assert again["compatibility"]["status"] == "invalid" and "co-resident" in again["compatibility"]["detail"]


RRS_CHAIN = """<algo name="chain" nchannels="1" nchunksperloop="1" proto="Simple" coll="reduce" inplace="0" redop="sum" ngpus="3">
  <gpu id="0" i_chunks="1" o_chunks="0" s_chunks="0">
    <tb id="0" send="1" recv="-1" chan="0">
      <step s="0" type="s" srcbuf="i" srcoff="0" dstbuf="i" dstoff="0" cnt="1" depid="-1" deps="-1" hasdep="0"/>
    </tb>
  </gpu>
  <gpu id="1" i_chunks="1" o_chunks="0" s_chunks="0">
    <tb id="0" send="2" recv="0" chan="0">
      <step s="0" type="rrs" srcbuf="i" srcoff="0" dstbuf="i" dstoff="0" cnt="1" depid="-1" deps="-1" hasdep="0"/>
    </tb>
  </gpu>
  <gpu id="2" i_chunks="1" o_chunks="1" s_chunks="0">
    <tb id="0" send="-1" recv="1" chan="0">
      <step s="0" type="rrc" srcbuf="i" srcoff="0" dstbuf="o" dstoff="0" cnt="1" depid="-1" deps="-1" hasdep="0"/>
    </tb>
  </gpu>
</algo>
"""


@pytest.mark.parametrize("lanes,iters", [(1, 1), (3, 2)])
def test_reduce_and_forward_is_staged_in_scratch(lanes, iters):
    """An 'rrs' forwards a partial sum it never stores; under pulls it gets a scratch store of its own."""
    compiled = compile_xml(RRS_CHAIN, nlanes=lanes, niters=iters)
    assert compiled.stats["staged_forwards"] == 1
    assert compiled.slots(1)[2] == 1 and compiled.slots(0)[2] == 0
    rng = np.random.default_rng(4)
    inputs = [rng.standard_normal(96).astype(np.float32) for _ in range(3)]
    outs = run_cpu(compiled, inputs, seed=7)
    np.testing.assert_allclose(outs[2][:96], inputs[0] + inputs[1] + inputs[2], rtol=1e-6, atol=1e-6)


@pytest.mark.parametrize("coll", ["allgather", "allreduce", "broadcast", "alltoall"])
@pytest.mark.parametrize("p", [2, 4, 8])
@pytest.mark.parametrize("lanes,iters,merge", [(1, 1, True), (3, 2, True), (2, 1, False)])
def test_push_programs_match_reference(coll, p, lanes, iters, merge):
    """Push mode: plain transfers become stores into the receiver; the randomized oracle still finds every result."""
    inplace = coll in ("allgather", "allreduce")
    slices = p if coll in ("allreduce", "alltoall") else 1
    xml = schedule_xml(coll, p, slices, inplace=inplace)
    plan = compile_xml(xml, nlanes=lanes, niters=iters, merge=merge, push=True)
    assert plan.stats["pushes"] > 0
    pulled = compile_xml(xml, nlanes=lanes, niters=iters, merge=merge)
    assert pulled.stats["pushes"] == 0
    count = p * 16 * slices
    rng = np.random.default_rng(p + lanes)
    ins = [rng.uniform(-1, 1, count).astype(np.float32) for _ in range(p)]
    exp = reference_result(coll, [a.astype(np.float64) for a in ins], rank_count=p)
    for seed in range(3):
        outs = run_cpu(plan, ins, seed=seed)
        for r in range(p):
            if exp[r] is not None:
                np.testing.assert_allclose(outs[r][:len(exp[r])], exp[r], atol=1e-5)


def test_push_steps_write_the_receiver_and_receives_wait_for_them():
    plan = compile_xml(schedule_xml("allgather", 4, 1), push=True)
    text = plan.describe(0)
    assert "-> r1:o[" in text or "-> r1:" in text          # rank 0 stores into a peer's output
    # a push waits for the receiver's start flag (block -1 is the per-rank start flag)
    assert "wait(r1,b-1,e1)" in text or "wait(r2,b-1,e1)" in text or "wait(r3,b-1,e1)" in text
