"""Property tests: random topologies and collectives through synthesis, checks, the chunk
simulator, the device compiler and the CPU interpreter."""
import numpy as np
from hypothesis import HealthCheck, given, settings, strategies as st

from vericcl_b200.examples import example_documents
from vericcl_b200.input.loader import resolve_documents
from vericcl_b200.program.device import compile_xml, run_cpu
from vericcl_b200.program.xmlio import canonical_xml, emit_xml, parse_xml
from vericcl_b200.synthesis import synthesize
from vericcl_b200.topology.nvswitch import nvswitch_topology
from vericcl_b200.verification.chunksim import check_program_numerics, reference_result


def _ring_plus(p, extra, rng_seed):
    """A topology with a bidirectional ring plus random extra links (always strongly connected)."""
    doc = nvswitch_topology(p, nvls=False)
    rng = np.random.default_rng(rng_seed)
    keep = set()
    for r in range(p):
        keep.add((r, (r + 1) % p))
        keep.add(((r + 1) % p, r))
    pairs = [(a, b) for a in range(p) for b in range(p) if a != b and (a, b) not in keep]
    rng.shuffle(pairs)
    keep.update(pairs[:extra])
    doc["directed_links"] = [e for e in doc["directed_links"] if (e["src"], e["dst"]) in keep]
    for e in doc["directed_links"]:
        e["beta_us_per_byte"] *= float(rng.uniform(1.0, 3.0))
    for res in doc["shared_resources"]:
        res["links"] = [l for l in res["links"] if tuple(l) in keep]
    doc["shared_resources"] = [r for r in doc["shared_resources"] if r["links"]]
    valid = {r["id"] for r in doc["shared_resources"]}
    for e in doc["directed_links"]:
        e["resources"] = [x for x in e["resources"] if x in valid]
    return doc


@settings(max_examples=25, deadline=None, suppress_health_check=[HealthCheck.too_slow])
@given(p=st.integers(2, 6), extra=st.integers(0, 12), seed=st.integers(0, 1000),
       op=st.sampled_from(["allreduce", "allgather", "reduce_scatter", "broadcast"]),
       method=st.sampled_from(["hierarchy", "constructive_trees"]), inplace=st.booleans(),
       lanes=st.integers(1, 3), iters=st.integers(1, 2))
def test_random_topology_end_to_end(p, extra, seed, op, method, inplace, lanes, iters):
    if op == "broadcast":
        inplace = False
    topo = _ring_plus(p, extra, seed)
    d = example_documents(op, method, p, total_size_bytes=p * 128, slice_size_bytes=128, inplace=inplace,
                          topology=topo, per_model_timeout_s=10)
    req = resolve_documents(d)
    bundle = synthesize(req)
    assert bundle.can_execute, bundle.checks
    count = p * 32
    ok, err = check_program_numerics(parse_xml(bundle.xml), count_per_rank=count, seed=seed)
    assert ok, err
    assert canonical_xml(emit_xml(parse_xml(bundle.xml))) == canonical_xml(bundle.xml)
    compiled = compile_xml(bundle.xml, nlanes=lanes, niters=iters)
    rng = np.random.default_rng(seed)
    ins = [rng.uniform(-1, 1, count).astype(np.float32) for _ in range(p)]
    exp = reference_result(op, [a.astype(np.float64) for a in ins], rank_count=p)
    outs = run_cpu(compiled, ins, seed=seed)
    for r in range(p):
        if exp[r] is not None:
            np.testing.assert_allclose(outs[r][:len(exp[r])], exp[r], atol=1e-5)


def _ancestors(instructions):
    """Operation id -> every operation it transitively depends on."""
    by_id = {i.operation_id: i for i in instructions}
    memo = {}

    def up(key):
        if key not in memo:
            memo[key] = set()
            for d in by_id[key].dependencies:
                if d in by_id:
                    memo[key] |= {d} | up(d)
        return memo[key]

    for key in by_id:
        up(key)
    return memo


@settings(max_examples=25, deadline=None, suppress_health_check=[HealthCheck.too_slow])
@given(p=st.integers(2, 6), extra=st.integers(0, 12), seed=st.integers(0, 1000),
       op=st.sampled_from(["allreduce", "allgather", "reduce_scatter"]), inplace=st.booleans(),
       scratch_slots=st.integers(1, 4))
def test_storage_plan_never_overwrites_a_live_value(p, extra, seed, op, inplace, scratch_slots):
    """Two values that share an address never overlap in time: every reader of the earlier one is an
    ancestor of the later one's producer (reads and writes alike ordered by the dependency DAG)."""
    from vericcl_b200.errors import ScratchBudgetError
    from vericcl_b200.program.storage import build_storage_plan
    topo = _ring_plus(p, extra, seed)
    d = example_documents(op, "hierarchy", p, total_size_bytes=p * 128, slice_size_bytes=128, inplace=inplace,
                          topology=topo, per_model_timeout_s=10, scratch_bytes=128 * scratch_slots)
    req = resolve_documents(d)
    try:
        bundle = synthesize(req, timing=False)
    except ScratchBudgetError:
        return                      # the budget is too small for this schedule: refused, never overwritten
    plan = build_storage_plan(bundle.network, req)
    anc = _ancestors(plan.instructions)
    readers = {}
    for ins in plan.instructions:
        for v in ins.inputs:
            readers.setdefault(v, set()).add(ins.operation_id)
    by_addr = {}
    for state, addr in plan.addresses.items():
        by_addr.setdefault((addr.rank, addr.buffer, addr.offset), []).append(state)

    def dead_before(u, w):
        """Every read of u (and u's own write) happens before w is written."""
        pw = plan.values[w].producer
        if pw is None:
            return False            # an initial value is there from the start
        before = anc[pw] | {pw}
        pu = plan.values[u].producer
        return (pu is None or pu in anc[pw]) and all(r in before for r in readers.get(u, ()))

    for states in by_addr.values():
        for i, u in enumerate(states):
            for w in states[i + 1:]:
                assert dead_before(u, w) or dead_before(w, u), (u, w)
