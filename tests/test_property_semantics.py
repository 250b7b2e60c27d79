"""Property tests of the collective semantics: duality, aliasing and reproducibility."""
from hypothesis import given, settings, strategies as st

from vericcl_b200.semantics.collective import CollectiveKind, CollectiveSpec, required_outputs
from vericcl_b200.semantics.versions import canonical, initial_state, input_aliases


@settings(max_examples=60, deadline=None)
@given(p=st.integers(1, 8), q=st.integers(1, 4))
def test_allreduce_is_reduce_scatter_then_allgather(p, q):
    """AR(rank, i) gets exactly the contributors RS leaves at its owner slot, which AG then copies everywhere."""
    n = p * q
    ar = required_outputs(CollectiveSpec(CollectiveKind.ALL_REDUCE), p, n)
    rs = required_outputs(CollectiveSpec(CollectiveKind.REDUCE_SCATTER), p, n)
    ag = required_outputs(CollectiveSpec(CollectiveKind.ALL_GATHER), p, q)
    for slot, contributors in ar.items():
        owner, j = divmod(slot.offset, q)
        rs_slot = next(s for s in rs if s.rank == owner and s.offset == j)
        assert rs[rs_slot] == contributors
        # the AllGather over q slices per rank delivers source slice owner*q + j to this offset
        gathered = [s for s in ag if s.rank == slot.rank and s.offset == slot.offset]
        assert len(gathered) == 1 and ag[gathered[0]] == frozenset({owner * q + j})


@settings(max_examples=60, deadline=None)
@given(p=st.integers(1, 8), q=st.integers(1, 4),
       kind=st.sampled_from([CollectiveKind.ALL_REDUCE, CollectiveKind.ALL_GATHER, CollectiveKind.REDUCE_SCATTER]))
def test_inplace_aliases_are_canonical_and_consistent(p, q, kind):
    """Every in-place alias of an input slot canonicalises to the same coordinate as the slot itself."""
    n = p * q
    spec = CollectiveSpec(kind, inplace=True)
    state = initial_state(spec, p, n)
    for rank in range(p):
        for index in range(n):
            home = canonical(spec, p, n, rank, "i", index)
            for alias in input_aliases(spec, p, n, rank, index):
                assert canonical(spec, p, n, *alias) == home
                assert state[alias] == state[(rank, "i", index)]
    # out-of-place layouts have no aliases
    plain = CollectiveSpec(kind)
    assert all(not input_aliases(plain, p, n, r, i) for r in range(p) for i in range(n))


def test_synthesis_is_reproducible():
    """The same request gives byte-identical XML (fresh solver process, no cache reuse)."""
    from vericcl_b200.examples import example_documents
    from vericcl_b200.input.loader import resolve_documents
    from vericcl_b200.synthesis import synthesize
    for op, method in (("allreduce", "hierarchy"), ("allgather", "constructive_trees")):
        docs = example_documents(op, method, 4, total_size_bytes=4 * 4096, slice_size_bytes=4096)
        first = synthesize(resolve_documents(docs)).xml
        second = synthesize(resolve_documents(docs)).xml
        assert first == second
