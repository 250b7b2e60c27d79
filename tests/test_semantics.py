from hypothesis import given, settings, strategies as st

from vericcl_b200.semantics.collective import CollectiveKind, CollectiveSpec, required_outputs


@settings(max_examples=60, deadline=None)
@given(p=st.integers(1, 8), q=st.integers(1, 4),
       kind=st.sampled_from([CollectiveKind.ALL_REDUCE, CollectiveKind.ALL_GATHER, CollectiveKind.REDUCE_SCATTER,
                             CollectiveKind.ALL_TO_ALL]))
def test_required_outputs_partition(p, q, kind):
    n = p * q
    out = required_outputs(CollectiveSpec(kind), p, n)
    if kind is CollectiveKind.ALL_GATHER:
        assert len(out) == p * p * n
        assert all(len(v) == 1 for v in out.values())
    elif kind is CollectiveKind.ALL_REDUCE:
        assert len(out) == p * n
        assert all(len(v) == p for v in out.values())
    elif kind is CollectiveKind.REDUCE_SCATTER:
        assert len(out) == n
        # every logical index reduced exactly once
        assert sorted(min(v) % n for v in out.values()) == list(range(n))
    else:
        # all-to-all is a permutation of original slices
        assert sorted(min(v) for v in out.values()) == list(range(p * n))


def test_rooted():
    out = required_outputs(CollectiveSpec(CollectiveKind.BROADCAST, root=2), 4, 3)
    assert all(v == frozenset({2 * 3 + s.offset}) for s, v in out.items())
    out = required_outputs(CollectiveSpec(CollectiveKind.REDUCE, root=1), 4, 2)
    assert {s.rank for s in out} == {1}
