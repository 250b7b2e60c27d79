"""Exact XML text of small schedules (format stability)."""
from pathlib import Path

from vericcl_b200.examples import example_documents
from vericcl_b200.input.loader import resolve_documents
from vericcl_b200.synthesis import synthesize

GOLDEN = Path(__file__).parent / "golden"


def _xml(op, inplace):
    d = example_documents(op, "hierarchy", 2, total_size_bytes=1024, slice_size_bytes=1024, inplace=inplace)
    return synthesize(resolve_documents(d)).xml


def test_two_rank_allreduce_out_of_place():
    assert _xml("allreduce", False) == (GOLDEN / "two_rank_allreduce_out_of_place.xml").read_text()


def test_two_rank_allgather_in_place():
    assert _xml("allgather", True) == (GOLDEN / "two_rank_allgather_in_place.xml").read_text()
