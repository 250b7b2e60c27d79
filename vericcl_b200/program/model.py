"""Records of the lowering pipeline: storage plan and native (XML) program.

Logical values (contributor sets) and physical addresses are kept apart:
``Address(rank, buffer, offset)`` names an i/o/s slot of one slice
(reference: vericcl/xml/v5_model.py:24-133).
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Mapping


@dataclass(frozen=True, order=True)
class Address:
    rank: int
    buffer: str          # i | o | s
    offset: int


@dataclass(frozen=True)
class Value:
    state_id: str
    rank: int
    index: int
    contributors: frozenset
    producer: str | None


@dataclass(frozen=True)
class Instruction:
    operation_id: str
    kind: str            # send | rrc | copy
    inputs: tuple        # state ids read (sender value first; accumulator second for rrc)
    output: str          # state id written
    rank: int            # rank that writes the output
    peer: int            # sending rank (-1 for copy)
    channel: int
    stage_id: int
    dependencies: frozenset
    priority_time: float


@dataclass(frozen=True)
class StoragePlan:
    values: Mapping[str, Value]
    initial_ids: tuple
    instructions: tuple
    addresses: Mapping[str, Address]
    outputs: Mapping[object, str]
    input_slots: Mapping[int, int]
    output_slots: Mapping[int, int]
    scratch_slots: Mapping[int, int]
    reuse: tuple = ()


@dataclass(frozen=True)
class NativeStep:
    kind: str                         # s r rrc rcs rrs rrcs cpy re nop
    src: Address | None
    dst: Address | None
    dependency_tb: int = -1
    dependency_step: int = -1
    has_dependence: bool = False
    count: int = 1
    operation_id: str = ""


@dataclass(frozen=True)
class NativeBlock:
    rank: int
    tb_id: int
    channel: int
    send_peer: int
    recv_peer: int
    steps: tuple


@dataclass(frozen=True)
class NativeProgram:
    name: str
    collective: str
    inplace: bool
    rank_count: int
    channels: int
    chunks_per_loop: int
    blocks: tuple
    input_slots: Mapping[int, int]
    output_slots: Mapping[int, int]
    scratch_slots: Mapping[int, int]
    proto: str = "Simple"
    redop: str = "nop"
    min_bytes: int = 0
    max_bytes: int = 0

    def rank_blocks(self, rank: int):
        return [b for b in self.blocks if b.rank == rank]

    def step_count(self) -> int:
        return sum(len(b.steps) for b in self.blocks)
