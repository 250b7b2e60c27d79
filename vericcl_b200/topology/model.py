"""Directed-link topology with shared resources.

Links carry α (µs) / β (µs per byte) costs and a channel limit; shared
resources cap the summed rate of their member links (reference:
vericcl/topology/model.py:37-178).  On an NVSwitch box every GPU has one
egress and one ingress NVLink port budget shared by all its peers, which is
modelled as ``nvlink-tx-<r>`` / ``nvlink-rx-<r>`` shared resources; NVLS
multicast groups are recorded separately so the lowering can map group
reduce/broadcast steps onto ``multimem`` instructions.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from types import MappingProxyType
from typing import Mapping, Tuple

from vericcl_b200.errors import SemanticError


@dataclass(frozen=True, order=True)
class LinkKey:
    src: int
    dst: int

    def __str__(self) -> str:
        return "%d:%d" % (self.src, self.dst)


@dataclass(frozen=True)
class DirectedLink:
    key: LinkKey
    alpha_us: float
    beta_us_per_byte: float
    max_channels: int = 16
    resource_ids: Tuple[str, ...] = ()
    physical_path: Tuple[str, ...] = ()

    @property
    def bandwidth_bytes_per_us(self) -> float:
        return 1.0 / self.beta_us_per_byte

    def time_us(self, payload_bytes: int) -> float:
        return self.alpha_us + self.beta_us_per_byte * payload_bytes


@dataclass(frozen=True)
class SharedResource:
    resource_id: str
    capacity_bytes_per_us: float
    links: frozenset
    kind: str = "other"


@dataclass(frozen=True)
class NodeGroup:
    node_id: int
    ranks: Tuple[int, ...]
    gateways: Tuple[int, ...] = ()


@dataclass(frozen=True)
class Topology:
    name: str
    rank_count: int
    nodes: Tuple[NodeGroup, ...]
    links: Mapping[LinkKey, DirectedLink]
    resources: Mapping[str, SharedResource] = field(default_factory=dict)
    groups: Tuple[Tuple[int, ...], ...] = ()
    multicast_groups: Tuple[Tuple[int, ...], ...] = ()

    def __post_init__(self):
        object.__setattr__(self, "links", MappingProxyType(dict(self.links)))
        object.__setattr__(self, "resources", MappingProxyType(dict(self.resources)))

    def link(self, key: LinkKey) -> DirectedLink:
        try:
            return self.links[key]
        except KeyError:
            raise SemanticError("no directed link %s" % key) from None

    def has_link(self, src: int, dst: int) -> bool:
        return LinkKey(src, dst) in self.links

    def out_neighbors(self, rank: int):
        return sorted(key.dst for key in self.links if key.src == rank)

    def in_neighbors(self, rank: int):
        return sorted(key.src for key in self.links if key.dst == rank)

    def node_of(self, rank: int) -> NodeGroup:
        for node in self.nodes:
            if rank in node.ranks:
                return node
        raise SemanticError("rank %d belongs to no node" % rank)

    def is_complete(self) -> bool:
        """True when every ordered pair of distinct ranks has a direct link."""
        return len(self.links) == self.rank_count * (self.rank_count - 1)

    def multicast_group_of(self, ranks) -> Tuple[int, ...] | None:
        wanted = set(ranks)
        for group in self.multicast_groups:
            if wanted <= set(group):
                return group
        return None

    def signature(self) -> dict:
        """Structure + costs, used for isomorphism-indexed history reuse."""
        return {"ranks": self.rank_count,
                "links": sorted((k.src, k.dst, v.alpha_us, v.beta_us_per_byte, v.max_channels)
                                for k, v in self.links.items()),
                "resources": sorted((r.resource_id, r.capacity_bytes_per_us, sorted((l.src, l.dst) for l in r.links))
                                    for r in self.resources.values())}
