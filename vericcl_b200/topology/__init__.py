"""Topology model, loader, NVSwitch generators and discovery (reference layer L1)."""
from .model import DirectedLink, LinkKey, NodeGroup, SharedResource, Topology
from .loader import load_topology, topology_from_document
from .nvswitch import nvswitch_topology, multinode_topology, discover_local_topology
from .legacy import convert_legacy_topology

__all__ = ["DirectedLink", "LinkKey", "NodeGroup", "SharedResource", "Topology", "load_topology",
           "topology_from_document", "nvswitch_topology", "multinode_topology", "discover_local_topology",
           "convert_legacy_topology"]
