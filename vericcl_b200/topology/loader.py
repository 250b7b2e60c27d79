"""Build a :class:`Topology` from a resolved request (reference: vericcl/topology/loader.py:289)."""
from __future__ import annotations

from vericcl_b200.errors import InputValidationError
from vericcl_b200.topology.model import DirectedLink, LinkKey, NodeGroup, SharedResource, Topology


def topology_from_document(doc: dict) -> Topology:
    links = {}
    for edge in doc["directed_links"]:
        key = LinkKey(edge["src"], edge["dst"])
        links[key] = DirectedLink(key, float(edge["alpha_us"]), float(edge["beta_us_per_byte"]),
                                  int(edge.get("max_channels", 16)), tuple(edge.get("resources", ())),
                                  tuple(edge.get("physical_path", ())))
    resources = {}
    for item in doc.get("shared_resources", ()):
        resources[item["id"]] = SharedResource(item["id"], float(item["capacity_bytes_per_us"]),
                                               frozenset(LinkKey(a, b) for a, b in item.get("links", ())),
                                               item.get("kind", "other"))
    nodes = tuple(NodeGroup(n["id"], tuple(n["ranks"]), tuple(n.get("gateways", ()))) for n in doc["nodes"])
    topo = Topology(doc.get("name", "unspecified"), int(doc["ranks"]), nodes, links, resources,
                    tuple(tuple(g) for g in doc.get("groups", ())),
                    tuple(tuple(g) for g in doc.get("multicast_groups", ())))
    for key, link in topo.links.items():
        for rid in link.resource_ids:
            if key not in topo.resources[rid].links:
                raise InputValidationError("link %s names resource %s that does not list it" % (key, rid))
    return topo


def load_topology(request) -> Topology:
    """Return the topology of a :class:`ResolvedInput`."""
    topo = topology_from_document(request.request_config["topology"])
    if topo.rank_count != request.rank_count:
        raise InputValidationError("topology rank count differs from the request")
    return topo
