"""Topology documents for a single NVSwitch domain (HGX/DGX B200).

Every GPU reaches every peer through NVSwitch with the full per-GPU NVLink 5
bandwidth, so a pairwise link is not the bottleneck; the per-GPU egress and
ingress port budgets are.  The generated document therefore has a complete
directed graph whose links all belong to the sender's ``nvlink-tx`` and the
receiver's ``nvlink-rx`` shared resources, plus one NVLS multicast group over
all ranks when the switch supports in-network reduction.  Units follow the
request schema: α in µs, β in µs per byte, capacities in bytes per µs.
Shared per-GPU resources follow the reference's shared-NIC template
(README.md:155-166 there), applied to NVLink ports.
"""
from __future__ import annotations

# Measured on B200s: peer copy ~770 GB/s per direction per GPU
# (nominal 900 GB/s).  1 GB/s = 1000 bytes/us.
B200_NVLINK_GBPS = 770.0
B200_ALPHA_US = 1.5
B200_HBM_GBPS = 6500.0


def nvswitch_topology(ranks: int, *, alpha_us: float = B200_ALPHA_US, link_gbps: float = B200_NVLINK_GBPS,
                      port_gbps: float | None = None, nvls: bool = True, name: str | None = None,
                      hbm_gbps: float = B200_HBM_GBPS, max_channels: int = 16) -> dict:
    """Return a topology.json document for ``ranks`` GPUs behind one NVSwitch."""
    port = link_gbps if port_gbps is None else port_gbps
    beta = 1.0 / (link_gbps * 1000.0)
    links, tx, rx = [], {r: [] for r in range(ranks)}, {r: [] for r in range(ranks)}
    for src in range(ranks):
        for dst in range(ranks):
            if src == dst:
                continue
            links.append({"src": src, "dst": dst, "alpha_us": alpha_us, "beta_us_per_byte": beta,
                          "max_channels": max_channels,
                          "resources": ["nvlink-tx-%d" % src, "nvlink-rx-%d" % dst],
                          "physical_path": ["gpu%d" % src, "nvswitch", "gpu%d" % dst]})
            tx[src].append([src, dst])
            rx[dst].append([src, dst])
    resources = []
    for r in range(ranks):
        if tx[r]:
            resources.append({"id": "nvlink-tx-%d" % r, "kind": "nvlink_port",
                              "capacity_bytes_per_us": port * 1000.0, "links": tx[r]})
            resources.append({"id": "nvlink-rx-%d" % r, "kind": "nvlink_port",
                              "capacity_bytes_per_us": port * 1000.0, "links": rx[r]})
    return {
        "name": name or "nvswitch-b200-x%d" % ranks,
        "ranks": ranks,
        "nodes": [{"id": 0, "ranks": list(range(ranks)), "gateways": []}],
        "directed_links": links,
        "shared_resources": resources,
        "groups": [],
        "multicast_groups": [list(range(ranks))] if nvls and ranks > 1 else [],
        "local_costs": hbm_local_costs(ranks, hbm_gbps),
    }


def hbm_local_costs(ranks: int, hbm_gbps: float = B200_HBM_GBPS) -> list:
    """Local copy and reduce costs of HBM-bound kernels for every rank."""
    copy_beta = 2.0 / (hbm_gbps * 1000.0)   # a copy reads and writes every byte
    reduce_beta = 3.0 / (hbm_gbps * 1000.0)  # two reads and one write
    return [{"rank": r, "copy": {"alpha_us": 1.0, "beta_us_per_byte": copy_beta},
             "reduce": {"alpha_us": 1.0, "beta_us_per_byte": reduce_beta}} for r in range(ranks)]


def multinode_topology(groups: int, per_group: int, *, intra_gbps: float = B200_NVLINK_GBPS,
                       inter_gbps: float = 25.0, intra_alpha_us: float = B200_ALPHA_US,
                       inter_alpha_us: float = 5.0, rank_shares: bool = False) -> dict:
    """Emulated multi-node topology: NVSwitch groups joined by a slow shared link.

    Used for the online repair configuration (2 groups × 4 ranks with a
    25 GB/s inter-group link, emulated on one box by throttling channels).
    Each group's outbound and inbound inter-group traffic shares one NIC-like
    resource of ``inter_gbps``; ``rank_shares`` adds the emulator's even split
    of it (see :func:`grouped_topology`).
    """
    return grouped_topology([per_group] * groups, inter_gbps=inter_gbps, inter_alpha_us=inter_alpha_us,
                            name="emulated-%dx%d" % (groups, per_group), rank_shares=rank_shares)


def grouped_topology(sizes, *, inter_gbps: float = 25.0, inter_alpha_us: float = 5.0, gateways=None,
                     name: str | None = None, rank_shares: bool = False) -> dict:
    """NVSwitch groups of the given sizes (they may differ) joined by slow shared inter-group links.

    ``gateways``: per group, the ranks that own the group's inter-group
    links (default: every member); links between non-gateway members of
    different groups are left out, as on nodes whose NICs hang off some GPUs.
    ``rank_shares``: also give every rank one resource of ``inter_gbps`` / (its
    group's size) on the inter-group links into it.  That is how the link
    emulator (``VERICCL_EMULATE``) enforces the shared link: each rank reads
    from other groups through its own even share, a token bucket, rather than
    drawing on the group's link while the other members are idle.
    """
    ranks = sum(sizes)
    starts = [sum(sizes[:i]) for i in range(len(sizes))]
    group = {}
    for g, (lo, n) in enumerate(zip(starts, sizes)):
        for r in range(lo, lo + n):
            group[r] = g
    gws = [list(range(lo, lo + n)) for lo, n in zip(starts, sizes)] if gateways is None else \
        [sorted(g) for g in gateways]
    doc = nvswitch_topology(ranks, nvls=False, name=name or "emulated-" + "+".join(map(str, sizes)))
    doc["nodes"] = [{"id": g, "ranks": list(range(lo, lo + n)), "gateways": gws[g]}
                    for g, (lo, n) in enumerate(zip(starts, sizes))]
    if gateways is not None:
        keep = [e for e in doc["directed_links"] if group[e["src"]] == group[e["dst"]] or
                (e["src"] in gws[group[e["src"]]] and e["dst"] in gws[group[e["dst"]]])]
        doc["directed_links"] = keep
        for res in doc["shared_resources"]:
            res["links"] = [pair for pair in res["links"] if group[pair[0]] == group[pair[1]] or
                            (pair[0] in gws[group[pair[0]]] and pair[1] in gws[group[pair[1]]])]
    nic = {}
    for edge in doc["directed_links"]:
        gs, gd = group[edge["src"]], group[edge["dst"]]
        if gs == gd:
            continue
        edge["alpha_us"] = inter_alpha_us
        edge["beta_us_per_byte"] = 1.0 / (inter_gbps * 1000.0)
        edge["physical_path"] = ["gpu%d" % edge["src"], "inter-group", "gpu%d" % edge["dst"]]
        for rid in ("nic-%d-tx" % gs, "nic-%d-rx" % gd):
            nic.setdefault(rid, []).append([edge["src"], edge["dst"]])
            edge["resources"].append(rid)
    for rid, members in sorted(nic.items()):
        doc["shared_resources"].append({"id": rid, "kind": "nic", "capacity_bytes_per_us": inter_gbps * 1000.0,
                                        "links": members})
    if rank_shares:
        shares = {}
        for edge in doc["directed_links"]:
            if group[edge["src"]] != group[edge["dst"]]:
                rid = "nic-share-rx-%d" % edge["dst"]
                shares.setdefault(rid, []).append([edge["src"], edge["dst"]])
                edge["resources"].append(rid)
        for rid, members in sorted(shares.items()):
            dst = members[0][1]
            doc["shared_resources"].append({"id": rid, "kind": "nic",
                                            "capacity_bytes_per_us": inter_gbps * 1000.0 / sizes[group[dst]],
                                            "links": members})
    doc["groups"] = [node["ranks"] for node in doc["nodes"]]
    doc["multicast_groups"] = [node["ranks"] for node in doc["nodes"] if len(node["ranks"]) > 1]
    return doc


def discover_local_topology(device_count: int | None = None) -> dict:
    """Probe the local box with NVML (read-only) and return a topology document.

    Falls back to the nominal B200 description when NVML is unavailable.  The
    probe only reads device attributes; it never changes a device setting.
    """
    count, nvlinks, multicast = device_count, None, True
    try:
        import pynvml  # provided by nvidia-ml-py
        pynvml.nvmlInit()
        try:
            count = count or pynvml.nvmlDeviceGetCount()
            handle = pynvml.nvmlDeviceGetHandleByIndex(0)
            active = 0
            for link in range(18):
                try:
                    if pynvml.nvmlDeviceGetNvLinkState(handle, link):
                        active += 1
                except pynvml.NVMLError:
                    break
            nvlinks = active
        finally:
            pynvml.nvmlShutdown()
    except Exception:
        pass
    count = count or 8
    doc = nvswitch_topology(count, nvls=multicast)
    doc["name"] = "discovered-nvswitch-x%d" % count + ("" if nvlinks is None else "-nv%d" % nvlinks)
    return doc
