"""Convert TACCL-format topology/sketch pairs into topology documents.

    python -m vericcl_b200.topology.legacy --topology topo.json --sketch sketch.json \\
        --reference-slice-bytes 1048576 [--local-hbm-gbps 6500] --out topology.json

TACCL describes a node by ``gpus_per_node`` and per-chunk durations in µs:
``alpha`` (start-up) and, per link class, ``node_betas_list`` (transfer
part) and ``node_invbws_list`` (whole chunk, ``alpha + beta``; authoritative
when both are given), either as class lists or as full ``links`` /
``betas`` / ``invbws`` matrices (row = receiver).  The class of a GPU pair
comes from the node type: NDv2 (DGX-1V hybrid cube-mesh: double-NVLink pairs
class 2, single pairs class 1), ``fit8`` (class 1 inside each group of four,
class 2 across) or, otherwise, every pair class 1.  The sketch gives the
node count, optional intra-node switch groups (each member's egress and
ingress become shared resources) and the inter-node relay: which local
ranks connect across nodes (``fully-connected``, ``direct-map`` or an
explicit map) and the remote per-chunk durations (``remote_alpha``,
``remote_beta``, ``remote_invbw``); every node pair and every node's NIC
egress / ingress becomes a shared resource.

Durations are per chunk of the reference slice size, so each becomes
``alpha_us`` plus ``beta_us_per_byte = (duration − alpha) / reference slice
bytes``, and a shared resource's capacity is the reference slice over its
transfer part.  The converted document keeps the sources, as canonical
JSON, under ``provenance`` (reference: vericcl/topology/legacy.py:231-372, whose
internal output form differs; the NDv2 link classes are a hardware fact and
are the same).
"""
from __future__ import annotations

import argparse
import json
import sys
from copy import deepcopy

from vericcl_b200.errors import InputValidationError

LEGACY_FORMAT = "taccl_topology_v2"

# DGX-1V / NDv2 NVLink wiring: pairs joined by two NVLinks, and by one
NDV2_DOUBLE = ((0, 2), (0, 3), (1, 2), (1, 5), (3, 7), (4, 6), (4, 7), (5, 6))
NDV2_SINGLE = ((0, 1), (0, 4), (1, 3), (2, 3), (2, 6), (4, 5), (5, 7), (6, 7))


def _int(value, name, minimum=0):
    if isinstance(value, bool) or not isinstance(value, int) or value < minimum:
        raise InputValidationError("%s must be an integer of at least %d" % (name, minimum))
    return value


def _num(value, name):
    if isinstance(value, bool) or not isinstance(value, (int, float)) or value < 0:
        raise InputValidationError("%s must be a nonnegative number" % name)
    return float(value)


def _classes(name: str, g: int, nclasses: int):
    """classes[dst][src]: 0 none, k for class k (1-based)."""
    lname = name.lower()
    if "ndv2" in lname:
        if g != 8 or nclasses < 2:
            raise InputValidationError("an NDv2 node has 8 GPUs and two link classes")
        table = [[0] * g for _ in range(g)]
        for cls, pairs in ((2, NDV2_DOUBLE), (1, NDV2_SINGLE)):
            for a, b in pairs:
                table[a][b] = table[b][a] = cls
        return table
    if "fit8" in lname and g == 8 and nclasses >= 2:
        return [[0 if s == d else (1 if s // 4 == d // 4 else 2) for s in range(g)] for d in range(g)]
    return [[0 if s == d else 1 for s in range(g)] for d in range(g)]


def _chunk(alpha, beta, invbw, where):
    """Per-chunk (alpha, transfer part) with invbw authoritative."""
    alpha = _num(alpha, where + " alpha")
    if invbw is not None:
        total = _num(invbw, where + " invbw")
        if total < alpha:
            raise InputValidationError("%s invbw is below its alpha" % where)
        return alpha, total - alpha
    if beta is None:
        raise InputValidationError("%s needs beta or invbw" % where)
    return alpha, _num(beta, where + " beta")


def _node_links(topo: dict, g: int):
    """[(src_local, dst_local, alpha, transfer)] inside one node."""
    alpha = topo.get("alpha")
    if alpha is None:
        raise InputValidationError("a TACCL topology needs alpha")
    out = []
    if all(k in topo for k in ("links", "betas", "invbws")):
        for d in range(g):
            for s in range(g):
                if topo["links"][d][s]:
                    a, t = _chunk(alpha, topo["betas"][d][s], topo["invbws"][d][s], "link %d->%d" % (s, d))
                    out.append((s, d, a, t))
        return out
    betas, invbws = topo.get("node_betas_list"), topo.get("node_invbws_list")
    if not isinstance(betas, list) or not isinstance(invbws, list) or not betas or len(betas) != len(invbws):
        raise InputValidationError("node_betas_list and node_invbws_list must be aligned, non-empty lists")
    classes = _classes(str(topo.get("name", "")), g, len(betas))
    for d in range(g):
        for s in range(g):
            cls = classes[d][s]
            if cls:
                a, t = _chunk(alpha, betas[cls - 1], invbws[cls - 1], "class %d" % cls)
                out.append((s, d, a, t))
    return out


def _canonical(value) -> str:
    return json.dumps(value, sort_keys=True, separators=(",", ":"))


def _connections(value, g: int) -> dict:
    if value == "fully-connected":
        return {r: tuple(range(g)) for r in range(g)}
    if value == "direct-map":
        return {r: (r,) for r in range(g)}
    if not isinstance(value, dict):
        raise InputValidationError("internode_conn must be fully-connected, direct-map or a map")
    out = {}
    for key, dests in value.items():
        src = int(key)
        if not 0 <= src < g or not isinstance(dests, list) or len(set(dests)) != len(dests) \
                or any(not isinstance(x, int) or not 0 <= x < g for x in dests):
            raise InputValidationError("internode_conn entries must map local ranks to distinct local ranks")
        out[src] = tuple(sorted(dests))
    return dict(sorted(out.items()))


def convert_legacy_topology(topology: dict, sketch: dict, *, reference_slice_bytes: int,
                            local_hbm_gbps: float | None = None) -> dict:
    """Topology document for a TACCL topology/sketch pair (inputs are not modified).

    TACCL sources carry no local copy/reduce costs; ``local_hbm_gbps`` adds
    HBM-bound ones for every rank.  Without it the document has none, and a
    prediction needs them from calibration (no cost is ever taken as zero).
    """
    topo, sk = deepcopy(topology), deepcopy(sketch)
    size = _int(reference_slice_bytes, "reference_slice_bytes", 1)
    g = _int(topo.get("gpus_per_node"), "gpus_per_node", 1)
    nodes = _int(sk.get("nnodes"), "nnodes", 1)
    links, resources = {}, []

    def link(src, dst, alpha, transfer):
        if (src, dst) in links:
            raise InputValidationError("link %d->%d appears twice" % (src, dst))
        if transfer <= 0:
            raise InputValidationError("link %d->%d has no transfer time" % (src, dst))
        links[(src, dst)] = {"src": src, "dst": dst, "alpha_us": alpha, "beta_us_per_byte": transfer / size,
                             "max_channels": 16, "resources": []}

    def resource(rid, kind, members, transfer):
        if members:
            resources.append({"id": rid, "kind": kind, "capacity_bytes_per_us": size / transfer,
                              "links": [list(m) for m in sorted(members)]})
            for m in members:
                links[m]["resources"].append(rid)

    local = _node_links(topo, g)
    for n in range(nodes):
        base = n * g
        for s, d, a, t in local:
            link(base + s, base + d, a, t)
    intra = sk.get("intranode_sketch", {"strategy": "none"}) or {"strategy": "none"}
    if intra.get("strategy") == "switch":
        for n in range(nodes):
            base = n * g
            for si, group in enumerate(intra.get("switches", [])):
                if any(not isinstance(x, int) or not 0 <= x < g for x in group) or len(set(group)) != len(group):
                    raise InputValidationError("switch groups must list distinct local ranks")
                for r in group:
                    out = [(base + r, base + q) for q in group if q != r and (base + r, base + q) in links]
                    inc = [(base + q, base + r) for q in group if q != r and (base + q, base + r) in links]
                    for direction, members in (("egress", out), ("ingress", inc)):
                        if members:
                            t = max(links[members[0]]["beta_us_per_byte"] * size, 1e-12)
                            resource("node-%d-switch-%d-rank-%d-%s" % (n, si, base + r, direction), "switch_port",
                                     members, t)
    gateways = set()
    if nodes > 1:
        inter = sk.get("internode_sketch") or {}
        if inter.get("strategy") != "relay":
            raise InputValidationError("multi-node TACCL sketches must use the relay inter-node strategy")
        conn = _connections(inter.get("internode_conn"), g)
        ra, rt = _chunk(topo.get("remote_alpha", 0), topo.get("remote_beta"), topo.get("remote_invbw"), "remote")
        egress = {n: [] for n in range(nodes)}
        ingress = {n: [] for n in range(nodes)}
        for sn in range(nodes):
            for dn in range(nodes):
                if sn == dn:
                    continue
                pair = []
                for s, dests in conn.items():
                    for d in dests:
                        key = (sn * g + s, dn * g + d)
                        link(key[0], key[1], ra, rt)
                        pair.append(key)
                        egress[sn].append(key)
                        ingress[dn].append(key)
                        gateways.update(key)
                resource("inter-node-%d-to-%d" % (sn, dn), "link", pair, rt)
        for n in range(nodes):
            resource("nic-node-%d-egress" % n, "nic", egress[n], rt)
            resource("nic-node-%d-ingress" % n, "nic", ingress[n], rt)
    for rec in links.values():
        rec["resources"] = sorted(rec["resources"])
    extra = {}
    if local_hbm_gbps is not None:
        from vericcl_b200.topology.nvswitch import hbm_local_costs
        extra["local_costs"] = hbm_local_costs(g * nodes, _num(local_hbm_gbps, "local_hbm_gbps") or 1.0)
    return {
        "name": str(topo.get("name", "taccl-topology")),
        "ranks": g * nodes,
        "nodes": [{"id": n, "ranks": list(range(n * g, (n + 1) * g)),
                   "gateways": [r for r in range(n * g, (n + 1) * g) if r in gateways]} for n in range(nodes)],
        "directed_links": [links[k] for k in sorted(links)],
        "shared_resources": sorted(resources, key=lambda r: r["id"]),
        "provenance": {"legacy_format": LEGACY_FORMAT, "reference_slice_bytes": size,
                       "source_topology": _canonical(topology), "source_sketch": _canonical(sketch)},
        **extra,
    }


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="vericcl_b200.topology.legacy")
    ap.add_argument("--topology", required=True)
    ap.add_argument("--sketch", required=True)
    ap.add_argument("--reference-slice-bytes", type=int, required=True)
    ap.add_argument("--local-hbm-gbps", type=float, default=None,
                    help="add HBM-bound local copy/reduce costs at this bandwidth")
    ap.add_argument("--out", required=True)
    args = ap.parse_args(argv)
    from vericcl_b200.utils.jsonio import atomic_write_json, strict_load
    doc = convert_legacy_topology(strict_load(args.topology), strict_load(args.sketch),
                                  reference_slice_bytes=args.reference_slice_bytes,
                                  local_hbm_gbps=args.local_hbm_gbps)
    atomic_write_json(args.out, doc)
    print(json.dumps({"ranks": doc["ranks"], "links": len(doc["directed_links"]),
                      "resources": len(doc["shared_resources"])}))
    return 0


if __name__ == "__main__":
    sys.exit(main())
