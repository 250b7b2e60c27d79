"""TACCL-format topology conversion (vericcl_b200/topology/legacy.py)."""
import json
from copy import deepcopy

import pytest

from vericcl_b200.errors import InputValidationError
from vericcl_b200.input.schema import TOPOLOGY, normalize
from vericcl_b200.topology import topology_from_document
from vericcl_b200.topology.legacy import NDV2_DOUBLE, NDV2_SINGLE, convert_legacy_topology, main

MB = 1 << 20


def ndv2(**kw):
    topo = {"name": "ndv2-test", "gpus_per_node": 8, "alpha": 4, "node_betas_list": [10, 5],
            "node_invbws_list": [14, 9], "remote_alpha": 6, "remote_beta": 40, "remote_invbw": 46}
    topo.update(kw)
    return topo


def relay(conn, nnodes=2, intra=None):
    return {"nnodes": nnodes, "intranode_sketch": intra or {"strategy": "none"},
            "internode_sketch": {"strategy": "relay", "internode_conn": conn}}


def valid(doc):
    normalize(TOPOLOGY, doc, "topology", {}, "test")
    return topology_from_document(doc)


def test_ndv2_two_nodes_fully_connected():
    topo, sketch = ndv2(), relay("fully-connected")
    before = (deepcopy(topo), deepcopy(sketch))
    doc = convert_legacy_topology(topo, sketch, reference_slice_bytes=MB)
    assert (topo, sketch) == before
    t = valid(doc)
    assert t.rank_count == 16
    # cube-mesh: 16 wired pairs per node, both directions; 8x8 relays per node pair, both directions
    assert len(doc["directed_links"]) == 2 * 32 + 2 * 64
    assert t.has_link(0, 4) and t.has_link(4, 0) and not t.has_link(0, 5) and not t.has_link(0, 6)
    assert t.has_link(0, 8) and t.has_link(7, 15) and t.has_link(15, 0)
    per = {(e["src"], e["dst"]): e for e in doc["directed_links"]}
    a, b = NDV2_DOUBLE[0], NDV2_SINGLE[0]
    # invbw is the whole chunk: class 2 (double links) transfers in 9 - 4 us, class 1 in 14 - 4 us
    assert per[a]["beta_us_per_byte"] == pytest.approx(5 / MB)
    assert per[b]["beta_us_per_byte"] == pytest.approx(10 / MB)
    assert per[a]["alpha_us"] == 4
    assert per[(0, 8)]["beta_us_per_byte"] == pytest.approx(40 / MB) and per[(0, 8)]["alpha_us"] == 6
    assert [n["gateways"] for n in doc["nodes"]] == [list(range(8)), list(range(8, 16))]
    ids = {r["id"]: r for r in doc["shared_resources"]}
    assert len(ids["inter-node-0-to-1"]["links"]) == 64
    assert len(ids["nic-node-0-egress"]["links"]) == 64
    assert ids["nic-node-1-ingress"]["capacity_bytes_per_us"] == pytest.approx(MB / 40)
    assert "nic-node-0-egress" in per[(0, 8)]["resources"] and "inter-node-0-to-1" in per[(0, 8)]["resources"]
    prov = doc["provenance"]
    assert prov["legacy_format"] == "taccl_topology_v2" and prov["reference_slice_bytes"] == MB
    assert json.loads(prov["source_topology"]) == topo and json.loads(prov["source_sketch"]) == sketch


def test_direct_map_relay_and_beta_fallback():
    topo = {"name": "pair", "gpus_per_node": 2, "alpha": 1, "node_betas_list": [3], "node_invbws_list": [None],
            "remote_alpha": 2, "remote_beta": 7}
    doc = convert_legacy_topology(topo, relay("direct-map"), reference_slice_bytes=1000)
    valid(doc)
    inter = [(e["src"], e["dst"]) for e in doc["directed_links"] if e["src"] // 2 != e["dst"] // 2]
    assert inter == [(0, 2), (1, 3), (2, 0), (3, 1)]
    per = {(e["src"], e["dst"]): e for e in doc["directed_links"]}
    assert per[(0, 1)]["beta_us_per_byte"] == pytest.approx(3 / 1000)     # no invbw: beta is the transfer part
    assert per[(1, 3)]["beta_us_per_byte"] == pytest.approx(7 / 1000)


def test_explicit_map_and_single_node():
    topo = ndv2(name="plain8", node_betas_list=[2], node_invbws_list=[6])
    doc = convert_legacy_topology(topo, relay({"0": [0, 4], "4": [4]}), reference_slice_bytes=MB)
    t = valid(doc)
    inter = sorted((e["src"], e["dst"]) for e in doc["directed_links"] if e["src"] // 8 != e["dst"] // 8)
    assert inter == [(0, 8), (0, 12), (4, 12), (8, 0), (8, 4), (12, 4)]
    assert all(t.has_link(s, d) for s in range(8) for d in range(8) if s != d)     # default: all pairs
    one = convert_legacy_topology(topo, {"nnodes": 1}, reference_slice_bytes=MB)
    assert valid(one).rank_count == 8 and one["nodes"][0]["gateways"] == []


def test_fit8_classes_and_matrices():
    topo = ndv2(name="fit8-box", node_betas_list=[1, 3], node_invbws_list=[5, 7])
    per = {(e["src"], e["dst"]): e for e in convert_legacy_topology(topo, {"nnodes": 1},
                                                                    reference_slice_bytes=100)["directed_links"]}
    assert per[(0, 3)]["beta_us_per_byte"] == pytest.approx(1 / 100)       # same half: class 1
    assert per[(0, 4)]["beta_us_per_byte"] == pytest.approx(3 / 100)       # across halves: class 2
    g = 3
    links = [[0, 1, 0], [1, 0, 1], [1, 1, 0]]                               # row = receiver
    mat = {"name": "m", "gpus_per_node": g, "alpha": 1, "links": links,
           "betas": [[0, 2, 0], [3, 0, 4], [5, 6, 0]], "invbws": [[0, 3, 0], [4, 0, 5], [6, 7, 0]]}
    doc = convert_legacy_topology(mat, {"nnodes": 1}, reference_slice_bytes=10)
    got = {(e["src"], e["dst"]): e["beta_us_per_byte"] for e in doc["directed_links"]}
    assert got == pytest.approx({(1, 0): 0.2, (0, 1): 0.3, (2, 1): 0.4, (0, 2): 0.5, (1, 2): 0.6})


def test_switch_groups_become_port_resources():
    topo = ndv2(name="sw", node_betas_list=[2], node_invbws_list=[6])
    sketch = relay("direct-map", intra={"strategy": "switch", "switches": [[0, 1, 2, 3], [4, 5, 6, 7]]})
    doc = convert_legacy_topology(topo, sketch, reference_slice_bytes=MB)
    valid(doc)
    ids = {r["id"]: r for r in doc["shared_resources"]}
    port = ids["node-1-switch-0-rank-9-egress"]
    assert port["kind"] == "switch_port" and sorted(map(tuple, port["links"])) == [(9, 8), (9, 10), (9, 11)]
    assert port["capacity_bytes_per_us"] == pytest.approx(MB / 2)
    assert sum(1 for r in ids if "switch" in r) == 2 * 8 * 2


@pytest.mark.parametrize("topo,sketch,msg", [
    (ndv2(gpus_per_node=4), {"nnodes": 1}, "NDv2"),
    (ndv2(), {"nnodes": 2}, "relay"),
    (ndv2(remote_invbw=1, remote_alpha=3), relay("direct-map"), "below"),
    (ndv2(), relay({"0": [9]}), "internode_conn"),
    (ndv2(node_betas_list=[1], node_invbws_list=[5]), {"nnodes": 1}, "NDv2"),
    (ndv2(alpha=None), {"nnodes": 1}, "alpha"),
    (ndv2(node_invbws_list=[4, 4]), {"nnodes": 1}, "transfer"),
])
def test_rejects_inconsistent_sources(topo, sketch, msg):
    with pytest.raises(InputValidationError, match=msg):
        convert_legacy_topology(topo, sketch, reference_slice_bytes=MB)


def test_converted_topology_synthesizes(tmp_path):
    from vericcl_b200.examples import example_documents
    from vericcl_b200.input.loader import resolve_documents
    from vericcl_b200.program.xmlio import parse_xml
    from vericcl_b200.synthesis import synthesize
    from vericcl_b200.verification.chunksim import check_program_numerics
    topo = {"name": "two-by-two", "gpus_per_node": 2, "alpha": 1, "node_betas_list": [1],
            "node_invbws_list": [2], "remote_alpha": 2, "remote_invbw": 10}
    tp, sp, out = tmp_path / "t.json", tmp_path / "s.json", tmp_path / "topology.json"
    tp.write_text(json.dumps(topo))
    sp.write_text(json.dumps(relay("direct-map")))
    assert main(["--topology", str(tp), "--sketch", str(sp), "--reference-slice-bytes", "1024",
                 "--local-hbm-gbps", "6500", "--out", str(out)]) == 0
    doc = json.loads(out.read_text())
    assert len(doc["local_costs"]) == 4
    bare = example_documents("allgather", "hierarchy", 4, total_size_bytes=4 * 1024, slice_size_bytes=1024,
                             topology=convert_legacy_topology(topo, relay("direct-map"), reference_slice_bytes=1024))
    missing = synthesize(resolve_documents(bare)).checks["prediction"]
    assert missing["status"] == "invalid" and "service:copy:0" in missing["detail"]
    d = example_documents("allgather", "hierarchy", 4, total_size_bytes=4 * 1024, slice_size_bytes=1024,
                          topology=doc)
    bundle = synthesize(resolve_documents(d))
    assert bundle.can_execute, bundle.checks
    ok, err = check_program_numerics(parse_xml(bundle.xml), count_per_rank=4 * 16, seed=1)
    assert ok, err
