"""End to end through the CLI in a child process: hierarchical solve, verify, reproducibility."""
import hashlib
import json
import os
import subprocess
import sys
from pathlib import Path

import pytest

from vericcl_b200.examples import example_documents, write_documents
from vericcl_b200.topology.nvswitch import multinode_topology

ROOT = Path(__file__).resolve().parents[1]


def _cli(args, cwd):
    env = dict(os.environ, PYTHONPATH=str(ROOT) + os.pathsep + os.environ.get("PYTHONPATH", ""),
               CUDA_VISIBLE_DEVICES="")
    return subprocess.run([sys.executable, "-m", "vericcl_b200"] + args, cwd=cwd, env=env, capture_output=True,
                          text=True, timeout=600)


def _docs_args(indir):
    out = []
    for k in ("topology", "sketch", "atom", "runtime"):
        out += ["--" + k, str(indir / (k + ".json"))]
    return out


@pytest.fixture
def two_node_inputs(tmp_path):
    """AllReduce on two groups of two ranks joined by a slow shared link (a two-node gateway topology)."""
    docs = example_documents("allreduce", "hierarchy", 4, total_size_bytes=16 << 10, slice_size_bytes=4 << 10,
                             topology=multinode_topology(2, 2, inter_gbps=25.0), tuning_rounds=1,
                             calibration=False)
    write_documents(tmp_path / "in", docs)
    return tmp_path / "in"


def test_hierarchical_solve_and_verify(two_node_inputs, tmp_path):
    base = ["--project-root", str(tmp_path), "--case", "e2e"]
    res = _cli(["solve"] + base + ["--run-id", "s"] + _docs_args(two_node_inputs), tmp_path)
    assert res.returncode == 0, res.stderr[-2000:]
    run = tmp_path / "examples" / "e2e" / "output" / "s"
    meta = json.loads((run / "run.json").read_text())
    assert meta["status"] == "finished" and meta["best"]["t_pred_us"] > 0
    checks = meta["best"]["checks"]
    assert all(v["status"] in ("valid", "not_run") for v in checks.values())
    sidecar = json.loads((run / "schedule.json").read_text())
    assert sidecar["checks"] == checks
    res = _cli(["verify"] + base + ["--run-id", "v"] + _docs_args(two_node_inputs)
               + ["--xml", str(run / "schedule.xml"), "--sidecar", str(run / "schedule.json"),
                  "--model", str(run / "model.json")], tmp_path)
    assert res.returncode == 0, res.stderr[-2000:]
    vmeta = json.loads((tmp_path / "examples" / "e2e" / "output" / "v" / "run.json").read_text())
    assert vmeta["best"]["t_pred_us"] == pytest.approx(meta["best"]["t_pred_us"])
    res = _cli(["inspect", "--run", str(run)], tmp_path)
    assert res.returncode == 0


def test_solves_are_reproducible(two_node_inputs, tmp_path):
    digests, preds = [], []
    for run_id in ("r1", "r2"):
        res = _cli(["solve", "--project-root", str(tmp_path), "--case", "repro", "--run-id", run_id]
                   + _docs_args(two_node_inputs), tmp_path)
        assert res.returncode == 0, res.stderr[-2000:]
        run = tmp_path / "examples" / "repro" / "output" / run_id
        digests.append(hashlib.sha256((run / "schedule.xml").read_bytes()).hexdigest())
        preds.append(json.loads((run / "run.json").read_text())["best"]["t_pred_us"])
    assert digests[0] == digests[1] and preds[0] == preds[1]


def test_bad_sidecar_is_rejected(two_node_inputs, tmp_path):
    base = ["--project-root", str(tmp_path), "--case", "bad"]
    assert _cli(["solve"] + base + ["--run-id", "s"] + _docs_args(two_node_inputs), tmp_path).returncode == 0
    run = tmp_path / "examples" / "bad" / "output" / "s"
    xml = (run / "schedule.xml").read_text()
    # drop one step: the schedule no longer delivers every output
    lines = xml.splitlines()
    cut = next(i for i, l in enumerate(lines) if "<step " in l)
    broken = tmp_path / "broken.xml"
    broken.write_text("\n".join(lines[:cut] + lines[cut + 1:]) + "\n")
    res = _cli(["verify"] + base + ["--run-id", "v"] + _docs_args(two_node_inputs)
               + ["--xml", str(broken), "--sidecar", str(run / "schedule.json")], tmp_path)
    assert res.returncode != 0
