"""Calibration campaign: probe → qualify → fit → publish a new model version.

Probe groups run in priority order (intra-node links, local, inter-node
links, shared modes).  Each job is executed by a probe executor (the native
multi-GPU worker, or an injected fake in tests), its samples are qualified
and fitted, and qualified components replace the model's estimates in a new
model version whose diff is recorded.  Shared-mode jobs become measured
``RateProfile`` rate vectors.  A calibration cache keyed by the exact
runtime identity (devices, driver, datatype, mode) lets later runs reuse
components (reference: vericcl/verification/online/campaign.py:35,
model_publication.py:62, component_cache.py:65-95).
"""
from __future__ import annotations

import json
import time
from dataclasses import asdict
from datetime import datetime, timezone
from pathlib import Path

from vericcl_b200.errors import BudgetExhausted, RuntimeFailure
from vericcl_b200.online.fitting import Sample, fit_curve, qualify
from vericcl_b200.online.probe_jobs import plan_probes
from vericcl_b200.performance.model import RateProfile, ServiceCost
from vericcl_b200.utils.hashing import digest


def publish_model(model, fitted: dict, profiles=(), *, stamp: str | None = None):
    """New model version from fitted components ``{component: [Segment]}``."""
    stamp = stamp or datetime.now(timezone.utc).isoformat()
    services = {}
    for component, segments in fitted.items():
        services[component] = tuple(ServiceCost(s.alpha_us, s.beta_us_per_byte, "measured", s.min_bytes,
                                                s.max_bytes, stamp) for s in segments)
    version = "measured-" + digest({"base": model.version, "services": {k: [asdict(c) for c in v]
                                                                         for k, v in services.items()},
                                    "profiles": [p.as_json() for p in profiles]})[:24]
    merged_profiles = None
    if profiles:
        # a new measurement of a sharing mode replaces the old one: same id, or the same set of flows (two modes
        # of one flow set would make the prediction ambiguous)
        fresh_ids = {p.profile_id for p in profiles}
        fresh_flows = {p.flows for p in profiles}
        kept = [p for p in model.profiles if p.profile_id not in fresh_ids and p.flows not in fresh_flows]
        merged_profiles = tuple(kept) + tuple(profiles)
    return model.with_updates(version, services=services, profiles=merged_profiles)


def run_calibration(request, topology, model, executor, *, lease=None, max_channels: int = 1, record_dir=None):
    """Run every probe job through ``executor(job) -> [Sample]``; return (model, report)."""
    cfg = request.request_config["sketch"]["calibration"]
    jobs = plan_probes(request, topology, max_channels=max_channels)
    fitted, profiles, report = {}, [], {"jobs": [], "rejected": {}}
    for job in jobs:
        if lease is not None:
            try:
                lease.check()
            except BudgetExhausted:
                report["stopped"] = "online budget exhausted"
                break
        try:
            samples = executor(job)
        except RuntimeFailure as error:
            report["rejected"][job.job_id] = str(error)
            continue
        report["jobs"].append({"job": job.job_id, "samples": len(samples)})
        if job.mode == "shared":
            rates = {}
            for flow in job.flows:
                mine = [s for s in samples if s.component == flow.flow_id]
                good, reasons = qualify(mine, max_cv=cfg["max_cv"])
                if not good:
                    break
                biggest = max(s.bytes for s in good)
                t = sorted(s.time_us for s in good if s.bytes == biggest)[len(good) // 2 if False else 0]
                rates[flow.flow_id] = biggest / t
            if len(rates) == len(job.flows):
                profiles.append(RateProfile(job.job_id, frozenset(rates), rates))
            continue
        flow = job.flows[0]
        good, reasons = qualify(samples, max_cv=cfg["max_cv"])
        if reasons:
            report["rejected"][job.job_id] = reasons
        if not good:
            continue
        try:
            segments = fit_curve(good, max_relative_error=cfg["max_relative_fit_error"])
        except RuntimeFailure as error:
            report["rejected"][job.job_id] = str(error)
            continue
        if any(s.relative_error > cfg["max_relative_fit_error"] for s in segments):
            report["rejected"][job.job_id] = "fit error above the limit"
            continue
        fitted[flow.component] = segments
    if cfg.get("probe_scope", "every_link") == "link_classes" and fitted:
        # a class representative's fit stands for every member of its class (and a node's probed rank for
        # the node's other ranks); the report names what stood for what
        from vericcl_b200.online.probe_jobs import representatives
        _, stands_for, local_ranks = representatives(topology)
        extended = dict(fitted)
        for component, segments in fitted.items():
            kind, _, suffix = component.partition(":")
            if kind in ("link", "rrc"):
                for member in stands_for.get(suffix, ()):
                    extended.setdefault("%s:%s" % (kind, member), segments)
            elif kind in ("copy", "reduce"):
                rank = int(suffix)
                node = topology.node_of(rank)
                for other in node.ranks:
                    extended.setdefault("%s:%d" % (kind, other), segments)
        report["represented"] = sorted(set(extended) - set(fitted))
        fitted = extended
    if not fitted and not profiles:
        return model, [], report
    new_model, diff = publish_model(model, fitted, profiles)
    report["published"] = new_model.version
    if record_dir is not None:
        path = Path(record_dir)
        path.mkdir(parents=True, exist_ok=True)
        (path / (new_model.version + ".json")).write_text(json.dumps(new_model.as_json(), indent=2))
        (path / (new_model.version + ".diff.json")).write_text(json.dumps(list(diff), indent=2, default=str))
    return new_model, list(diff), report


def calibration_identity(request, device_names=(), driver: str = "") -> str:
    return digest({"devices": list(device_names), "driver": driver, "datatype": request.collective.datatype,
                   "reduction": request.collective.reduction_op, "ranks": request.rank_count})


def save_calibration(index_path, identity: str, model) -> None:
    from vericcl_b200.utils.jsonio import atomic_write_json
    path = Path(index_path)
    data = json.loads(path.read_text()) if path.exists() else {}
    data[identity] = {"model": model.as_json(), "saved": time.time()}
    atomic_write_json(path, data)


def lookup_calibration(index_path, identity: str, max_age_s: float):
    from vericcl_b200.performance.model import CostModel
    path = Path(index_path)
    if not path.exists():
        return None
    entry = json.loads(path.read_text()).get(identity)
    if entry is None or time.time() - entry["saved"] > max_age_s:
        return None
    return CostModel.from_json(entry["model"])


def simulated_executor(topology, *, seed: int = 0, noise: float = 0.01, source: str = "test_simulation"):
    """Analytic probe executor for tests: t = α + β·bytes with small noise (never qualifies as native)."""
    import random
    rng = random.Random(seed)

    def run(job):
        out = []
        for size in job.payload_sizes:
            for launch in range(4):
                for flow in job.flows:
                    if flow.kind in ("copy", "reduce"):
                        t = 1.0 + size / 3.0e6
                    else:
                        from vericcl_b200.topology.model import LinkKey
                        link = topology.link(LinkKey(flow.src, flow.dst))
                        t = link.alpha_us + link.beta_us_per_byte * size * (len(job.flows) if job.mode == "shared" else 1)
                    out.append(Sample(flow.flow_id if job.mode == "shared" else flow.component, size,
                                      t * (1 + noise * rng.uniform(-1, 1)), source, launch))
        return out
    return run
