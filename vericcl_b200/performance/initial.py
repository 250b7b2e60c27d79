"""Initial cost model from the request's explicit components.

Link components come from ``directed_links``; local ``copy``/``reduce`` from
``local_costs``; an ``rrc`` (receive-reduce-copy) estimate is link + the
receiver's reduce (marked ``estimated`` and replaced by a measured rrc later);
NVLS group components ``mc_reduce:<g>``/``mc_store:<g>`` are estimated from
the slowest member link.  No missing component is ever filled with zero
(reference: vericcl/performance/initial.py:8-40).
"""
from __future__ import annotations

from dataclasses import asdict

from vericcl_b200.performance.model import CostModel, ServiceCost
from vericcl_b200.utils.hashing import digest


def model_context(request) -> dict:
    return {"datatype": request.collective.datatype, "reduction_op": request.collective.reduction_op,
            "protocol": request.request_config["runtime"]["protocol"]}


def initial_cost_model(request) -> CostModel:
    topology = request.request_config["topology"]
    services, resources, estimates = {}, {}, {}
    for item in topology["local_costs"]:
        for kind in ("copy", "reduce"):
            if kind in item:
                services["%s:%d" % (kind, item["rank"])] = (ServiceCost(**dict(item[kind])),)
    for edge in topology["directed_links"]:
        suffix = "%d:%d" % (edge["src"], edge["dst"])
        link = ServiceCost(edge["alpha_us"], edge["beta_us_per_byte"])
        services["link:" + suffix] = (link,)
        resources["link:" + suffix] = 1.0 / link.beta_us_per_byte
        local = services.get("reduce:%d" % edge["dst"])
        if local:
            red = local[0]
            services["rrc:" + suffix] = (ServiceCost(link.alpha_us + red.alpha_us,
                                                     link.beta_us_per_byte + red.beta_us_per_byte,
                                                     source="estimated"),)
            estimates["rrc:" + suffix] = {"formula": "link + receiver reduce",
                                          "components": ["link:" + suffix, "reduce:%d" % edge["dst"]]}
    resources.update({item["id"]: item["capacity_bytes_per_us"] for item in topology["shared_resources"]})
    links = {(e["src"], e["dst"]): e for e in topology["directed_links"]}
    for index, group in enumerate(topology.get("multicast_groups", ())):
        members = [links[(a, b)] for a in group for b in group if a != b and (a, b) in links]
        if not members:
            continue
        alpha = max(e["alpha_us"] for e in members)
        beta = max(e["beta_us_per_byte"] for e in members)
        for kind in ("mc_reduce", "mc_store"):
            services["%s:%d" % (kind, index)] = (ServiceCost(alpha, beta, source="estimated"),)
        estimates["mc:%d" % index] = {"formula": "slowest member link", "group": list(group)}
    required = {"copy:%d" % r for r in range(request.rank_count)}
    if request.collective.reduction_op is not None:
        required |= {"reduce:%d" % r for r in range(request.rank_count)}
        required |= {"rrc:%d:%d" % (e["src"], e["dst"]) for e in topology["directed_links"]}
    context = {"datatype": request.collective.datatype, "reduction_op": request.collective.reduction_op,
               "protocol": request.request_config["runtime"]["protocol"]}
    metadata = {"origin": "explicit_request", "initial_estimates": estimates,
                "missing_initial_components": sorted(required - services.keys())}
    version = "initial-" + digest({"services": {k: [asdict(c) for c in v] for k, v in services.items()},
                                   "resources": resources, "context": context})[:24]
    return CostModel(version, services, resources, context=context, metadata=metadata)
