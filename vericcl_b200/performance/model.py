"""Piecewise α/β cost model with component provenance.

Components are keyed ``link:s:d``, ``rrc:s:d``, ``copy:r``, ``reduce:r`` and
``mc_reduce:g`` / ``mc_store:g`` for NVLS group operations.  Each component is
a tuple of :class:`ServiceCost` segments over disjoint payload-size domains
with a source (initial / estimated / measured / history).  Shared resources
have capacities in bytes/µs; measured concurrency modes are
:class:`RateProfile` records (reference: vericcl/performance/model.py:74-159,
vericcl/performance/profiles.py:11).
"""
from __future__ import annotations

import math
from dataclasses import asdict, dataclass, field
from datetime import datetime
from types import MappingProxyType
from typing import Mapping

from vericcl_b200.errors import SemanticError

SOURCES = frozenset({"initial", "estimated", "measured", "history"})


def finite(value, name, *, positive=False) -> float:
    if isinstance(value, bool) or not isinstance(value, (int, float)) or not math.isfinite(value) or value < 0 \
            or (positive and value == 0):
        raise SemanticError(name + " must be finite and " + ("positive" if positive else "nonnegative"))
    return float(value)


@dataclass(frozen=True)
class ServiceCost:
    alpha_us: float
    beta_us_per_byte: float
    source: str = "initial"
    min_bytes: int = 1
    max_bytes: int | None = None
    measured_at: str | None = None

    def __post_init__(self):
        object.__setattr__(self, "alpha_us", finite(self.alpha_us, "alpha_us"))
        object.__setattr__(self, "beta_us_per_byte", finite(self.beta_us_per_byte, "beta_us_per_byte",
                                                            positive=True))
        if self.source not in SOURCES:
            raise SemanticError("invalid cost source " + repr(self.source))
        if isinstance(self.min_bytes, bool) or not isinstance(self.min_bytes, int) or self.min_bytes < 1:
            raise SemanticError("cost size domain must start at a positive byte count")
        if self.max_bytes is not None and (not isinstance(self.max_bytes, int) or self.max_bytes < self.min_bytes):
            raise SemanticError("cost size domain is invalid")
        if self.source in ("measured", "history"):
            if self.measured_at is None:
                raise SemanticError("measured costs need their measurement time")
            stamp = datetime.fromisoformat(self.measured_at.replace("Z", "+00:00"))
            if stamp.tzinfo is None:
                raise SemanticError("measurement timestamp needs a timezone")

    def covers(self, size: int) -> bool:
        return self.min_bytes <= size and (self.max_bytes is None or size <= self.max_bytes)

    def time_us(self, size: int) -> float:
        return self.alpha_us + self.beta_us_per_byte * size


@dataclass(frozen=True)
class RateProfile:
    """Measured per-flow rates (bytes/µs) for one concurrency mode."""

    profile_id: str
    flows: frozenset
    rates: Mapping[str, float]
    startup_us: Mapping[str, float] = field(default_factory=dict)
    source: str = "measured"

    def applies(self, group) -> bool:
        return frozenset(op.flow_id for op in group) == self.flows

    def as_json(self) -> dict:
        return {"profile_id": self.profile_id, "flows": sorted(self.flows), "rates": dict(self.rates),
                "startup_us": dict(self.startup_us), "source": self.source}


@dataclass(frozen=True)
class CostModel:
    version: str
    services: Mapping[str, tuple]
    resources: Mapping[str, float] = field(default_factory=dict)
    profiles: tuple = ()
    context: Mapping[str, object] = field(default_factory=dict)
    metadata: Mapping[str, object] = field(default_factory=dict)

    def __post_init__(self):
        if not isinstance(self.version, str) or not self.version:
            raise SemanticError("cost model needs a version identity")
        services = {}
        for key, values in self.services.items():
            values = tuple(sorted(values, key=lambda v: v.min_bytes))
            if not values or not all(isinstance(v, ServiceCost) for v in values):
                raise SemanticError("component %s must hold ServiceCost segments" % key)
            for left, right in zip(values, values[1:]):
                if left.max_bytes is None or left.max_bytes >= right.min_bytes:
                    raise SemanticError("service size domains overlap for " + key)
            services[key] = values
        resources = {k: finite(v, "resource capacity", positive=True) for k, v in self.resources.items()}
        if len({p.profile_id for p in self.profiles}) != len(self.profiles):
            raise SemanticError("duplicate profile identity")
        object.__setattr__(self, "services", MappingProxyType(services))
        object.__setattr__(self, "resources", MappingProxyType(resources))
        object.__setattr__(self, "profiles", tuple(self.profiles))
        object.__setattr__(self, "context", MappingProxyType(dict(self.context)))
        object.__setattr__(self, "metadata", MappingProxyType(dict(self.metadata)))

    def service_for(self, key: str, size: int) -> ServiceCost | None:
        return next((v for v in self.services.get(key, ()) if v.covers(size)), None)

    def with_updates(self, version, *, services=None, resources=None, profiles=None):
        """Return (new model, component diff); the version must change."""
        if version == self.version:
            raise SemanticError("a model update needs a new version identity")
        svc, res, changes = dict(self.services), dict(self.resources), []
        for key, value in (services or {}).items():
            old = self.services.get(key)
            svc[key] = tuple(value)
            changes.append({"component": "service:" + key,
                            "before": None if old is None else [asdict(c) for c in old],
                            "after": [asdict(c) for c in value]})
        for key, value in (resources or {}).items():
            changes.append({"component": "resource:" + key, "before": self.resources.get(key), "after": value})
            res[key] = value
        prof = self.profiles if profiles is None else tuple(profiles)
        if profiles is not None:
            changes.append({"component": "profiles", "before": [p.as_json() for p in self.profiles],
                            "after": [p.as_json() for p in prof]})
        return CostModel(version, svc, res, prof, self.context, self.metadata), tuple(changes)

    def as_json(self) -> dict:
        return {"version": self.version,
                "services": {k: [asdict(c) for c in v] for k, v in sorted(self.services.items())},
                "resources": dict(sorted(self.resources.items())),
                "profiles": [p.as_json() for p in self.profiles],
                "context": dict(self.context), "metadata": dict(self.metadata)}

    @classmethod
    def from_json(cls, doc: dict) -> "CostModel":
        return cls(doc["version"], {k: tuple(ServiceCost(**c) for c in v) for k, v in doc["services"].items()},
                   doc.get("resources", {}),
                   tuple(RateProfile(p["profile_id"], frozenset(p["flows"]), p["rates"], p.get("startup_us", {}),
                                     p.get("source", "measured")) for p in doc.get("profiles", ())),
                   doc.get("context", {}), doc.get("metadata", {}))
