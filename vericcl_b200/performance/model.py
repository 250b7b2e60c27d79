"""Cost model: per-component latency/bandwidth curves, resource capacities, measured sharing modes.

A component is a key naming one kind of work on specific hardware:
``link:s:d`` (a transfer s→d), ``rrc:s:d`` (receive, reduce and store),
``copy:r`` / ``reduce:r`` (local HBM work on rank r) and
``mc_reduce:g`` / ``mc_store:g`` (NVLS work of multicast group g).  Its curve
is a list of *segments*, each valid on a closed payload range and giving
``time(n) = alpha + beta * n``.  Segments remember where their numbers come
from (initial request, estimate, measurement, history) so predictions can say
how much of their time rests on measurements.

Capacities (bytes/µs) belong to shared resources; on an NVSwitch box these
are every GPU's NVLink transmit and receive ports (``nvlink-tx-r`` /
``nvlink-rx-r``), the switch's in-network reduction (``nvls-g``) and, on an
emulated multi-node box, the inter-group links.  A *sharing mode* is a set of
flows that were measured running together, with the rate each one reached.

The JSON layout and the component keys are the reference's exchange format
(vericcl/performance/model.py:74-159, vericcl/performance/profiles.py:11), so
model files move between the two; the code is this project's own.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field, fields
from datetime import datetime
from types import MappingProxyType
from typing import Mapping

from vericcl_b200.errors import SemanticError

PROVENANCE = ("initial", "estimated", "measured", "history")
_TIMED = ("measured", "history")


def _reject(msg: str):
    raise SemanticError(msg)


def real(value, what: str, *, strictly_positive: bool = False) -> float:
    """``value`` as a float after checking it is a real, finite, non-negative number (positive if asked)."""
    ok = isinstance(value, (int, float)) and not isinstance(value, bool) and math.isfinite(value)
    ok = ok and (value > 0 if strictly_positive else value >= 0)
    if not ok:
        _reject("%s=%r is not a %s number" % (what, value, "positive finite" if strictly_positive else
                                               "non-negative finite"))
    return float(value)


# the name the rest of the package imports
finite = real


def _byte_count(value, what: str) -> int:
    if isinstance(value, bool) or not isinstance(value, int):
        _reject("%s must be an integer byte count, got %r" % (what, value))
    return value


@dataclass(frozen=True)
class ServiceCost:
    """One segment of a component's curve: time(n) = alpha_us + beta_us_per_byte * n for n in [min, max]."""

    alpha_us: float
    beta_us_per_byte: float
    source: str = "initial"
    min_bytes: int = 1
    max_bytes: int | None = None
    measured_at: str | None = None

    def __post_init__(self):
        set_ = object.__setattr__
        set_(self, "alpha_us", real(self.alpha_us, "alpha_us"))
        set_(self, "beta_us_per_byte", real(self.beta_us_per_byte, "beta_us_per_byte", strictly_positive=True))
        if self.source not in PROVENANCE:
            _reject("segment provenance %r is not one of %s" % (self.source, ", ".join(PROVENANCE)))
        lo = _byte_count(self.min_bytes, "min_bytes")
        if lo <= 0:
            _reject("a segment covers payloads of at least one byte (min_bytes=%d)" % lo)
        if self.max_bytes is not None and _byte_count(self.max_bytes, "max_bytes") < lo:
            _reject("segment range [%d, %d] is empty" % (lo, self.max_bytes))
        if self.source in _TIMED:
            # a measured number is only comparable with others when we know when it was taken
            when = self.measured_at
            try:
                stamp = datetime.fromisoformat(str(when).replace("Z", "+00:00")) if when else None
            except ValueError:
                stamp = None
            if stamp is None or stamp.utcoffset() is None:
                _reject("a %s segment needs an ISO-8601 measured_at with a UTC offset, got %r" % (self.source, when))

    def covers(self, size: int) -> bool:
        return size >= self.min_bytes and (self.max_bytes is None or size <= self.max_bytes)

    def time_us(self, size: int) -> float:
        return self.alpha_us + self.beta_us_per_byte * size

    @property
    def rate_bytes_per_us(self) -> float:
        return 1.0 / self.beta_us_per_byte

    def to_json(self) -> dict:
        return {f.name: getattr(self, f.name) for f in fields(self)}


@dataclass(frozen=True)
class RateProfile:
    """A measured sharing mode: the flows in ``flows`` ran together at ``rates`` (bytes/µs each)."""

    profile_id: str
    flows: frozenset
    rates: Mapping[str, float]
    startup_us: Mapping[str, float] = field(default_factory=dict)
    source: str = "measured"

    def __post_init__(self):
        object.__setattr__(self, "flows", frozenset(self.flows))
        missing = self.flows - set(self.rates)
        if missing:
            _reject("sharing mode %s has no rate for %s" % (self.profile_id, sorted(missing)))
        object.__setattr__(self, "rates", MappingProxyType(
            {k: real(v, "rate of " + k, strictly_positive=True) for k, v in self.rates.items()}))
        object.__setattr__(self, "startup_us", MappingProxyType(dict(self.startup_us)))

    def applies(self, group) -> bool:
        """True when the active operations ``group`` are exactly this mode's flows."""
        return self.flows == frozenset(op.flow_id for op in group)

    def as_json(self) -> dict:
        return {"profile_id": self.profile_id, "flows": sorted(self.flows), "rates": dict(self.rates),
                "startup_us": dict(self.startup_us), "source": self.source}


def _curve(key: str, segments) -> tuple:
    """Segments of one component, ordered by payload and checked to be disjoint."""
    segs = sorted(tuple(segments), key=lambda s: s.min_bytes)
    if not segs:
        _reject("component %s has no segment" % key)
    for s in segs:
        if not isinstance(s, ServiceCost):
            _reject("component %s holds %r, not a ServiceCost" % (key, type(s).__name__))
    for lower, upper in zip(segs, segs[1:]):
        # an open-ended segment must be the last; a closed one must end before the next starts
        if lower.max_bytes is None or upper.min_bytes <= lower.max_bytes:
            _reject("component %s: segments starting at %d and %d overlap" % (key, lower.min_bytes,
                                                                              upper.min_bytes))
    return tuple(segs)


@dataclass(frozen=True)
class CostModel:
    """A versioned, immutable cost model (see the module docstring)."""

    version: str
    services: Mapping[str, tuple]
    resources: Mapping[str, float] = field(default_factory=dict)
    profiles: tuple = ()
    context: Mapping[str, object] = field(default_factory=dict)
    metadata: Mapping[str, object] = field(default_factory=dict)

    def __post_init__(self):
        if not (isinstance(self.version, str) and self.version.strip()):
            _reject("every cost model carries a non-empty version string")
        curves = {key: _curve(key, segs) for key, segs in self.services.items()}
        caps = {key: real(v, "capacity of " + key, strictly_positive=True) for key, v in self.resources.items()}
        profiles = tuple(self.profiles)
        seen = set()
        for p in profiles:
            if p.profile_id in seen:
                _reject("sharing mode %s appears twice" % p.profile_id)
            seen.add(p.profile_id)
        for name, value in (("services", curves), ("resources", caps), ("context", dict(self.context)),
                            ("metadata", dict(self.metadata))):
            object.__setattr__(self, name, MappingProxyType(value))
        object.__setattr__(self, "profiles", profiles)

    # -- queries -----------------------------------------------------------------
    def service_for(self, key: str, size: int) -> ServiceCost | None:
        """The segment of component ``key`` that covers a ``size``-byte payload (None when there is none)."""
        for seg in self.services.get(key, ()):
            if seg.covers(size):
                return seg
        return None

    def capacity(self, resource: str) -> float | None:
        return self.resources.get(resource)

    def measured_mode(self, group) -> RateProfile | None:
        """The measured sharing mode whose flows are exactly those of ``group`` (at most one may match)."""
        hits = [p for p in self.profiles if p.applies(group)]
        if len(hits) > 1:
            _reject("sharing modes %s all describe the same flows" % [p.profile_id for p in hits])
        return hits[0] if hits else None

    # -- evolution -----------------------------------------------------------------
    def with_updates(self, version, *, services=None, resources=None, profiles=None):
        """A successor model under a new version and the list of components that changed.

        ``services`` replaces whole curves, ``resources`` capacities, ``profiles`` the
        sharing modes.  Each change record holds the component name and its value
        before and after, in JSON form.
        """
        if version == self.version:
            _reject("an updated model must not reuse version %r" % version)
        curves, caps = dict(self.services), dict(self.resources)
        diff = []
        for key, segs in sorted((services or {}).items()):
            before = curves.get(key)
            curves[key] = tuple(segs)
            diff.append({"component": "service:" + key,
                         "before": [s.to_json() for s in before] if before is not None else None,
                         "after": [s.to_json() for s in segs]})
        for key, cap in sorted((resources or {}).items()):
            diff.append({"component": "resource:" + key, "before": caps.get(key), "after": cap})
            caps[key] = cap
        modes = self.profiles
        if profiles is not None:
            modes = tuple(profiles)
            diff.append({"component": "profiles", "before": [p.as_json() for p in self.profiles],
                         "after": [p.as_json() for p in modes]})
        successor = CostModel(version, curves, caps, modes, dict(self.context), dict(self.metadata))
        return successor, tuple(diff)

    # -- JSON ------------------------------------------------------------------------
    def as_json(self) -> dict:
        return {"version": self.version,
                "services": {key: [s.to_json() for s in segs] for key, segs in sorted(self.services.items())},
                "resources": {key: self.resources[key] for key in sorted(self.resources)},
                "profiles": [p.as_json() for p in self.profiles],
                "context": dict(self.context), "metadata": dict(self.metadata)}

    @classmethod
    def from_json(cls, doc: dict) -> "CostModel":
        curves = {key: tuple(ServiceCost(**seg) for seg in segs) for key, segs in doc["services"].items()}
        modes = tuple(RateProfile(p["profile_id"], frozenset(p["flows"]), p["rates"], p.get("startup_us", {}),
                                  p.get("source", "measured")) for p in doc.get("profiles", ()))
        return cls(doc["version"], curves, doc.get("resources", {}), modes, doc.get("context", {}),
                   doc.get("metadata", {}))
