"""Decision-scope no-improvement certificates with exact rational evidence.

A repair round explores a finite scope: the incumbent plus every variant its
strategies produce (:func:`vericcl_b200.tuning.strategies.implementations`).
A certificate shows that no member of that scope beats the incumbent under
the current cost model, in one of two forms that an independent checker can
re-derive:

* ``bound`` — for scopes whose variants keep the incumbent's work (order,
  channel and allocation strategies only): an LP relaxation in the form
  min c·x, A·x ≥ b, x ≥ 0, whose single variable is the completion time and
  whose rows say it is at least the optimistic finish of every operation
  (release time, longest dependency chain, α plus bytes at the fastest rate
  the model allows anywhere, so contention can only add to it), with a dual
  vector y.  :func:`verify_lp_dual` checks y ≥ 0 and Aᵀy ≤ c in exact
  rationals; b·y is then a lower bound on every member's T_pred.
* ``leaves`` — one record per variant: its XML digest and its exact T_pred
  as a fraction (or why it cannot execute).  The checker regenerates and
  re-lowers every variant and compares.

Certificates bind the model version and digest, the incumbent XML digest and
the scope identity (digest of the strategy list), so they go stale when any
of them changes (reference: vericcl/solver/proof_bounds.py:38,
vericcl/verification/proof_check.py:120-260).
"""
from __future__ import annotations

import hashlib
import json
from dataclasses import dataclass
from fractions import Fraction

from vericcl_b200.errors import SemanticError

FIXED_WORK_FAMILIES = frozenset({"order", "channel", "allocation"})
GRAMMAR = "vericcl_b200.scope.v1"


def rational(value) -> Fraction:
    if isinstance(value, bool):
        raise SemanticError("rational evidence cannot hold booleans")
    if isinstance(value, Fraction):
        return value
    try:
        return Fraction(str(value))
    except (ValueError, ZeroDivisionError) as error:
        raise SemanticError("evidence must hold finite rationals: %r" % (value,)) from error


def _digest(doc) -> str:
    return hashlib.sha256(json.dumps(doc, sort_keys=True, separators=(",", ":")).encode()).hexdigest()


@dataclass(frozen=True)
class VerifiedBound:
    value: Fraction
    model_version: str
    scope_id: str
    certificate: dict

    @property
    def digest(self) -> str:
        return _digest(self.certificate)


def verify_lp_dual(*, matrix, rhs, objective, dual, model_version: str, scope_id: str) -> VerifiedBound:
    """Exact check of a dual certificate for min c·x s.t. A·x ≥ b, x ≥ 0; returns the bound b·y."""
    if not model_version or not scope_id:
        raise SemanticError("a bound needs the model and scope it belongs to")
    a = [[rational(v) for v in row] for row in matrix]
    b = [rational(v) for v in rhs]
    c = [rational(v) for v in objective]
    y = [rational(v) for v in dual]
    if len(a) != len(b) or len(y) != len(b) or any(len(row) != len(c) for row in a):
        raise SemanticError("dual certificate dimensions disagree")
    if any(v < 0 for v in y):
        raise SemanticError("dual multipliers must be nonnegative")
    for j in range(len(c)):
        if sum((a[i][j] * y[i] for i in range(len(a))), Fraction(0)) > c[j]:
            raise SemanticError("dual certificate violates A-transpose y <= c in column %d" % j)
    value = sum((bi * yi for bi, yi in zip(b, y)), Fraction(0))
    cert = {"form": "min_cx_Ax_ge_b_x_ge_0", "matrix": [[str(v) for v in row] for row in a],
            "rhs": [str(v) for v in b], "objective": [str(v) for v in c], "dual": [str(v) for v in y],
            "model_version": model_version, "scope_id": scope_id}
    return VerifiedBound(value, model_version, scope_id, cert)


def model_digest(model) -> str:
    return _digest(model.as_json())


def scope_id(strategies) -> str:
    return _digest([s.as_json() for s in strategies])


def fixed_work(strategies) -> bool:
    return all(s.family in FIXED_WORK_FAMILIES for s in strategies)


def optimistic_relaxation(executable, model):
    """(A, b, c) of the fixed-work relaxation: T ≥ optimistic finish of every operation.

    Each operation runs at the faster of its own service rate and the largest rate any measured sharing mode
    gives its flow (the only rates the simulator can give it), with no contention at all.
    """
    measured = {}
    for profile in model.profiles:
        for flow, rate in profile.rates.items():
            measured[flow] = max(measured.get(flow, Fraction(0)), rational(rate))
    ops = {op.operation_id: op for op in executable.operations}
    finish, pending = {}, dict(ops)
    while pending:
        ready = sorted(k for k, op in pending.items() if set(op.after) <= finish.keys())
        if not ready:
            raise SemanticError("relaxation dependencies contain a cycle")
        for key in ready:
            op = pending.pop(key)
            start = max([rational(op.release_us)] + [finish[d] for d in op.after])
            if op.kind == "nop":
                finish[key] = start
                continue
            cost = model.service_for(op.component, op.nbytes)
            if cost is None:
                raise SemanticError("the relaxation needs a service cost for " + op.component)
            rate = max(1 / rational(cost.beta_us_per_byte), measured.get(op.flow_id, Fraction(0)))
            finish[key] = start + rational(cost.alpha_us) + Fraction(op.nbytes) / rate
    bounds = [finish[k] for k in sorted(finish)] or [Fraction(0)]
    return [[1] for _ in bounds], [str(v) for v in bounds], [1]


def _incumbent_ratio(bundle) -> Fraction:
    ratio = bundle.prediction.exact_completion_ratio if bundle.prediction is not None else None
    if ratio is None:
        raise SemanticError("the incumbent has no exact prediction")
    return Fraction(*ratio)


def _leaf(strategy, index, bundle) -> dict:
    rec = {"key": "%s/%d" % (strategy.strategy_id, index),
           "xml_sha256": hashlib.sha256(bundle.xml.encode()).hexdigest() if bundle is not None else None}
    if bundle is None or not bundle.can_execute or bundle.prediction is None \
            or bundle.prediction.exact_completion_ratio is None:
        rec["status"] = "not_executable"
    else:
        num, den = bundle.prediction.exact_completion_ratio
        rec["status"] = "valid"
        rec["t_pred"] = "%d/%d" % (num, den)
    return rec


def _leaves(incumbent, strategies, lower, max_channels):
    from vericcl_b200.tuning.strategies import implementations
    out = []
    for strategy in strategies:
        for index, variant in enumerate(implementations(strategy, incumbent.network, lower.topology,
                                                        max_channels=max_channels)):
            try:
                bundle = lower(variant)
            except SemanticError:
                bundle = None
            out.append(_leaf(strategy, index, bundle))
    return out


def certify_scope(incumbent, strategies, model, *, lower, max_channels: int = 16, use_bound: bool = True) -> dict:
    """Certificate that no variant of ``strategies`` improves ``incumbent`` (or the evidence that one does)."""
    sid = scope_id(strategies)
    cert = {"schema": 1, "grammar": GRAMMAR, "scope_id": sid, "model_version": model.version,
            "model_digest": model_digest(model),
            "incumbent_xml_sha256": hashlib.sha256(incumbent.xml.encode()).hexdigest(),
            "incumbent_t_pred": "%d/%d" % incumbent.prediction.exact_completion_ratio,
            "bound": None, "leaves": []}
    incumbent_value = _incumbent_ratio(incumbent)
    if use_bound and fixed_work(strategies):
        a, b, c = optimistic_relaxation(incumbent.executable, model)
        top = max(range(len(b)), key=lambda i: rational(b[i]))
        bound = verify_lp_dual(matrix=a, rhs=b, objective=c, dual=[int(i == top) for i in range(len(b))],
                               model_version=model.version, scope_id=sid)
        if bound.value >= incumbent_value:
            cert["bound"] = bound.certificate
            return cert
    if incumbent.network is None:
        raise SemanticError("the incumbent has no network form to enumerate")
    cert["leaves"] = _leaves(incumbent, strategies, lower, max_channels)
    return cert


@dataclass(frozen=True)
class ProofResult:
    status: str              # proven_no_improvement | improvement_exists | stale | invalid | incomplete
    message: str
    checked_leaves: int = 0
    counterexample: dict | None = None


def check_no_improvement(certificate, incumbent, strategies, model, *, lower, max_channels: int = 16) -> ProofResult:
    """Independent re-derivation of a certificate from the incumbent, the strategies and the model."""
    if certificate.get("schema") != 1 or certificate.get("grammar") != GRAMMAR:
        return ProofResult("invalid", "unknown certificate grammar")
    if (certificate.get("model_version") != model.version or certificate.get("model_digest") != model_digest(model)
            or certificate.get("scope_id") != scope_id(strategies)
            or certificate.get("incumbent_xml_sha256") != hashlib.sha256(incumbent.xml.encode()).hexdigest()):
        return ProofResult("stale", "model, incumbent or scope changed since the certificate was made")
    incumbent_value = _incumbent_ratio(incumbent)
    if rational(certificate.get("incumbent_t_pred")) != incumbent_value:
        return ProofResult("invalid", "incumbent completion differs from the exact replay")
    if certificate.get("bound") is not None:
        if certificate.get("leaves"):
            return ProofResult("invalid", "a certificate holds either a bound or leaves, not both")
        if not fixed_work(strategies):
            return ProofResult("invalid", "the fixed-work relaxation does not cover path or structure variants")
        raw = certificate["bound"]
        a, b, c = optimistic_relaxation(incumbent.executable, model)
        canon = {"matrix": [[str(rational(v)) for v in row] for row in a], "rhs": [str(rational(v)) for v in b],
                 "objective": [str(rational(v)) for v in c]}
        for key, expected in canon.items():
            supplied = raw.get(key)
            got = [[str(rational(v)) for v in row] for row in supplied] if key == "matrix" and supplied is not None \
                else [str(rational(v)) for v in (supplied or [])]
            if got != expected:
                return ProofResult("invalid", "the submitted LP is not the reconstructed relaxation (%s)" % key)
        try:
            bound = verify_lp_dual(matrix=a, rhs=b, objective=c, dual=raw.get("dual", []),
                                   model_version=model.version, scope_id=certificate["scope_id"])
        except SemanticError as error:
            return ProofResult("invalid", str(error))
        if bound.value < incumbent_value:
            return ProofResult("incomplete", "the verified bound does not reach the incumbent")
        return ProofResult("proven_no_improvement", "the exact relaxation bound reaches the incumbent")
    expected = _leaves(incumbent, strategies, lower, max_channels)
    supplied = {rec["key"]: rec for rec in certificate.get("leaves", [])}
    if len(supplied) != len(certificate.get("leaves", [])):
        return ProofResult("invalid", "duplicate leaf claims")
    checked = 0
    for rec in expected:
        claim = supplied.pop(rec["key"], None)
        if claim is None:
            return ProofResult("incomplete", "variant %s has no evidence" % rec["key"], checked)
        if claim != rec:
            return ProofResult("invalid", "leaf %s does not match its re-derivation" % rec["key"], checked, rec)
        checked += 1
        if rec["status"] == "valid" and rational(rec["t_pred"]) < incumbent_value:
            return ProofResult("improvement_exists", "variant %s is faster" % rec["key"], checked, rec)
    if supplied:
        return ProofResult("invalid", "claims for variants outside the scope", checked)
    return ProofResult("proven_no_improvement", "every variant of the scope is at least as slow", checked)
