"""A small MILP modelling layer solved with HiGHS (``scipy.optimize.milp``).

This is the package's replacement for the reference's SCIP adapter
(vericcl/solver/scip_api.py:97-278): variables with bounds and integrality,
sparse linear constraints, indicator-style big-M disjunctions, a warm-start
check, lexicographic multi-objective solving, a time limit and MIP gap, and
an *owned* mode that solves in a child process so a stuck solve can be
killed at its lease deadline (vericcl/solver/worker_scope.py:110-238).
Proven outcomes are cached by the model's content hash.
"""
from __future__ import annotations

import os
import pickle
import subprocess
import sys
import threading
import time
from contextlib import contextmanager
from dataclasses import dataclass, field
from pathlib import Path

import numpy as np

from vericcl_b200.errors import SolverError
from vericcl_b200.utils.hashing import digest

INF = float("inf")


@dataclass
class Var:
    index: int
    name: str
    lb: float
    ub: float
    integer: bool


@dataclass
class Solution:
    status: str                 # optimal | feasible | infeasible | timeout | error
    objective: float | None
    values: dict = field(default_factory=dict)
    gap: float | None = None
    runtime_s: float = 0.0
    message: str = ""

    @property
    def usable(self) -> bool:
        return self.status in ("optimal", "feasible") and self.values is not None

    def __getitem__(self, name):
        return self.values[name]


class Model:
    """Linear model: ``minimise c·x  s.t.  lo <= A x <= hi, lb <= x <= ub``."""

    def __init__(self, name: str = "model"):
        self.name = name
        self.vars: list[Var] = []
        self.by_name: dict[str, Var] = {}
        self.rows: list[tuple[dict, float, float, str]] = []
        self.objective: dict[int, float] = {}
        self.objective_constant = 0.0

    # -- variables ---------------------------------------------------------
    def add_var(self, name: str, lb: float = 0.0, ub: float = INF, integer: bool = False) -> Var:
        if name in self.by_name:
            raise SolverError("duplicate variable " + name)
        var = Var(len(self.vars), name, lb, ub, integer)
        self.vars.append(var)
        self.by_name[name] = var
        return var

    def binary(self, name: str) -> Var:
        return self.add_var(name, 0.0, 1.0, True)

    def continuous(self, name: str, lb: float = 0.0, ub: float = INF) -> Var:
        return self.add_var(name, lb, ub, False)

    # -- constraints -------------------------------------------------------
    def add(self, terms, lo: float = -INF, hi: float = INF, name: str = "") -> None:
        """Add ``lo <= sum(coef * var) <= hi``; ``terms`` is [(coef, Var)]."""
        row = {}
        for coef, var in terms:
            row[var.index] = row.get(var.index, 0.0) + float(coef)
        self.rows.append((row, float(lo), float(hi), name))

    def add_le(self, terms, rhs, name=""):
        self.add(terms, -INF, rhs, name)

    def add_ge(self, terms, rhs, name=""):
        self.add(terms, rhs, INF, name)

    def add_eq(self, terms, rhs, name=""):
        self.add(terms, rhs, rhs, name)

    def indicator_le(self, binary: Var, terms, rhs, big_m: float, name=""):
        """``binary = 1  =>  sum(terms) <= rhs`` via big-M."""
        self.add_le(list(terms) + [(big_m, binary)], rhs + big_m, name)

    def disjunction(self, a_end, b_start, b_end, a_start, order: Var, big_m: float, name=""):
        """Either a finishes before b starts (order=1) or b before a (order=0)."""
        self.add_le([(1, a_end), (-1, b_start), (big_m, order)], big_m, name + ":ab")
        self.add_le([(1, b_end), (-1, a_start), (-big_m, order)], 0.0, name + ":ba")

    def minimize(self, terms, constant: float = 0.0) -> None:
        self.objective = {}
        for coef, var in terms:
            self.objective[var.index] = self.objective.get(var.index, 0.0) + float(coef)
        self.objective_constant = constant

    # -- checks ------------------------------------------------------------
    def evaluate(self, values: dict) -> float:
        return self.objective_constant + sum(c * values[self.vars[i].name] for i, c in self.objective.items())

    def violated(self, values: dict, tol: float = 1e-6) -> list:
        """Names of constraints a candidate assignment violates (warm-start check)."""
        bad = []
        for var in self.vars:
            v = values.get(var.name)
            if v is None or v < var.lb - tol or v > var.ub + tol or (var.integer and abs(v - round(v)) > tol):
                bad.append("bound:" + var.name)
        for row, lo, hi, name in self.rows:
            total = sum(c * values.get(self.vars[i].name, 0.0) for i, c in row.items())
            if total < lo - tol or total > hi + tol:
                bad.append(name or "row")
        return bad

    def fingerprint(self) -> str:
        return digest({"v": [(v.name, v.lb if v.lb != -INF else "-inf", v.ub if v.ub != INF else "inf", v.integer)
                             for v in self.vars],
                       "r": [(sorted(r.items()), lo if lo != -INF else "-inf", hi if hi != INF else "inf")
                             for r, lo, hi, _ in self.rows],
                       "o": sorted(self.objective.items())})

    # -- solving -----------------------------------------------------------
    def arrays(self):
        n = len(self.vars)
        c = np.zeros(n)
        for i, coef in self.objective.items():
            c[i] = coef
        lb = np.array([v.lb for v in self.vars], dtype=float)
        ub = np.array([v.ub for v in self.vars], dtype=float)
        integrality = np.array([1 if v.integer else 0 for v in self.vars], dtype=np.uint8)
        if self.rows:
            from scipy.sparse import coo_matrix
            data, ri, ci, lo, hi = [], [], [], [], []
            for r, (row, rlo, rhi, _) in enumerate(self.rows):
                for i, coef in row.items():
                    data.append(coef)
                    ri.append(r)
                    ci.append(i)
                lo.append(rlo)
                hi.append(rhi)
            a = coo_matrix((data, (ri, ci)), shape=(len(self.rows), n)).tocsr()
            return c, lb, ub, integrality, a, np.array(lo), np.array(hi)
        return c, lb, ub, integrality, None, None, None

    def solve(self, *, time_limit: float = 60.0, mip_gap: float = 0.0, threads: int = 1) -> Solution:
        with _solver_output_to_stderr():
            return _solve_arrays(self.arrays(), [v.name for v in self.vars], self.objective_constant,
                                 time_limit, mip_gap)

    def solve_lp_duals(self, *, time_limit: float = 60.0):
        """Solve the LP relaxation and return ``(solution, duals)``: ``duals[r]`` = ∂objective/∂(bound of row r).

        For a ``≤`` row the dual is ≤ 0 (raising the bound can only lower the
        minimum), for a ``≥`` row ≥ 0, and an equality row's dual is free.  A
        row bounded on both sides reports the side that binds.  Integrality is
        ignored.
        """
        from scipy.optimize import linprog
        c, lb, ub, _, a, lo, hi = self.arrays()
        start = time.monotonic()
        ub_rows, ub_rhs, ub_sign, ub_of, eq_rows, eq_rhs, eq_of = [], [], [], [], [], [], []
        dense = a.toarray() if a is not None else np.zeros((0, len(c)))
        for r in range(dense.shape[0]):
            if lo[r] == hi[r]:
                eq_of.append(r)
                eq_rows.append(dense[r])
                eq_rhs.append(hi[r])
                continue
            if hi[r] != INF:
                ub_of.append(r)
                ub_rows.append(dense[r])
                ub_rhs.append(hi[r])
                ub_sign.append(1.0)
            if lo[r] != -INF:
                ub_of.append(r)
                ub_rows.append(-dense[r])
                ub_rhs.append(-lo[r])
                ub_sign.append(-1.0)
        with _solver_output_to_stderr():
            res = linprog(c, A_ub=np.array(ub_rows) if ub_rows else None, b_ub=ub_rhs or None,
                          A_eq=np.array(eq_rows) if eq_rows else None, b_eq=eq_rhs or None,
                          bounds=list(zip(lb, [None if u == INF else u for u in ub])), method="highs",
                          options={"time_limit": max(0.05, float(time_limit))})
        runtime = time.monotonic() - start
        if res.x is None or res.status != 0:
            # duals are only meaningful at a proven optimum: anything else (limit, infeasible, unbounded) is unusable
            status = {1: "timeout", 2: "infeasible"}.get(res.status, "error")
            return Solution(status, None, {}, None, runtime, str(res.message)), []
        duals = [0.0] * dense.shape[0]
        for k, r in enumerate(ub_of):
            value = float(res.ineqlin.marginals[k]) * ub_sign[k]
            if abs(value) > abs(duals[r]):
                duals[r] = value
        for k, r in enumerate(eq_of):
            duals[r] = float(res.eqlin.marginals[k])
        values = {v.name: float(x) for v, x in zip(self.vars, res.x)}
        return Solution("optimal", float(res.fun) + self.objective_constant, values, None, runtime,
                        str(res.message)), duals


_QUIET_LOCK = threading.Lock()
_QUIET = {"depth": 0, "saved": None}


@contextmanager
def _solver_output_to_stderr():
    """Send what the solver library prints on file descriptor 1 to standard error for the block.

    The package's commands print JSON lines on standard output; the HiGHS
    library writes progress text straight to descriptor 1.  Nested and
    concurrent blocks share one redirection, restored when the last one ends.
    """
    with _QUIET_LOCK:
        if _QUIET["depth"] == 0:
            try:
                sys.stdout.flush()
                _QUIET["saved"] = os.dup(1)
                os.dup2(2, 1)
            except (OSError, ValueError):
                _QUIET["saved"] = None
        _QUIET["depth"] += 1
    try:
        yield
    finally:
        with _QUIET_LOCK:
            _QUIET["depth"] -= 1
            if _QUIET["depth"] == 0 and _QUIET["saved"] is not None:
                os.dup2(_QUIET["saved"], 1)
                os.close(_QUIET["saved"])
                _QUIET["saved"] = None


def _solve_arrays(arrays, names, constant, time_limit, mip_gap) -> Solution:
    from scipy.optimize import Bounds, LinearConstraint, milp
    c, lb, ub, integrality, a, lo, hi = arrays
    start = time.monotonic()
    constraints = [] if a is None else [LinearConstraint(a, lo, hi)]
    options = {"time_limit": max(0.05, float(time_limit)), "mip_rel_gap": float(mip_gap), "disp": False}
    try:
        res = milp(c, constraints=constraints, integrality=integrality, bounds=Bounds(lb, ub), options=options)
    except Exception as error:  # pragma: no cover - scipy internal failure
        return Solution("error", None, {}, None, time.monotonic() - start, str(error))
    runtime = time.monotonic() - start
    if res.x is None:
        status = "infeasible" if res.status == 2 else "timeout" if res.status == 1 else "error"
        return Solution(status, None, {}, None, runtime, str(res.message))
    values = {name: float(v) for name, v in zip(names, res.x)}
    gap = getattr(res, "mip_gap", None)
    status = "optimal" if res.status == 0 else "feasible"
    return Solution(status, float(res.fun) + constant, values, gap, runtime, str(res.message))


_CACHE: dict[str, Solution] = {}


def _worker_main() -> None:
    """Child side of an owned solve: a pickled problem on stdin, the pickled :class:`Solution` on stdout."""
    arrays, names, constant, time_limit, mip_gap = pickle.load(sys.stdin.buffer)
    # the solver library may print to file descriptor 1: keep the result channel to ourselves
    result_fd = os.dup(1)
    os.dup2(2, 1)
    try:
        result = _solve_arrays(arrays, names, constant, time_limit, mip_gap)
    except BaseException as error:  # pragma: no cover
        result = Solution("error", None, {}, None, 0.0, repr(error))
    with os.fdopen(result_fd, "wb") as channel:
        channel.write(pickle.dumps(result))


def solve_owned(model: Model, *, time_limit: float = 60.0, mip_gap: float = 0.0, grace_s: float = 5.0,
                use_cache: bool = True) -> Solution:
    """Solve in a fresh child process that is killed if it outlives its lease.

    The child is a new interpreter running :func:`_worker_main`, not a fork:
    forking a process in which HiGHS has already run copies its thread pool's
    locks in a held state and the child's solve never starts.  Proven-optimal
    outcomes are cached by model fingerprint, so identical subproblems
    (isomorphic templates) are solved once.
    """
    key = model.fingerprint() + ":%g" % mip_gap
    if use_cache and key in _CACHE:
        return _CACHE[key]
    payload = pickle.dumps((model.arrays(), [v.name for v in model.vars], model.objective_constant,
                            time_limit, mip_gap))
    root = str(Path(__file__).resolve().parents[2])
    env = dict(os.environ, PYTHONPATH=root + os.pathsep + os.environ.get("PYTHONPATH", ""))
    proc = subprocess.Popen([sys.executable, "-c", "from vericcl_b200.solver.milp import _worker_main; "
                             "_worker_main()"], stdin=subprocess.PIPE,
                            stdout=subprocess.PIPE, stderr=subprocess.PIPE, env=env, start_new_session=True)
    try:
        out, err = proc.communicate(payload, timeout=time_limit + grace_s)
    except subprocess.TimeoutExpired:
        proc.kill()
        proc.communicate()
        return Solution("timeout", None, {}, None, time_limit, "owned solver exceeded its lease")
    try:
        result = pickle.loads(out)
    except Exception:
        tail = err.decode(errors="replace")[-300:]
        result = Solution("error", None, {}, None, 0.0, "solver worker exited %s without a result: %s"
                          % (proc.returncode, tail))
    if use_cache and result.status == "optimal":
        _CACHE[key] = result
    return result


def solve_lexicographic(model: Model, objectives, *, time_limit: float = 60.0, mip_gap: float = 0.0,
                        tolerance: float = 1e-6, owned: bool = False) -> Solution:
    """Solve objectives in priority order, fixing each optimum before the next."""
    best = None
    for level, terms in enumerate(objectives):
        model.minimize(terms)
        sol = solve_owned(model, time_limit=time_limit, mip_gap=mip_gap) if owned else \
            model.solve(time_limit=time_limit, mip_gap=mip_gap)
        if not sol.usable:
            return best if best is not None else sol
        best = sol
        if level + 1 < len(objectives):
            model.add_le(list(terms), sol.objective + tolerance * max(1.0, abs(sol.objective)),
                         name="lex%d" % level)
    return best
