"""A compact reduced ordered binary decision diagram (ROBDD) package.

Used to select batches of repair strategies: each strategy is a variable,
pairwise conflicts (strategies touching the same operation or resource) are
encoded as ¬(a ∧ b), and the batch is a satisfying assignment with the most
strategies.  Nodes are hash-consed in a unique table; ``apply`` is memoised
(the reference uses CUDD through the ``dd`` package:
vericcl/verification/bdd_backend.py:92-235; this is a self-contained
implementation of the same data structure).
"""
from __future__ import annotations


class BDD:
    FALSE = 0
    TRUE = 1

    def __init__(self):
        self.nodes = [(None, None, None), (None, None, None)]   # (var, low, high)
        self.unique = {}
        self._apply_cache = {}
        self.vars = []

    def var(self, name) -> int:
        if name not in self.vars:
            self.vars.append(name)
        return self._mk(self.vars.index(name), self.FALSE, self.TRUE)

    def _mk(self, v, lo, hi):
        if lo == hi:
            return lo
        key = (v, lo, hi)
        node = self.unique.get(key)
        if node is None:
            node = len(self.nodes)
            self.nodes.append(key)
            self.unique[key] = node
        return node

    def _var_of(self, u):
        return self.nodes[u][0] if u > 1 else len(self.vars) + 1

    def apply(self, op: str, u: int, v: int) -> int:
        key = (op, u, v)
        if key in self._apply_cache:
            return self._apply_cache[key]
        if u <= 1 and v <= 1:
            res = int({"and": u and v, "or": u or v, "xor": u != v, "imp": (not u) or v}[op])
        else:
            vu, vv = self._var_of(u), self._var_of(v)
            top = min(vu, vv)
            u0, u1 = (self.nodes[u][1], self.nodes[u][2]) if vu == top else (u, u)
            v0, v1 = (self.nodes[v][1], self.nodes[v][2]) if vv == top else (v, v)
            res = self._mk(top, self.apply(op, u0, v0), self.apply(op, u1, v1))
        self._apply_cache[key] = res
        return res

    def neg(self, u: int) -> int:
        return self.apply("xor", u, self.TRUE)

    def conj(self, items) -> int:
        out = self.TRUE
        for u in items:
            out = self.apply("and", out, u)
        return out

    def count(self, u: int) -> int:
        """Number of satisfying assignments over all declared variables."""
        memo = {}

        def rec(x, level):
            if x <= 1:
                return x * (2 ** (len(self.vars) - level))
            key = (x, level)
            if key in memo:
                return memo[key]
            v, lo, hi = self.nodes[x]
            skip = 2 ** (v - level)
            res = skip * (rec(lo, v + 1) + rec(hi, v + 1))
            memo[key] = res
            return res
        return rec(u, 0)

    def best_assignment(self, u: int, weights=None):
        """Satisfying assignment maximising the summed weight of true variables.

        Variables that a path skips are unconstrained there and are set true
        exactly when their weight is positive.
        """
        weights = weights or {name: 1.0 for name in self.vars}
        nvars = len(self.vars)
        memo = {}

        def free(lo, hi):
            assign = {}
            score = 0.0
            for level in range(lo, hi):
                name = self.vars[level]
                take = weights.get(name, 0.0) > 0
                assign[name] = take
                score += weights.get(name, 0.0) if take else 0.0
            return score, assign

        def rec(x):
            # best over variables from this node's level to the end
            if x == self.FALSE:
                return None
            if x == self.TRUE:
                return (0.0, {})
            if x in memo:
                return memo[x]
            v, lo, hi = self.nodes[x]
            best = None
            for value, child in ((False, lo), (True, hi)):
                sub = rec(child)
                if sub is None:
                    continue
                gap_score, gap = free(v + 1, self._var_of(child) if child > 1 else nvars)
                score = sub[0] + gap_score + (weights.get(self.vars[v], 0.0) if value else 0.0)
                if best is None or score > best[0]:
                    assign = dict(sub[1])
                    assign.update(gap)
                    assign[self.vars[v]] = value
                    best = (score, assign)
            memo[x] = best
            return best

        res = rec(u)
        if res is None:
            return None
        top = self._var_of(u) if u > 1 else nvars
        lead_score, lead = free(0, top)
        assign = dict(res[1])
        assign.update(lead)
        return assign


def select_compatible(strategies, conflicts, weights=None):
    """Largest-weight set of strategies with no conflicting pair, via a BDD."""
    bdd = BDD()
    names = [s for s in strategies]
    for name in names:
        bdd.var(name)
    constraint = bdd.TRUE
    for a, b in conflicts:
        clause = bdd.neg(bdd.apply("and", bdd.var(a), bdd.var(b)))
        constraint = bdd.apply("and", constraint, clause)
    assignment = bdd.best_assignment(constraint, weights)
    return [n for n in names if assignment and assignment.get(n)]
