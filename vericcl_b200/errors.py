"""Error hierarchy and CLI exit codes.

The exit codes follow the reference CLI contract (vericcl/cli/main.py:57-80):
2 = invalid input, 5 = semantic/verification failure, 7 = budget exhausted,
8 = runtime/native failure, 130 = interrupted.
"""


class VericclError(Exception):
    """Base class of every error raised by this package."""

    exit_code = 8


class InputValidationError(VericclError):
    """One of the four JSON documents (or an override) is invalid."""

    exit_code = 2


class SemanticError(VericclError):
    """A schedule, plan or program violates collective or storage semantics."""

    exit_code = 5


class ScratchBudgetError(SemanticError):
    """The scratch budget cannot hold a schedule's execution order; ``needed_bytes`` would."""

    def __init__(self, message: str, needed_bytes: int):
        super().__init__(message)
        self.needed_bytes = needed_bytes


class SolverError(VericclError):
    """The MILP backend failed or returned an unusable result."""

    exit_code = 5


class BudgetExhausted(VericclError):
    """A stage lease or the run's wall-clock limit ran out."""

    exit_code = 7


class RuntimeFailure(VericclError):
    """Native execution, a probe or the control plane failed."""

    exit_code = 8


class NativeUnavailable(RuntimeFailure):
    """The compiled extension is missing where native code is required."""
