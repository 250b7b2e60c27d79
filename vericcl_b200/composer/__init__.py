"""Schedule composition (reference: vericcl/composer/)."""
from .compose import NetworkCandidate, NetworkOperation, compose_routes, list_schedule

__all__ = ["NetworkCandidate", "NetworkOperation", "compose_routes", "list_schedule"]
