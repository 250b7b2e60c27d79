"""Process groups, the symmetric peer-mapped heap and plan execution."""
from .comm import Communicator, PlanHandle

__all__ = ["Communicator", "PlanHandle"]
