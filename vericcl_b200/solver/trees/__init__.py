"""Constructive tree synthesis (method ``constructive_trees``)."""
from .construct import construct_network, construct_trees

__all__ = ["construct_network", "construct_trees"]
