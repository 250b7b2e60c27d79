"""Request input: schema DSL, loader, resolved records (reference layer L0)."""
from .loader import load_request, resolve_documents, parse_override
from .models import ResolvedInput, Hyperparameters, SolverConfig

__all__ = ["load_request", "resolve_documents", "parse_override", "ResolvedInput", "Hyperparameters",
           "SolverConfig"]
