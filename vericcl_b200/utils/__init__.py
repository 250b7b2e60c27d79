"""Shared helpers: strict JSON, digests, atomic file IO, exact arithmetic."""
from .jsonio import strict_loads, strict_load, canonical_dumps, atomic_write_text, atomic_write_json
from .hashing import sha256_hex, digest

__all__ = ["strict_loads", "strict_load", "canonical_dumps", "atomic_write_text",
           "atomic_write_json", "sha256_hex", "digest"]
