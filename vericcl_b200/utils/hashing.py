"""Content digests used for identities (models, candidates, checkpoints)."""
from __future__ import annotations

import hashlib

from .jsonio import canonical_dumps


def sha256_hex(data) -> str:
    if isinstance(data, str):
        data = data.encode()
    return hashlib.sha256(data).hexdigest()


def digest(value) -> str:
    """sha256 of the canonical JSON form of ``value``."""
    return sha256_hex(canonical_dumps(value))
