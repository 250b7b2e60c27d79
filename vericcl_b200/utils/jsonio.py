"""Strict JSON parsing and atomic, fsync'd writes.

Mirrors the reference's input contract (docs/input-schema.md:3): duplicate
keys, non-finite numbers and excessive nesting are rejected, and published
files are replaced atomically (vericcl/execution/context.py atomic writes).
"""
from __future__ import annotations

import json
import math
import os
import tempfile
from pathlib import Path

from vericcl_b200.errors import InputValidationError

MAX_DEPTH = 64


def _reject_duplicates(pairs):
    result = {}
    for key, value in pairs:
        if key in result:
            raise InputValidationError("duplicate JSON key: %r" % (key,))
        result[key] = value
    return result


def _reject_constant(token):
    raise InputValidationError("non-finite JSON number: %s" % token)


def _depth(value, level=0):
    if level > MAX_DEPTH:
        raise InputValidationError("JSON nesting exceeds %d levels" % MAX_DEPTH)
    if isinstance(value, dict):
        for item in value.values():
            _depth(item, level + 1)
    elif isinstance(value, list):
        for item in value:
            _depth(item, level + 1)


def strict_loads(text: str):
    """Parse JSON text; reject duplicate keys, NaN/Infinity and deep nesting."""
    try:
        value = json.loads(text, object_pairs_hook=_reject_duplicates, parse_constant=_reject_constant)
    except json.JSONDecodeError as error:
        raise InputValidationError("invalid JSON: %s" % error) from error
    _depth(value)
    return value


def strict_load(path) -> object:
    return strict_loads(Path(path).read_text())


def _finite(value):
    if isinstance(value, float) and not math.isfinite(value):
        raise InputValidationError("non-finite number cannot be serialised")
    if isinstance(value, dict):
        for item in value.values():
            _finite(item)
    elif isinstance(value, (list, tuple)):
        for item in value:
            _finite(item)


def canonical_dumps(value) -> str:
    """Deterministic JSON text (sorted keys, compact separators)."""
    _finite(value)
    return json.dumps(value, sort_keys=True, separators=(",", ":"), allow_nan=False)


def atomic_write_text(path, text: str, mode: int | None = None) -> Path:
    """Write ``text`` to ``path`` through a temporary file, fsync, rename."""
    path = Path(path)
    path.parent.mkdir(parents=True, exist_ok=True)
    fd, tmp = tempfile.mkstemp(prefix="." + path.name + ".", dir=str(path.parent))
    try:
        with os.fdopen(fd, "w") as handle:
            handle.write(text)
            handle.flush()
            os.fsync(handle.fileno())
        if mode is not None:
            os.chmod(tmp, mode)
        os.replace(tmp, path)
        dirfd = os.open(str(path.parent), os.O_RDONLY)
        try:
            os.fsync(dirfd)
        finally:
            os.close(dirfd)
    except BaseException:
        if os.path.exists(tmp):
            os.unlink(tmp)
        raise
    return path


def atomic_write_json(path, value, *, indent: int | None = 2, mode: int | None = None) -> Path:
    _finite(value)
    text = json.dumps(value, indent=indent, sort_keys=True, allow_nan=False) + "\n"
    return atomic_write_text(path, text, mode)
