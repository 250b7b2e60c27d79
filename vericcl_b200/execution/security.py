"""Redaction of secrets in logged payloads (reference: vericcl/execution/security.py:29-115)."""
from __future__ import annotations

import re

SECRET_KEYS = re.compile(r"(pass(word)?|secret|token|key|credential|auth)", re.IGNORECASE)
SECRET_VALUES = [re.compile(p) for p in (r"(?i)bearer\s+[a-z0-9._\-]+", r"ghp_[A-Za-z0-9]{20,}",
                                         r"-----BEGIN [A-Z ]*PRIVATE KEY-----")]
ENVIRONMENT_ALLOWLIST = frozenset({"CUDA_HOME", "CUDA_VISIBLE_DEVICES", "LD_LIBRARY_PATH", "NCCL_BUFFSIZE",
                                   "NCCL_NVLS_ENABLE", "NCCL_PROTO", "NCCL_ALGO", "PATH", "PYTHONPATH",
                                   "OMP_NUM_THREADS", "VERICCL_NVLS", "VERICCL_HEAP_BYTES"})


class Redactor:
    def __init__(self, extra_values=()):
        self.values = [v for v in extra_values if v]

    def redact(self, value):
        if isinstance(value, dict):
            return {k: ("<redacted>" if SECRET_KEYS.search(str(k)) and not isinstance(v, (int, float, bool))
                        else self.redact(v)) for k, v in value.items()}
        if isinstance(value, (list, tuple)):
            return [self.redact(v) for v in value]
        if isinstance(value, str):
            out = value
            for literal in self.values:
                out = out.replace(literal, "<redacted>")
            for pattern in SECRET_VALUES:
                out = pattern.sub("<redacted>", out)
            return out
        return value


def filtered_environment(env: dict) -> dict:
    return {k: v for k, v in env.items() if k in ENVIRONMENT_ALLOWLIST}
