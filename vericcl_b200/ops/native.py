"""Loading of the in-tree native modules.

``plan()`` returns the schedule compiler / CPU interpreter module and builds
it on first use when it is missing (a g++ build of a few seconds).  ``cuda()``
returns the CUDA extension; on a machine with a GPU a missing or broken CUDA
extension is an error, never a silent fallback.
"""
from __future__ import annotations

import importlib.util
import sys
import threading

from vericcl_b200.errors import NativeUnavailable

_lock = threading.Lock()
_modules: dict = {}


def _load(name: str, path):
    spec = importlib.util.spec_from_file_location(name, str(path))
    module = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(module)
    sys.modules[name] = module
    return module


def plan():
    with _lock:
        if "plan" not in _modules:
            from vericcl_b200.ops.build import build_plan_module
            try:
                path = build_plan_module()
            except Exception as error:
                raise NativeUnavailable("cannot build the schedule compiler: %s" % error) from error
            _modules["plan"] = _load("_vbplan", path)
        return _modules["plan"]


def cuda():
    with _lock:
        if "cuda" not in _modules:
            import torch  # noqa: F401  (loads libtorch before the extension)
            from vericcl_b200.ops.build import build_cuda_module
            try:
                path = build_cuda_module()
            except Exception as error:
                raise NativeUnavailable("cannot build the CUDA extension: %s" % error) from error
            _modules["cuda"] = _load("_vbcuda", path)
        return _modules["cuda"]


def cuda_available() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False
