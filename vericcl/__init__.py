"""``vericcl``: the module name the reference's users invoke (``python -m vericcl``).

The implementation lives in :mod:`vericcl_b200`; this package only forwards
the command line to it (reference entry point: vericcl/__main__.py:1-5).
"""
from vericcl_b200 import __version__  # noqa: F401
