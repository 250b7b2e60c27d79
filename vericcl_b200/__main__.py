"""``python -m vericcl_b200`` entry point (reference: vericcl/__main__.py:1-5)."""
import sys

from vericcl_b200.cli.main import main

if __name__ == "__main__":
    sys.exit(main())
