"""``python -m vericcl {solve,verify,calibrate,inspect,resume,manual-generate}`` (same CLI as ``python -m vericcl_b200``)."""
import sys

from vericcl_b200.cli.main import main

if __name__ == "__main__":
    sys.exit(main())
