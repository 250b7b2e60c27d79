"""Run the README's command blocks marked ``<!-- doc-test: cpu -->`` in a scratch directory."""
import os
import re
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def _blocks():
    text = (ROOT / "README.md").read_text()
    return re.findall(r"<!-- doc-test: cpu -->\s*```bash\n(.*?)```", text, flags=re.S)


def test_readme_has_marked_blocks():
    assert len(_blocks()) >= 2


@pytest.mark.parametrize("index", range(len(_blocks())))
def test_documented_command_block(index, tmp_path):
    script = _blocks()[index].replace("python ", sys.executable + " ")
    env = dict(os.environ, PYTHONPATH=str(ROOT) + os.pathsep + os.environ.get("PYTHONPATH", ""),
               CUDA_VISIBLE_DEVICES="")
    res = subprocess.run(["bash", "-e", "-c", script], cwd=tmp_path, env=env, capture_output=True, text=True,
                         timeout=900)
    assert res.returncode == 0, res.stdout[-2000:] + res.stderr[-2000:]
