"""CPU tier: bench.py's output contract. Rank 0 prints exactly one JSON line on standard output;
anything else written to file descriptor 1 during the run (Python prints, NCCL's version banner
from inside the library) goes to stderr."""

from __future__ import annotations

import json
import subprocess
import sys

from conftest import ROOT


def test_only_the_result_line_reaches_stdout():
    code = (
        "import os, sys\n"
        f"sys.path.insert(0, {str(ROOT)!r})\n"
        "import bench\n"
        "with bench.StdoutToStderr():\n"
        "    print('python noise')\n"
        "    os.write(1, b'NCCL version x.y.z\\n')\n"
        "    bench.emit(bench.json.dumps({'metric': 'm', 'value': 1.0}))\n"
        "    print('more noise')\n"
        "print('after the run')\n"
    )
    res = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=120)
    assert res.returncode == 0, res.stderr
    lines = res.stdout.splitlines()
    assert json.loads(lines[0]) == {"metric": "m", "value": 1.0}
    assert lines[1:] == ["after the run"]
    assert "python noise" in res.stderr and "NCCL version" in res.stderr and "more noise" in res.stderr
