"""The package's searcher_e2e program (bench.py's e2e_searcher): the end-to-end query rate
through the C++ drop-in Searcher (Searcher::search on a host query, then copyResultToHost, the
reference caller's sequence, src/search/searcher.cpp:344-397). Small shapes: the program runs,
replays its CUDA graph and reports the fields bench.py reads."""

from __future__ import annotations

import json
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
EXE = ROOT / "zero-copy-gpu-vector-search-re-ranking-engine_b200" / "searcher_e2e"

pytestmark = pytest.mark.gpu


def run(*args):
    assert EXE.exists(), f"{EXE} is not built"
    res = subprocess.run([str(EXE), *args], capture_output=True, text=True, timeout=300)
    assert res.returncode == 0, res.stderr
    return json.loads(res.stdout.strip().splitlines()[-1])


@pytest.mark.parametrize("dtype,dim", [(4, 768), (0, 384), (1, 384)])
def test_dense_searcher_rate(dtype, dim):
    out = run("docs=20000", f"dim={dim}", f"dtype={dtype}", "k=10", "metric=0", "steps=50", "warmup=5")
    assert out["steps"] == 50 and out["graph"] is True
    assert out["queries_per_s"] > 0 and out["ms_per_query"] > 0 and out["search_gpu_ms_mean"] > 0
    assert out["h2d_bytes_per_step"] == dim * 4 and out["d2h_bytes_per_step"] == 10 * 8


def test_hybrid_searcher_rate():
    out = run("docs=20000", "dim=384", "dtype=1", "k=10", "metric=0", "steps=50", "warmup=5", "vocab=3000",
              "mean_len=40", "terms=12", "weight=0.5")
    assert out["graph"] is True and out["queries_per_s"] > 0
    assert out["h2d_bytes_per_step"] == 384 * 4 + 12 * 4
