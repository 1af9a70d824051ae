"""Shared test setup: import paths, the `gpu` marker and small helpers.

Tests marked `gpu` need a CUDA device (a B200) and call the CUDA library through its C ABI;
everything else runs on CPU. The oracle (oracle/) is the checker in both tiers.
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
PKG = ROOT / "zero-copy-gpu-vector-search-re-ranking-engine_b200"
for p in (ROOT, PKG, ROOT / "oracle"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device; calls the sm_100a library")


@pytest.fixture(scope="session")
def golden():
    d = ROOT / "tests" / "golden"
    return {name: np.load(d / f"{name}.npz") for name in ("formats", "scan_small", "kat")}


@pytest.fixture(scope="session")
def orc():
    import oracle

    oracle.lib()
    return oracle


@pytest.fixture(scope="session")
def zc():
    """The CUDA library binding; builds it in-tree if it is missing."""
    import zcgvs_sm100

    if not zcgvs_sm100.LIB_PATH.exists():
        zcgvs_sm100.build()
    zcgvs_sm100.lib()
    return zcgvs_sm100


def assert_topk_parity(gpu_idx, gpu_val, ref_scores, k, *, exact, tol=1e-4, id_base=0):
    """Checks a GPU top-k against the oracle's full score rows.

    exact=True (integer-valued paths): ids and scores must equal the oracle's (score desc,
    id asc) selection bit for bit. exact=False (float paths): every returned score must match
    the oracle's score of the returned id within `tol` (relative to max(1, |score|)), the list
    must be descending, and the id set may differ from the oracle's only among documents whose
    score is within `tol` of the k-th score (near-ties).
    """
    import oracle

    ref_idx, ref_val = oracle.topk(ref_scores, k, id_base)
    gpu_idx = np.asarray(gpu_idx).reshape(ref_idx.shape)
    gpu_val = np.asarray(gpu_val).reshape(ref_val.shape)
    if exact:
        np.testing.assert_array_equal(gpu_idx, ref_idx)
        np.testing.assert_array_equal(gpu_val, ref_val)
        return
    for q in range(ref_idx.shape[0]):
        row = ref_scores[q]
        ids = gpu_idx[q]
        assert (ids >= id_base).all() and (ids < id_base + row.shape[0]).all(), "id out of range"
        exact_scores = row[ids - id_base]
        scale = np.maximum(1.0, np.abs(exact_scores))
        assert np.all(np.abs(gpu_val[q] - exact_scores) <= tol * scale), "scores differ beyond tolerance"
        assert np.all(np.diff(gpu_val[q]) <= tol), "not descending"
        assert len(set(ids.tolist())) == k, "duplicate ids"
        kth = ref_val[q, -1]
        band = tol * max(1.0, abs(float(kth)))
        ref_set = set(ref_idx[q].tolist())
        for i in set(ids.tolist()) ^ ref_set:
            assert abs(float(row[i - id_base]) - float(kth)) <= 2 * band, f"id {i} is not a near-tie"
