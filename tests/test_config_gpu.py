"""GPU tier: one search from a JSON config (the reference's config file format), through the C++
loader (configFromJsonFile), the stores it names (EmbeddingStore::loadFromFile, with relative
paths resolved against the config's directory and its parent) and a VectorEngine built from its
search fields; the result equals the oracle's coarse-plus-rescore pipeline."""

from __future__ import annotations

import json
import os
import shutil
import subprocess

import numpy as np
import pytest

from conftest import PKG, ROOT

import formats  # noqa: E402

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def driver(zc, tmp_path_factory):
    exe = tmp_path_factory.mktemp("cpp") / "config_search"
    cuda = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    cxx = shutil.which("g++") or shutil.which("c++")
    cmd = [cxx, "-std=c++17", "-O2", f"-I{ROOT / 'include'}", f"-I{cuda}/include",
           str(ROOT / "tests/cpp/config_search.cpp"), "-o", str(exe), f"-L{PKG}", "-lzcgvs_sm100",
           f"-L{cuda}/lib64", "-lcudart", f"-Wl,-rpath,{PKG}"]
    subprocess.run(cmd, check=True, capture_output=True, text=True)
    return exe


def test_search_from_a_json_config(driver, orc, tmp_path):
    n, dim, batch = 20_000, 256, 4
    corpus = orc.normal_rows(n, dim, 1212)
    (tmp_path / "data").mkdir()
    (tmp_path / "configs").mkdir()
    formats.write_embeddings(tmp_path / "data" / "coarse.zcve", corpus, normalized=True, dtype="int8_row")
    formats.write_embeddings(tmp_path / "data" / "fine.zcve", corpus, normalized=True, dtype="float16")
    config = tmp_path / "configs" / "search.json"
    config.write_text(json.dumps({
        "embeddings_path": "data/coarse.zcve", "rescore_embeddings_path": "data/fine.zcve",
        "metadata_path": "data/absent.meta", "metric": "Cosine", "default_top_k": 10, "default_candidates": 100,
        "rescore_candidates": 64, "use_cuda_graphs": True, "device_id": 0}))
    queries = orc.normal_rows(batch, dim, 1213)
    qpath = tmp_path / "q.f32"
    queries.tofile(qpath)
    res = subprocess.run([str(driver), f"config={config}", f"queries={qpath}", f"batch={batch}",
                          f"out={tmp_path / 'r'}"], capture_output=True, text=True, timeout=300, cwd=tmp_path / "configs")
    assert res.returncode == 0, res.stdout + res.stderr
    assert "graph=1 rescore=1" in res.stdout
    ids = np.fromfile(tmp_path / "r.ids", dtype=np.int32).reshape(batch, 10)
    scores = np.fromfile(tmp_path / "r.scores", dtype=np.float32).reshape(batch, 10)
    # Resolved options: candidates 100, rescore width max(64, 100) = 100, top 10.
    q8, s8 = orc.quantize_rows_i8(corpus)
    cand, _ = orc.scan_topk(q8, orc.DTYPE_I8_ROW, dim, queries, 100, row_scales=s8, metric=orc.METRIC_COSINE)
    ref_i, ref_s = orc.rescore_topk(orc.to_f16_bits(corpus), orc.DTYPE_F16, dim, queries, cand, 10,
                                    metric=orc.METRIC_COSINE)
    np.testing.assert_array_equal(ids, ref_i)
    np.testing.assert_allclose(scores, ref_s, rtol=0, atol=1e-4)
