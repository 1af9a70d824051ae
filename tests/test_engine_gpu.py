"""GPU tier: zcgvs::VectorEngine (include/zcgvs/engine/vector_engine.hpp), the reference Engine's
request path over this library's Searcher, driven by tests/cpp/engine_search.cpp. The engine's
answers must equal the oracle's searches under the reference's rules: an allow list becomes a
mask, hybrid queries use the tokenizer ids minus [CLS] / [SEP], negatives and repeats, the
Searcher returns `candidates` hits of which the first top_k are kept, a rescore store rescoring
`rescore_candidates` coarse hits, graph replay counted in the stats."""

from __future__ import annotations

import os
import shutil
import subprocess

import numpy as np
import pytest

from conftest import PKG, ROOT

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def driver(zc, tmp_path_factory):
    exe = tmp_path_factory.mktemp("cpp") / "engine_search"
    cuda = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    cxx = shutil.which("g++") or shutil.which("c++")
    subprocess.run([cxx, "-std=c++17", "-O2", f"-I{ROOT / 'include'}", f"-I{cuda}/include",
                    str(ROOT / "tests/cpp/engine_search.cpp"), "-o", str(exe), f"-L{PKG}", "-lzcgvs_sm100",
                    f"-L{cuda}/lib64", "-lcudart", f"-Wl,-rpath,{PKG}"], check=True, capture_output=True, text=True)
    return exe


def run(driver, tmp_path, corpus, queries, top_k, **kw):
    n, dim = corpus.shape
    batch = queries.shape[0]
    np.ascontiguousarray(corpus, dtype=np.float32).tofile(tmp_path / "c.f32")
    np.ascontiguousarray(queries, dtype=np.float32).tofile(tmp_path / "q.f32")
    args = [str(driver), f"corpus={tmp_path / 'c.f32'}", f"n={n}", f"dim={dim}", f"queries={tmp_path / 'q.f32'}",
            f"batch={batch}", f"top_k={top_k}", f"out={tmp_path / 'r'}"] + [f"{k}={v}" for k, v in kw.items()]
    res = subprocess.run(args, capture_output=True, text=True, timeout=300)
    assert res.returncode == 0, res.stdout + res.stderr
    ids = np.fromfile(tmp_path / "r.ids", dtype=np.int32).reshape(batch, top_k)
    scores = np.fromfile(tmp_path / "r.scores", dtype=np.float32).reshape(batch, top_k)
    return ids, scores, res.stdout


def test_engine_dense_search_with_allow_list(driver, orc, tmp_path):
    n, dim = 5000, 256
    corpus = orc.normal_rows(n, dim, 61)
    queries = orc.normal_rows(3, dim, 62)
    allow = np.random.default_rng(63).choice(n, size=2000, replace=False).astype(np.int32)
    allow = np.concatenate([allow, np.array([-5, n + 3, allow[0]], dtype=np.int32)])  # ignored, repeated
    allow.tofile(tmp_path / "allow.i32")
    ids, scores, out = run(driver, tmp_path, corpus, queries, 7, dtype=4, candidates=20, allow=tmp_path / "allow.i32",
                           allow_n=allow.size)
    mask = np.zeros(n, dtype=np.uint8)
    mask[allow[(allow >= 0) & (allow < n)]] = 1
    q8, s8 = orc.quantize_rows_i8(corpus)
    ref_i, ref_s = orc.scan_topk(q8, orc.DTYPE_I8_ROW, dim, queries, 20, row_scales=s8, mask=mask,
                                 metric=orc.METRIC_COSINE)
    np.testing.assert_array_equal(ids, ref_i[:, :7])
    np.testing.assert_array_equal(scores, ref_s[:, :7])
    assert mask[ids].all()
    assert "dtype=int8_row" in out and "hits0=7" in out


def test_engine_hybrid_search_prepares_terms(driver, orc, tmp_path):
    import lexical_index as li

    n, dim, vocab, batch = 20000, 256, 2000, 2
    offsets, docs, weights = (t.numpy() for t in li.synthetic_corpus(n, vocab, 40.0, 1.1, 71, k1=0.9, b=0.4))
    terms = li.synthetic_queries(batch, vocab, 1.1, 72)
    corpus = orc.normal_rows(n, dim, 73)
    queries = orc.normal_rows(batch, dim, 74)
    offsets.astype(np.int64).tofile(tmp_path / "off.i64")
    docs.astype(np.int32).tofile(tmp_path / "docs.i32")
    weights.astype(np.float32).tofile(tmp_path / "w.f32")
    flat = []
    for q in range(batch):
        t = [int(x) for x in terms[q] if x >= 0]
        encoded = [101] + t + [t[0], -1] + [102]  # [CLS] terms, a repeat, a negative id, [SEP]
        flat += [len(encoded)] + encoded
    np.asarray(flat, dtype=np.int32).tofile(tmp_path / "terms.i32")
    ids, scores, out = run(driver, tmp_path, corpus, queries, 10, dtype=4, candidates=50, hybrid=1, weight=0.5,
                           offsets=tmp_path / "off.i64", docs=tmp_path / "docs.i32", weights=tmp_path / "w.f32",
                           vocab=vocab, terms=tmp_path / "terms.i32")
    q8, s8 = orc.quantize_rows_i8(corpus)
    ref_i, ref_s = orc.hybrid_topk(q8, orc.DTYPE_I8_ROW, dim, queries, 50, offsets, docs, weights, vocab, terms, 0.5,
                                   row_scales=s8, metric=orc.METRIC_COSINE)
    np.testing.assert_array_equal(ids, ref_i[:, :10])
    np.testing.assert_array_equal(scores, ref_s[:, :10])
    assert f"lexical={docs.size}" in out


def test_engine_rescore_with_graph_replay_and_stats(driver, orc, tmp_path):
    n, dim = 8192, 256
    corpus = orc.normal_rows(n, dim, 81)
    queries = orc.normal_rows(2, dim, 82)
    ids, scores, out = run(driver, tmp_path, corpus, queries, 5, dtype=4, rescore_dtype=1, candidates=20,
                           rescore=200, graph=1, repeat=3)
    q8, s8 = orc.quantize_rows_i8(corpus)
    cand, _ = orc.scan_topk(q8, orc.DTYPE_I8_ROW, dim, queries, 200, row_scales=s8, metric=orc.METRIC_COSINE)
    ref_i, ref_s = orc.rescore_topk(orc.to_f16_bits(corpus), orc.DTYPE_F16, dim, queries, cand, 20,
                                    metric=orc.METRIC_COSINE)
    np.testing.assert_array_equal(ids, ref_i[:, :5])
    np.testing.assert_allclose(scores, ref_s[:, :5], rtol=0, atol=1e-4)
    assert "rescore=float16" in out and "captures=1 launches=3 graph=1" in out and "major=10" in out


def test_engine_resolution_raises_candidates_to_top_k(driver, orc, tmp_path):
    n, dim = 3000, 128
    corpus = orc.normal_rows(n, dim, 91)
    queries = orc.normal_rows(1, dim, 92)
    ids, scores, out = run(driver, tmp_path, corpus, queries, 30, dtype=4, candidates=10)
    q8, s8 = orc.quantize_rows_i8(corpus)
    ref_i, ref_s = orc.scan_topk(q8, orc.DTYPE_I8_ROW, dim, queries, 30, row_scales=s8, metric=orc.METRIC_COSINE)
    np.testing.assert_array_equal(ids, ref_i)
    np.testing.assert_array_equal(scores, ref_s)
    assert "hits0=30" in out
