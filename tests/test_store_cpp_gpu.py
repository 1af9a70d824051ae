"""GPU tier: the C++ drop-in layer's stores and Searcher on files. A small driver
(tests/cpp/store_search.cpp, compiled here against include/zcgvs/ and libzcgvs_sm100.so) loads
ZCVE / ZCVL files with EmbeddingStore::loadFromFile / LexicalIndex::loadFromFile (the payload
streamed through pinned chunks into device memory), or builds a store on the device with
fromHostMatrix + append, and runs Searcher::search. Results must equal the oracle's search over
the same encoded rows bit for bit: reference-written version-2 files of every reference dtype,
version-3 per-row int8 files (the extension that carries row scales), a multi-chunk file, a per-row
store grown by append, and a per-row coarse search rescored against an fp16 file with graph
replay."""

from __future__ import annotations

import os
import shutil
import subprocess

import numpy as np
import pytest

from conftest import PKG, ROOT

import formats  # noqa: E402

pytestmark = pytest.mark.gpu

GOLDEN = np.load(ROOT / "tests" / "golden" / "files.npz")


@pytest.fixture(scope="module")
def driver(zc, tmp_path_factory):
    exe = tmp_path_factory.mktemp("cpp") / "store_search"
    cuda = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    cxx = shutil.which("g++") or shutil.which("c++")
    cmd = [cxx, "-std=c++17", "-O2", f"-I{ROOT / 'include'}", f"-I{cuda}/include", str(ROOT / "tests/cpp/store_search.cpp"),
           "-o", str(exe), f"-L{PKG}", "-lzcgvs_sm100", f"-L{cuda}/lib64", "-lcudart", f"-Wl,-rpath,{PKG}"]
    subprocess.run(cmd, check=True, capture_output=True, text=True)
    return exe


def run(driver, tmp_path, queries, k, metric=1, expect_ok=True, **kw):
    batch, dim = queries.shape
    qpath = tmp_path / "q.f32"
    np.ascontiguousarray(queries, dtype=np.float32).tofile(qpath)
    args = [str(driver), f"queries={qpath}", f"batch={batch}", f"dim={dim}", f"k={k}", f"metric={metric}",
            f"out={tmp_path / 'r'}"] + [f"{key}={val}" for key, val in kw.items()]
    res = subprocess.run(args, capture_output=True, text=True, timeout=300)
    if not expect_ok:
        assert res.returncode != 0
        return res.stderr
    assert res.returncode == 0, res.stdout + res.stderr
    ids = np.fromfile(tmp_path / "r.ids", dtype=np.int32).reshape(batch, k)
    scores = np.fromfile(tmp_path / "r.scores", dtype=np.float32).reshape(batch, k)
    return ids, scores, res.stdout


@pytest.mark.parametrize("dtype", ["float32", "float16", "int8", "binary"])
def test_reference_written_files_search_like_the_oracle(driver, orc, tmp_path, dtype):
    path = tmp_path / "c.zcve"
    path.write_bytes(GOLDEN[f"zcve_{dtype}"].tobytes())
    h, storage, _ = formats.read_encoded_embeddings(path)
    queries = orc.normal_rows(2, 70, 71)
    ids, scores, _ = run(driver, tmp_path, queries, 5, corpus=path)
    stored = storage.view(np.uint16) if dtype == "float16" else storage
    ref_i, ref_s = orc.scan_topk(stored, formats.DTYPE_NAMES[dtype], 70, queries, 5, scale=h["scale"])
    np.testing.assert_array_equal(ids, ref_i)
    if dtype == "binary":
        np.testing.assert_array_equal(scores, ref_s)
    else:
        np.testing.assert_allclose(scores, ref_s, rtol=0, atol=1e-5)


@pytest.mark.parametrize("n,dim,batch", [(3000, 384, 3), (200_000, 256, 2), (70_000, 768, 64)])
def test_version3_per_row_file_searches_like_the_oracle(driver, orc, tmp_path, n, dim, batch):
    """Per-row int8 from a version-3 file; 200K x 256 streams in two pinned chunks; batch 64 over
    70K rows takes the tensor-core path. Integer dots: bit-exact."""
    corpus = orc.normal_rows(n, dim, 300 + dim)
    path = tmp_path / "c.zcve"
    formats.write_embeddings(path, corpus, normalized=True, dtype="int8_row")
    queries = orc.normal_rows(batch, dim, 301 + dim)
    ids, scores, out = run(driver, tmp_path, queries, 10, corpus=path)
    assert "dtype=4 row_scales=1" in out
    q, s = orc.quantize_rows_i8(corpus)
    ref_i, ref_s = orc.scan_topk(q, orc.DTYPE_I8_ROW, dim, queries, 10, row_scales=s)
    np.testing.assert_array_equal(ids, ref_i)
    np.testing.assert_array_equal(scores, ref_s)


def test_per_row_store_built_on_device_and_grown_by_append(driver, orc, tmp_path):
    """fromHostMatrix(Int8PerRow) + append: the device converter writes codes and row scales, the
    growth copies both; the search equals the oracle over the whole quantised matrix."""
    n, dim = 5000, 200
    corpus = orc.normal_rows(n, dim, 77)
    host = tmp_path / "h.f32"
    corpus.tofile(host)
    queries = orc.normal_rows(4, dim, 78)
    ids, scores, out = run(driver, tmp_path, queries, 20, host=host, n=n, dtype=4, append=1700)
    assert f"docs={n} dtype=4 row_scales=1" in out
    q, s = orc.quantize_rows_i8(corpus)
    ref_i, ref_s = orc.scan_topk(q, orc.DTYPE_I8_ROW, dim, queries, 20, row_scales=s)
    np.testing.assert_array_equal(ids, ref_i)
    np.testing.assert_array_equal(scores, ref_s)


def test_per_row_coarse_with_fp16_rescore_file_and_graph_replay(driver, orc, tmp_path):
    n, dim, m, k = 8192, 256, 256, 10
    corpus = orc.normal_rows(n, dim, 31)
    coarse, fine = tmp_path / "coarse.zcve", tmp_path / "fine.zcve"
    formats.write_embeddings(coarse, corpus, normalized=True, dtype="int8_row")
    formats.write_embeddings(fine, corpus, normalized=True, dtype="float16")
    queries = orc.normal_rows(3, dim, 32)
    ids, scores, out = run(driver, tmp_path, queries, k, metric=0, corpus=coarse, rescore=fine, m=m, graph=1)
    assert "graph_launches=3" in out
    q, s = orc.quantize_rows_i8(corpus)
    cand, _ = orc.scan_topk(q, orc.DTYPE_I8_ROW, dim, queries, m, row_scales=s, metric=orc.METRIC_COSINE)
    ref_i, ref_s = orc.rescore_topk(orc.to_f16_bits(corpus), orc.DTYPE_F16, dim, queries, cand, k,
                                    metric=orc.METRIC_COSINE)
    np.testing.assert_array_equal(ids, ref_i)
    np.testing.assert_allclose(scores, ref_s, rtol=0, atol=1e-4)


def test_loader_rejects_per_row_dtype_in_version2_and_short_files(driver, orc, tmp_path):
    corpus = orc.normal_rows(64, 32, 5)
    path = tmp_path / "c.zcve"
    formats.write_embeddings(path, corpus, normalized=True, dtype="int8_row")
    raw = bytearray(path.read_bytes())
    raw[4:8] = (2).to_bytes(4, "little")
    bad = tmp_path / "v2.zcve"
    bad.write_bytes(bytes(raw))
    err = run(driver, tmp_path, orc.normal_rows(1, 32, 6), 5, corpus=bad, expect_ok=False)
    assert "version 3" in err
    short = tmp_path / "short.zcve"
    short.write_bytes(path.read_bytes()[:-3])
    err = run(driver, tmp_path, orc.normal_rows(1, 32, 6), 5, corpus=short, expect_ok=False)
    assert "ends early" in err


def test_searcher_throws_when_candidates_overflow_and_recovers(driver, orc, tmp_path):
    """A query of the tensor-core path whose candidates overflow its buffer after every retry gets
    an incomplete top-k; the Searcher reads the device status word with the result and throws
    std::runtime_error instead of returning it. The test hook caps the buffer at 5 entries for
    k = 10 (a host-side setting: no device fault is involved). The driver then restores the
    default cap and searches again with the same Searcher: the word was cleared, the result is
    the oracle's."""
    n, dim, batch, k = 70_000, 256, 64, 10
    corpus = orc.normal_rows(n, dim, 4242)
    path = tmp_path / "c.zcve"
    formats.write_embeddings(path, corpus, normalized=True, dtype="int8_row")
    queries = orc.normal_rows(batch, dim, 4243)
    qpath = tmp_path / "q.f32"
    queries.tofile(qpath)
    res = subprocess.run([str(driver), f"queries={qpath}", f"batch={batch}", f"dim={dim}", f"k={k}", "metric=1",
                          f"out={tmp_path / 'r'}", f"corpus={path}", "cap=5"], capture_output=True, text=True,
                         timeout=300)
    assert res.returncode == 1, res.stdout + res.stderr
    assert "search incomplete" in res.stderr and "more candidates than its buffer holds" in res.stderr, res.stderr
    assert "recovered" in res.stdout
    ids = np.fromfile(tmp_path / "r.ids", dtype=np.int32).reshape(batch, k)
    scores = np.fromfile(tmp_path / "r.scores", dtype=np.float32).reshape(batch, k)
    q, s = orc.quantize_rows_i8(corpus)
    ref_i, ref_s = orc.scan_topk(q, orc.DTYPE_I8_ROW, dim, queries, k, row_scales=s)
    np.testing.assert_array_equal(ids, ref_i)
    np.testing.assert_array_equal(scores, ref_s)
