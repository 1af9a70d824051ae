"""GPU tier: the native row-sharded search (zcgvs_sharded_*, the C++ ShardedSearcher).

* zcgvs_merge_topk_lists reads an all-gather's packed [P, 2, B, k] output in place, adds each
  list's id offset and writes the owned shard-local candidates: checked against a Python merge.
* One rank (world 1, runs on any GPU box): the handle's dense search (streaming scan, tensor-core
  dispatch, fp16 on the tensor cores) and its coarse-plus-rescore search equal the one-GPU
  library calls bit for bit, directly and replayed from the captured CUDA graph.
* P ranks over NCCL (two or more GPUs), one process each: every rank's result equals the
  oracle's one-corpus search (bit-exact for per-row int8 and the 1-bit coarse stage, rescored
  scores within 1e-4), through the Python binding and through the C++ ShardedSearcher.
"""

from __future__ import annotations

import os
import shutil
import subprocess

import numpy as np
import pytest

from conftest import PKG, ROOT

pytestmark = pytest.mark.gpu

FLT_MAX = np.finfo(np.float32).max


def _dev(a):
    import torch

    a = np.ascontiguousarray(a)
    if a.dtype == np.uint16:
        a = a.view(np.int16)
    elif a.dtype == np.uint32:
        a = a.view(np.int32)
    return torch.from_numpy(a).cuda()


def _python_merge(ids, scores, offsets, k, own):
    lists, batch, _ = ids.shape
    out_i = np.full((batch, k), -1, dtype=np.int32)
    out_s = np.full((batch, k), -FLT_MAX, dtype=np.float32)
    owned = np.full((batch, k), -1, dtype=np.int32)
    for q in range(batch):
        entries = [(float(s), int(i) + int(offsets[p]))
                   for p in range(lists) for i, s in zip(ids[p, q], scores[p, q]) if i >= 0]
        entries.sort(key=lambda e: (-e[0], e[1]))
        for j, (s, i) in enumerate(entries[:k]):
            out_i[q, j], out_s[q, j] = i, s
            owned[q, j] = i - own[0] if own[0] <= i < own[1] else -1
    return out_i, out_s, owned


def test_merge_lists_reads_the_allgather_layout(zc):
    import torch

    rng = np.random.default_rng(5)
    lists, batch, k_in, k = 4, 6, 50, 40
    ids = rng.integers(0, 1000, size=(lists, batch, k_in)).astype(np.int32)
    scores = (rng.integers(-40, 40, size=ids.shape) / 4).astype(np.float32)  # many ties
    ids[:, 2, -5:] = -1
    packed = np.stack([ids, scores.view(np.int32)], axis=1)  # [P, 2, B, k_in]
    offsets = np.array([0, 1000, 2000, 3000], dtype=np.int32)
    d = torch.from_numpy(packed.copy()).cuda().reshape(-1)
    out = (torch.empty((batch, k), dtype=torch.int32, device="cuda"),
           torch.empty((batch, k), dtype=torch.float32, device="cuda"))
    owned = torch.empty((batch, k), dtype=torch.int32, device="cuda")
    zc.merge_topk_lists(d, d[batch * k_in:].view(torch.float32), 2 * batch * k_in, lists, batch, k_in, k,
                        list_id_offsets=torch.from_numpy(offsets).cuda(), out=out, own_range=(1000, 2000),
                        out_owned=owned)
    torch.cuda.synchronize()
    ref_i, ref_s, ref_o = _python_merge(ids, scores, offsets, k, (1000, 2000))
    np.testing.assert_array_equal(out[0].cpu().numpy(), ref_i)
    np.testing.assert_array_equal(out[1].cpu().numpy(), ref_s)
    np.testing.assert_array_equal(owned.cpu().numpy(), ref_o)


def _one_rank_searcher(zc, n):
    return zc.ShardedSearcher(zc.ShardedSearcher.unique_id(), 1, 0, n)


@pytest.mark.parametrize("name,batch", [("i8row", 3), ("i8row", 64), ("bin", 16), ("f16", 32)])
def test_one_rank_dense_search_equals_the_library_call(zc, orc, name, batch):
    import torch

    n, dim, k = 70_000, 256, 50
    corpus = orc.normal_rows(n, dim, 71)
    queries = _dev(orc.normal_rows(batch, dim, 72))
    dtype = {"i8row": zc.DTYPE_I8_ROW, "bin": zc.DTYPE_BINARY, "f16": zc.DTYPE_F16}[name]
    storage, _, rs = orc.encode(corpus, dtype)
    d_store, d_rs = _dev(storage), (None if rs is None else _dev(rs))
    s = _one_rank_searcher(zc, n)
    try:
        if name == "f16":
            ref = zc.gemm_topk(d_store, dtype, dim, queries, k)
        else:
            ref = zc.scan_topk(d_store, dtype, dim, queries, k, row_scales=d_rs)
        for graph in (False, True, True, True):  # direct; first graph search (runs + captures); replays
            got = s.search(d_store, dtype, dim, queries, k, row_scales=d_rs, tensor_f16=(name == "f16"), graph=graph)
            torch.cuda.synchronize()
            assert torch.equal(got[0], ref[0]) and torch.equal(got[1], ref[1]), f"graph={graph}"
        assert s.status() == (0, 0)
    finally:
        s.close()


def test_one_rank_rescore_search_equals_the_pipeline(zc, orc):
    import torch

    n, dim, batch, m, k = 70_000, 256, 16, 500, 10
    corpus = orc.normal_rows(n, dim, 81)
    queries = _dev(orc.normal_rows(batch, dim, 82))
    codes, store = _dev(orc.pack_binary(corpus)), _dev(orc.to_f16_bits(corpus))
    cand = zc.scan_topk(codes, zc.DTYPE_BINARY, dim, queries, m)
    ref = zc.rescore_topk(store, zc.DTYPE_F16, dim, queries, cand[0], k, metric=zc.METRIC_COSINE)
    s = _one_rank_searcher(zc, n)
    try:
        for graph in (False, True, True):
            got = s.rescore_search(codes, zc.DTYPE_BINARY, store, zc.DTYPE_F16, dim, queries, m, k,
                                   metric=zc.METRIC_COSINE, graph=graph)
            torch.cuda.synchronize()
            assert torch.equal(got[0], ref[0]) and torch.equal(got[1], ref[1]), f"graph={graph}"
        assert s.status() == (0, 0)
    finally:
        s.close()


def test_sharded_handle_rejects_bad_arguments(zc):
    import torch

    s = _one_rank_searcher(zc, 1000)
    try:
        shard = torch.zeros((999, 64), dtype=torch.int8, device="cuda")
        q = torch.zeros((1, 64), dtype=torch.float32, device="cuda")
        with pytest.raises(zc.InvalidArgument, match="differs from this rank's shard"):
            s.search(shard, zc.DTYPE_I8, 64, q, 10)
        shard = torch.zeros((1000, 64), dtype=torch.int8, device="cuda")
        with pytest.raises(zc.InvalidArgument, match="rows per shard"):
            s.search(shard, zc.DTYPE_I8, 64, q, 1001)
        with pytest.raises(zc.InvalidArgument, match="fp16 shard"):
            s.search(shard, zc.DTYPE_I8, 64, q, 10, tensor_f16=True)
    finally:
        s.close()


# ---------------------------------------------------------------------------------------------
# Several ranks over NCCL
# ---------------------------------------------------------------------------------------------
N, DIM, BATCH, K, M = 140_011, 256, 64, 50, 500


def _worker(rank, world, id_path, result_path):
    import sys
    import time

    for p in (str(ROOT), str(PKG), str(ROOT / "oracle")):
        sys.path.insert(0, p)
    import torch

    import oracle
    import zcgvs_sm100 as zc

    torch.cuda.set_device(rank)
    if rank == 0:
        with open(id_path + ".tmp", "wb") as f:
            f.write(zc.ShardedSearcher.unique_id())
        os.replace(id_path + ".tmp", id_path)
    for _ in range(600):
        if os.path.exists(id_path):
            break
        time.sleep(0.1)
    with open(id_path, "rb") as f:
        nccl_id = f.read()
    s = zc.ShardedSearcher(nccl_id, world, rank, N)
    try:
        corpus = oracle.normal_rows(N, DIM, 91)[s.begin:s.end]
        queries = _dev(oracle.normal_rows(BATCH, DIM, 92))
        codes, rs = oracle.quantize_rows_i8(corpus)
        out = {}
        for graph in (False, True, True):
            i, v = s.search(_dev(codes), zc.DTYPE_I8_ROW, DIM, queries, K, row_scales=_dev(rs), graph=graph)
        out["i8_ids"], out["i8_scores"] = i.cpu().numpy(), v.cpu().numpy()
        f16 = _dev(oracle.to_f16_bits(corpus))
        for graph in (False, True, True):
            i, v = s.search(f16, zc.DTYPE_F16, DIM, queries, K, metric=zc.METRIC_COSINE, tensor_f16=True, graph=graph)
        out["f16_ids"], out["f16_scores"] = i.cpu().numpy(), v.cpu().numpy()
        bits = _dev(oracle.pack_binary(corpus))
        for graph in (False, True, True):
            i, v = s.rescore_search(bits, zc.DTYPE_BINARY, f16, zc.DTYPE_F16, DIM, queries, M, 10,
                                    metric=zc.METRIC_COSINE, graph=graph)
        out["rs_ids"], out["rs_scores"] = i.cpu().numpy(), v.cpu().numpy()
        out["status"] = np.array(s.status())
        np.savez(f"{result_path}.{rank}.npz", **out)
    finally:
        s.close()


def test_native_sharded_search_over_nccl(tmp_path, orc):
    import torch
    import torch.multiprocessing as mp

    world = min(torch.cuda.device_count(), 8)
    if world < 2:
        pytest.skip("needs two or more GPUs")
    path = str(tmp_path / "native")
    mp.start_processes(_worker, args=(world, str(tmp_path / "nccl.id"), path), nprocs=world, start_method="spawn")
    corpus = orc.normal_rows(N, DIM, 91)
    queries = orc.normal_rows(BATCH, DIM, 92)
    q8, s8 = orc.quantize_rows_i8(corpus)
    ref_i, ref_s = orc.scan_topk(q8, orc.DTYPE_I8_ROW, DIM, queries, K, row_scales=s8)
    f16 = orc.to_f16_bits(corpus)
    # fp16 on the tensor cores rounds the queries to fp16: the oracle scores the same queries.
    q16 = orc.to_f16_bits(queries).view(np.float16).astype(np.float32)
    f16_scores = orc.scores(f16, orc.DTYPE_F16, DIM, q16, metric=orc.METRIC_COSINE)
    c_ids, _ = orc.scan_topk(orc.pack_binary(corpus), orc.DTYPE_BINARY, DIM, queries, M)
    rs_i, rs_s = orc.rescore_topk(f16, orc.DTYPE_F16, DIM, queries, c_ids, 10, metric=orc.METRIC_COSINE)
    from conftest import assert_topk_parity

    for rank in range(world):
        got = np.load(f"{path}.{rank}.npz")
        assert tuple(got["status"]) == (0, 0)
        np.testing.assert_array_equal(got["i8_ids"], ref_i)
        np.testing.assert_array_equal(got["i8_scores"], ref_s)
        assert_topk_parity(got["f16_ids"], got["f16_scores"], f16_scores, K, exact=False)
        np.testing.assert_array_equal(got["rs_ids"], rs_i)
        np.testing.assert_allclose(got["rs_scores"], rs_s, rtol=0, atol=1e-4)


@pytest.fixture(scope="module")
def cpp_driver(zc, tmp_path_factory):
    exe = tmp_path_factory.mktemp("cpp") / "sharded_search"
    cuda = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    cxx = shutil.which("g++") or shutil.which("c++")
    cmd = [cxx, "-std=c++17", "-O2", f"-I{ROOT / 'include'}", f"-I{cuda}/include",
           str(ROOT / "tests/cpp/sharded_search.cpp"), "-o", str(exe), f"-L{PKG}", "-lzcgvs_sm100",
           f"-L{cuda}/lib64", "-lcudart", f"-Wl,-rpath,{PKG}"]
    subprocess.run(cmd, check=True, capture_output=True, text=True)
    return exe


def _run_cpp_ranks(exe, tmp_path, world, corpus, queries, k, extra):
    host, qpath = tmp_path / "c.f32", tmp_path / "q.f32"
    corpus.tofile(host)
    queries.tofile(qpath)
    n, dim = corpus.shape
    procs = [subprocess.Popen([str(exe), f"id={tmp_path / 'id'}", f"world={world}", f"rank={r}", f"host={host}",
                               f"n={n}", f"dim={dim}", f"queries={qpath}", f"batch={queries.shape[0]}", f"k={k}",
                               f"out={tmp_path / f'r{r}'}"] + extra,
                              stdout=subprocess.PIPE, stderr=subprocess.PIPE, text=True) for r in range(world)]
    outs = [p.communicate(timeout=600) for p in procs]
    for p, (o, e) in zip(procs, outs):
        assert p.returncode == 0, o + e
    return [(np.fromfile(tmp_path / f"r{r}.ids", dtype=np.int32).reshape(queries.shape[0], k),
             np.fromfile(tmp_path / f"r{r}.scores", dtype=np.float32).reshape(queries.shape[0], k))
            for r in range(world)]


def test_cpp_sharded_searcher(cpp_driver, orc, tmp_path):
    """The C++ ShardedSearcher on every GPU of the box (one rank when there is one GPU): a per-row
    int8 dense search replayed from its graph, and a 1-bit coarse search rescored against fp16
    rows; every rank's result equals the oracle's one-corpus pipeline."""
    import torch

    world = min(torch.cuda.device_count(), 8)
    n, dim, batch = 90_001, 256, 8
    corpus = orc.normal_rows(n, dim, 61)
    queries = orc.normal_rows(batch, dim, 62)
    q8, s8 = orc.quantize_rows_i8(corpus)
    ref_i, ref_s = orc.scan_topk(q8, orc.DTYPE_I8_ROW, dim, queries, 20, row_scales=s8)
    for ids, scores in _run_cpp_ranks(cpp_driver, tmp_path, world, corpus, queries, 20,
                                      ["dtype=4", "graph=1", "passes=3"]):
        np.testing.assert_array_equal(ids, ref_i)
        np.testing.assert_array_equal(scores, ref_s)
    c_ids, _ = orc.scan_topk(orc.pack_binary(corpus), orc.DTYPE_BINARY, dim, queries, 300)
    rs_i, rs_s = orc.rescore_topk(orc.to_f16_bits(corpus), orc.DTYPE_F16, dim, queries, c_ids, 10,
                                  metric=orc.METRIC_COSINE)
    (tmp_path / "id").unlink()
    for ids, scores in _run_cpp_ranks(cpp_driver, tmp_path, world, corpus, queries, 10,
                                      ["dtype=3", "rescore_dtype=1", "m=300", "metric=0", "graph=1", "passes=2"]):
        np.testing.assert_array_equal(ids, rs_i)
        np.testing.assert_allclose(scores, rs_s, rtol=0, atol=1e-4)
