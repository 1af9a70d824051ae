"""GPU tier: zcgvs_merge_topk and the row-sharded search.

The merge must return the (score desc, id asc) top-k of the union of its lists; a corpus split
into P shards, each searched with its id_base and then merged, must equal the single-corpus
search bit for bit on integer-valued paths (per-row int8). With two or more GPUs the same
search runs as NCCL ranks (one process per GPU).
"""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

FLT_MAX = np.finfo(np.float32).max


def reference_merge(ids, scores, k):
    lists, batch, k_in = ids.shape
    out_i = np.full((batch, k), -1, dtype=np.int32)
    out_s = np.full((batch, k), -FLT_MAX, dtype=np.float32)
    for q in range(batch):
        entries = [(float(s), int(i)) for i, s in zip(ids[:, q].ravel(), scores[:, q].ravel()) if i >= 0]
        entries.sort(key=lambda e: (-e[0], e[1]))
        for j, (s, i) in enumerate(entries[:k]):
            out_i[q, j] = i
            out_s[q, j] = s
    return out_i, out_s


@pytest.mark.parametrize("lists,k_in,k", [(2, 10, 10), (8, 100, 100), (3, 7, 20), (8, 1024, 1024), (16, 1024, 64)])
def test_merge_random_lists(zc, lists, k_in, k):
    import torch

    rng = np.random.default_rng(lists * 1000 + k_in)
    batch = 5
    ids = rng.permutation(lists * batch * k_in * 4)[: lists * batch * k_in].reshape(lists, batch, k_in).astype(np.int32)
    scores = rng.integers(-50, 50, size=ids.shape).astype(np.float32) / 8  # many ties
    ids[:, 1, -3:] = -1                                                    # padding slots
    out_i, out_s = zc.merge_topk(torch.from_numpy(ids).cuda(), torch.from_numpy(scores).cuda(), k)
    torch.cuda.synchronize()
    ref_i, ref_s = reference_merge(ids, scores, k)
    np.testing.assert_array_equal(out_i.cpu().numpy(), ref_i)
    np.testing.assert_array_equal(out_s.cpu().numpy(), ref_s)


@pytest.mark.parametrize("shards", [2, 3, 8])
def test_sharded_search_on_one_gpu(zc, orc, shards):
    import torch

    import sharded

    n, dim, batch, k = 50000, 256, 4, 100
    corpus = orc.normal_rows(n, dim, 77)
    queries = orc.normal_rows(batch, dim, 78)
    storage, _, row_scales = orc.encode(corpus, 4)
    d_store = torch.from_numpy(storage).cuda()
    d_scales = torch.from_numpy(row_scales).cuda()
    d_q = torch.from_numpy(queries).cuda()
    all_i, all_s = [], []
    for r in range(shards):
        b, e = sharded.shard_bounds(n, shards, r)
        i, s = zc.scan_topk(d_store[b:e], 4, dim, d_q, k, row_scales=d_scales[b:e], id_base=b)
        all_i.append(i)
        all_s.append(s)
    out_i, out_s = zc.merge_topk(torch.stack(all_i), torch.stack(all_s), k)
    torch.cuda.synchronize()
    ref_i, ref_s = orc.scan_topk(storage, 4, dim, queries, k, row_scales=row_scales)
    np.testing.assert_array_equal(out_i.cpu().numpy(), ref_i)
    np.testing.assert_array_equal(out_s.cpu().numpy(), ref_s)


def test_merge_rejects_oversized_input(zc):
    import torch

    ids = torch.zeros((17, 1, 1024), dtype=torch.int32, device="cuda")
    with pytest.raises(zc.InvalidArgument):
        zc.merge_topk(ids, ids.float(), 10)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _nccl_worker(rank, world, port, result_path):
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    for p in (root, os.path.join(root, "zero-copy-gpu-vector-search-re-ranking-engine_b200"), os.path.join(root, "oracle")):
        sys.path.insert(0, p)
    from datetime import timedelta

    import torch
    import torch.distributed as dist

    import oracle
    import sharded

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        n, dim, k = 40000, 128, 50
        corpus = oracle.normal_rows(n, dim, 99)
        queries = oracle.normal_rows(3, dim, 98)
        storage, _, row_scales = oracle.encode(corpus, 4)
        b, e = sharded.shard_bounds(n, world, rank)
        local = sharded.scan_shard_search(torch.from_numpy(storage[b:e]).cuda(), 4, dim,
                                          row_scales=torch.from_numpy(row_scales[b:e]).cuda())
        ids, scores = sharded.ShardedSearch(b, e, local).search(torch.from_numpy(queries).cuda(), k)
        torch.cuda.synchronize()
        np.savez(f"{result_path}.{rank}.npz", ids=ids.cpu().numpy(), scores=scores.cpu().numpy())
    finally:
        dist.destroy_process_group()


def test_sharded_search_over_nccl(tmp_path, orc):
    import torch
    import torch.multiprocessing as mp

    world = min(torch.cuda.device_count(), 8)
    if world < 2:
        pytest.skip("needs two or more GPUs")
    path = str(tmp_path / "nccl")
    mp.start_processes(_nccl_worker, args=(world, _free_port(), path), nprocs=world, start_method="spawn")
    n, dim, k = 40000, 128, 50
    storage, _, row_scales = orc.encode(orc.normal_rows(n, dim, 99), 4)
    ref_i, ref_s = orc.scan_topk(storage, 4, dim, orc.normal_rows(3, dim, 98), k, row_scales=row_scales)
    for rank in range(world):
        got = np.load(f"{path}.{rank}.npz")
        np.testing.assert_array_equal(got["ids"], ref_i)
        np.testing.assert_array_equal(got["scores"], ref_s)


def _dev(a):
    import torch

    a = np.ascontiguousarray(a)
    if a.dtype == np.uint16:
        a = a.view(np.int16)
    elif a.dtype == np.uint32:
        a = a.view(np.int32)
    return torch.from_numpy(a).cuda()


def _nccl_rescore_worker(rank, world, port, result_path):
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    for p in (root, os.path.join(root, "zero-copy-gpu-vector-search-re-ranking-engine_b200"), os.path.join(root, "oracle")):
        sys.path.insert(0, p)
    from datetime import timedelta

    import torch
    import torch.distributed as dist

    import oracle
    import sharded
    import zcgvs_sm100 as zc

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        n, dim, batch, m, k = 30011, 256, 5, 500, 10
        corpus = oracle.normal_rows(n, dim, 501)
        queries = _dev(oracle.normal_rows(batch, dim, 502))
        b, e = sharded.shard_bounds(n, world, rank)
        codes = _dev(oracle.pack_binary(corpus[b:e]))
        store = _dev(oracle.to_f16_bits(corpus[b:e]))
        ws = zc.Workspace(torch.device("cuda", rank))

        def coarse(q, mm, id_base):
            return zc.scan_topk(codes, zc.DTYPE_BINARY, dim, q, mm, id_base=id_base, workspace=ws)

        def rescore(q, local, kk):
            return zc.rescore_topk(store, zc.DTYPE_F16, dim, q, local, kk, metric=zc.METRIC_COSINE)

        ids, scores = sharded.ShardedRescoreSearch(b, e, coarse, rescore).search(queries, m, k)
        torch.cuda.synchronize()
        np.savez(f"{result_path}.{rank}.npz", ids=ids.cpu().numpy(), scores=scores.cpu().numpy())
    finally:
        dist.destroy_process_group()


def test_sharded_coarse_rescore_over_nccl(tmp_path, orc):
    """The row-sharded 1-bit coarse search with fp16 rescoring (two exchanges) over NCCL ranks
    equals the one-corpus pipeline of the oracle on every rank."""
    import torch
    import torch.multiprocessing as mp

    world = min(torch.cuda.device_count(), 8)
    if world < 2:
        pytest.skip("needs two or more GPUs")
    path = str(tmp_path / "nccl_rescore")
    mp.start_processes(_nccl_rescore_worker, args=(world, _free_port(), path), nprocs=world, start_method="spawn")
    n, dim, batch, m, k = 30011, 256, 5, 500, 10
    corpus = orc.normal_rows(n, dim, 501)
    queries = orc.normal_rows(batch, dim, 502)
    c_ids, _ = orc.scan_topk(orc.pack_binary(corpus), orc.DTYPE_BINARY, dim, queries, m)
    ref_i, ref_s = orc.rescore_topk(orc.to_f16_bits(corpus), orc.DTYPE_F16, dim, queries, c_ids, k,
                                    metric=orc.METRIC_COSINE)
    for rank in range(world):
        got = np.load(f"{path}.{rank}.npz")
        np.testing.assert_array_equal(got["ids"], ref_i)
        np.testing.assert_allclose(got["scores"], ref_s, rtol=0, atol=1e-4)
