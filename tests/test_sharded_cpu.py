"""CPU tier: the row-sharded search's host logic on world_size-2 (and 3) gloo process groups.

Each rank searches its shard through the oracle (CPU stand-ins for zcgvs_scan_topk and
zcgvs_merge_topk, injected into ShardedSearch), exchanges through torch.distributed, and must
return the single-corpus oracle result on every rank. The CUDA merge itself is covered by the
GPU tier.
"""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def oracle_merge(ids, scores, k):
    import torch

    import oracle

    lists, batch, k_in = ids.shape
    out_i = np.empty((batch, k), dtype=np.int32)
    out_s = np.empty((batch, k), dtype=np.float32)
    for q in range(batch):
        cand_ids = ids[:, q, :].reshape(-1).numpy()
        cand_sc = scores[:, q, :].reshape(-1).numpy()
        keep = cand_ids >= 0
        # Score row over the candidate ids only: everything else is absent.
        n = int(cand_ids[keep].max()) + 1 if keep.any() else 1
        row = np.full(n, -np.inf, dtype=np.float32)
        row[cand_ids[keep]] = cand_sc[keep]
        i, s = oracle.topk(row, min(k, n))
        i, s = i[0], s[0]
        live = np.isfinite(s)
        out_i[q] = -1
        out_s[q] = np.finfo(np.float32).min
        out_i[q, : live.sum()] = i[live]
        out_s[q, : live.sum()] = s[live]
    return torch.from_numpy(out_i), torch.from_numpy(out_s)


def worker(rank, world, port, n, dim, batch, k, dtype, result_path):
    import torch
    import torch.distributed as dist

    import oracle
    import sharded

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        corpus = oracle.normal_rows(n, dim, 1234)
        queries = oracle.normal_rows(batch, dim, 4321)
        storage, scale, row_scales = oracle.encode(corpus, dtype)
        begin, end = sharded.shard_bounds(n, world, rank)

        def local(qs, kk, id_base):
            rs = None if row_scales is None else row_scales[begin:end]
            i, s = oracle.scan_topk(storage[begin:end], dtype, dim, qs, kk, scale=scale, row_scales=rs,
                                    id_base=id_base)
            return torch.from_numpy(i), torch.from_numpy(s)

        search = sharded.ShardedSearch(begin, end, local, merge=oracle_merge)
        ids, scores = search.search(queries, k)
        np.savez(f"{result_path}.{rank}.npz", ids=ids.numpy(), scores=scores.numpy())
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,dtype", [(2, 4), (3, 4), (2, 0), (3, 0), (4, 3)])
def test_sharded_search_equals_single_corpus(tmp_path, world, dtype):
    import torch.multiprocessing as mp

    import oracle

    n, dim, batch, k = 3001, 64, 3, 25
    path = str(tmp_path / "res")
    mp.start_processes(worker, args=(world, free_port(), n, dim, batch, k, dtype, path), nprocs=world,
                       start_method="spawn")
    corpus = oracle.normal_rows(n, dim, 1234)
    queries = oracle.normal_rows(batch, dim, 4321)
    storage, scale, row_scales = oracle.encode(corpus, dtype)
    ref_i, ref_s = oracle.scan_topk(storage, dtype, dim, queries, k, scale=scale, row_scales=row_scales)
    for rank in range(world):
        got = np.load(f"{path}.{rank}.npz")
        np.testing.assert_array_equal(got["ids"], ref_i)
        np.testing.assert_array_equal(got["scores"], ref_s)


def test_shard_bounds_cover_rows_once():
    import sharded

    for n in (0, 1, 7, 1000, 1001):
        for world in (1, 2, 3, 8):
            spans = [sharded.shard_bounds(n, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            assert max(e - b for b, e in spans) - min(e - b for b, e in spans) <= 1


def rescore_worker(rank, world, port, n, dim, batch, m, k, result_path):
    import torch
    import torch.distributed as dist

    import oracle
    import sharded

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        corpus = oracle.normal_rows(n, dim, 777)
        queries = oracle.normal_rows(batch, dim, 778)
        codes = oracle.pack_binary(corpus)
        store = oracle.to_f16_bits(corpus)
        begin, end = sharded.shard_bounds(n, world, rank)

        def coarse(qs, mm, id_base):
            i, s = oracle.scan_topk(codes[begin:end], oracle.DTYPE_BINARY, dim, qs, mm, id_base=id_base)
            return torch.from_numpy(i), torch.from_numpy(s)

        def rescore(qs, local, kk):
            i, s = oracle.rescore_topk(store[begin:end], oracle.DTYPE_F16, dim, qs, local.numpy(), kk)
            return torch.from_numpy(i), torch.from_numpy(s)

        search = sharded.ShardedRescoreSearch(begin, end, coarse, rescore, merge=oracle_merge)
        ids, scores = search.search(queries, m, k)
        np.savez(f"{result_path}.{rank}.npz", ids=ids.numpy(), scores=scores.numpy())
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_sharded_coarse_rescore_equals_single_corpus(tmp_path, world):
    """BASELINE config 3 split over ranks: per-shard 1-bit top-m, exchange and merge, each rank
    rescores the global candidates it owns against its fp16 rows, exchange and merge. Every rank
    must hold the one-corpus pipeline's result bit for bit."""
    import torch.multiprocessing as mp

    import oracle

    n, dim, batch, m, k = 4001, 128, 3, 64, 10
    path = str(tmp_path / "rescore")
    mp.start_processes(rescore_worker, args=(world, free_port(), n, dim, batch, m, k, path), nprocs=world,
                       start_method="spawn")
    corpus = oracle.normal_rows(n, dim, 777)
    queries = oracle.normal_rows(batch, dim, 778)
    cand, _ = oracle.scan_topk(oracle.pack_binary(corpus), oracle.DTYPE_BINARY, dim, queries, m)
    ref_i, ref_s = oracle.rescore_topk(oracle.to_f16_bits(corpus), oracle.DTYPE_F16, dim, queries, cand, k)
    for rank in range(world):
        got = np.load(f"{path}.{rank}.npz")
        np.testing.assert_array_equal(got["ids"], ref_i)
        np.testing.assert_array_equal(got["scores"], ref_s)


def test_sharded_rescore_rejects_candidates_beyond_a_shard():
    """m above a shard's rows (or k above m) is rejected before any exchange, as the reference
    rejects k above the corpus (src/cuda/topk.cu:146-153)."""
    import sharded

    search = sharded.ShardedRescoreSearch(0, 100, lambda *a: None, lambda *a: None, merge=lambda *a: None)
    for m, k in [(101, 10), (50, 51), (50, 0)]:
        with pytest.raises(ValueError):
            search.search(None, m, k)


def test_sharded_search_rejects_k_beyond_a_shard():
    """A k that a one-GPU search over the whole corpus would accept but one shard cannot hold is
    rejected before any exchange, with the shard's row count in the message."""
    import sharded

    search = sharded.ShardedSearch(100, 150, lambda *a: None, merge=lambda *a: None)
    for k in (51, 0):
        with pytest.raises(ValueError, match="rows per shard"):
            search.search(None, k)
