"""GPU tier: parity at the benchmarked shapes.

Every workload bench.py times is run here exactly as the bench builds it (the same seeded device
generators, corpus sizes, batches and library calls, through bench.py's own workload classes),
and a subset of its queries is checked against the CPU oracle:

* config 1: fp32 5,183 x 384, cosine, top-10, all 300 queries;
* config 2 at batch 1,024: per-row int8 1M x 768, top-100, through the tensor-core dispatch of
  zcgvs_scan_topk; 32 of the 1,024 queries, bit-exact;
* config 3: 1-bit codes of 10M x 1024 fp16 rows, Hamming top-1,000 then fp16 rescore to top-10,
  batch 64; 4 queries, the coarse stage bit-exact and the rescored top-10 within the float
  tolerance over the gathered candidate rows;
* config 4: fp16 768-d rows, batch 4,096, top-100 on the tensor cores, over a 5M-row slice of
  the 50M-row corpus (one GPU's share is 6.25M at 8 GPUs); 8 queries within the float tolerance;
* config 5: hybrid BM25 + fp16 dense over the 2M-document Zipf(1.1) / Poisson(200) index;
  16 queries, lexical scores bit-exact (dense weight 0) and the blended top-10 within the float
  tolerance (dense weight 0.5).

Integer-valued results must equal the oracle bit for bit; float results must agree within
1e-4 relative to max(1, |score|), with id sets equal modulo near-ties at the k-th score (the
reference's own tolerance, tests/cpp/test_scan_paths.cu:128, and its id-exactness standard,
tests/cpp/test_pipeline.cu:95-106). Every search must leave the workspace's device status word
at 0 (no bounded wait ran out, no candidate buffer overflowed).
"""

from __future__ import annotations

import os

import numpy as np
import pytest

from conftest import assert_topk_parity

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def bench():
    import bench as b

    return b


@pytest.fixture(autouse=True)
def oracle_threads(orc):
    orc.set_threads(os.cpu_count() or 1)
    yield
    orc.set_threads(1)
    import torch

    torch.cuda.synchronize()
    torch.cuda.empty_cache()


def _setup(bench, zc, wl):
    import torch

    wl.setup(torch, zc, torch.device("cuda", torch.cuda.current_device()), 0, 1)
    torch.cuda.synchronize()
    return wl


def test_cfg1_fp32_all_300_queries(bench, zc, orc):
    import torch

    wl = _setup(bench, zc, bench.Cfg1())
    stream = torch.cuda.current_stream()
    ids, vals = [], []
    for i in range(wl.NQ):
        wl.step_direct(i, stream)
        ids.append(wl.out[0].clone())
        vals.append(wl.out[1].clone())
    assert wl.ws.status() == 0
    ids = torch.cat(ids).cpu().numpy()
    vals = torch.cat(vals).cpu().numpy()
    corpus = wl.corpus.cpu().numpy()
    ref = orc.scores(corpus, orc.DTYPE_F32, wl.D, wl.queries.cpu().numpy(), metric=orc.METRIC_COSINE)
    assert_topk_parity(ids, vals, ref, wl.K, exact=False)


def test_cfg2_int8_row_batch_1024_through_the_tensor_core_dispatch(bench, zc, orc):
    import torch

    wl = _setup(bench, zc, bench.Cfg2(1024))
    zc.kernel_timing(True)
    try:
        wl.step_direct(0, torch.cuda.current_stream())
        torch.cuda.synchronize()
        assert zc.kernel_timing_read("gemm_filter")[1] >= 1, "batch 1,024 did not take the tensor-core path"
    finally:
        zc.kernel_timing(False)
    assert wl.ws.status() == 0
    sel = np.arange(0, 1024, 32)
    got_i = wl.out[0].cpu().numpy()[sel]
    got_v = wl.out[1].cpu().numpy()[sel]
    queries = wl.queries[:1024].cpu().numpy()[sel]
    ref_i, ref_v = orc.scan_topk(wl.codes.cpu().numpy(), orc.DTYPE_I8_ROW, wl.D, queries, wl.K,
                                 row_scales=wl.scales.cpu().numpy())
    np.testing.assert_array_equal(got_i, ref_i)
    np.testing.assert_array_equal(got_v, ref_v)


def test_cfg3_binary_coarse_and_fp16_rescore_at_10M(bench, zc, orc):
    import torch

    wl = _setup(bench, zc, bench.Cfg3())
    q = wl.queries[:wl.B]
    wl._run(q, torch.cuda.current_stream())
    torch.cuda.synchronize()
    assert wl.ws.status() == 0
    sel = np.array([0, 21, 42, 63])
    cand = wl.cand[0].cpu().numpy()[sel]
    cand_v = wl.cand[1].cpu().numpy()[sel]
    qh = q.cpu().numpy()[sel]
    codes = wl.codes.cpu().numpy().view(np.uint32)
    ref_i, ref_v = orc.scan_topk(codes, orc.DTYPE_BINARY, wl.D, qh, wl.M)
    np.testing.assert_array_equal(cand, ref_i)
    np.testing.assert_array_equal(cand_v, ref_v)
    out_i = wl.out[0].cpu().numpy()[sel]
    out_v = wl.out[1].cpu().numpy()[sel]
    for r in range(len(sel)):
        # The candidates' fp16 rows, in id order (so positions order ties as ids do).
        order = np.sort(cand[r])
        rows = wl.store_i16[torch.from_numpy(order.astype(np.int64)).cuda()].cpu().numpy().view(np.uint16)
        ref = orc.scores(rows, orc.DTYPE_F16, wl.D, qh[r:r + 1], metric=orc.METRIC_COSINE)
        local = np.searchsorted(order, out_i[r])
        assert (order[local] == out_i[r]).all(), "a rescored id is not one of the coarse candidates"
        assert_topk_parity(local[None, :], out_v[r:r + 1], ref, wl.K, exact=False)


def test_cfg4_fp16_batch_4096_on_a_5M_row_slice(bench, zc, orc):
    import torch

    wl = bench.Cfg4()
    wl.N = 5_000_000
    _setup(bench, zc, wl)
    ids, vals = wl._run(wl.queries)
    torch.cuda.synchronize()
    assert wl.ws.status() == 0
    sel = np.arange(0, 4096, 512)
    got_i = ids.cpu().numpy()[sel]
    got_v = vals.cpu().numpy()[sel]
    store = wl.shard_i16.cpu().numpy().view(np.uint16)
    ref = orc.scores(store, orc.DTYPE_F16, wl.D, wl.queries.cpu().numpy()[sel], metric=orc.METRIC_COSINE)
    del store
    assert_topk_parity(got_i, got_v, ref, wl.K, exact=False)


def test_cfg5_hybrid_on_the_2M_document_zipf_index(bench, zc, orc):
    import torch

    wl = _setup(bench, zc, bench.Cfg5())
    sel = np.arange(16) * 61
    dense = wl.dense_i16.cpu().numpy().view(np.uint16)
    docs = wl.index.docs.cpu().numpy()
    weights = wl.index.weights.cpu().numpy()
    queries = wl.queries.cpu().numpy()[sel]
    terms = wl.terms_h[sel]
    for weight in (0.0, 0.5):
        got_i, got_v = [], []
        for j in sel:
            i, v = zc.hybrid_topk(wl.dense_i16, zc.DTYPE_F16, wl.D, wl.queries[j:j + 1], wl.K, wl.index,
                                  wl.terms[j:j + 1], weight, metric=zc.METRIC_COSINE, workspace=wl.ws)
            got_i.append(i.clone())
            got_v.append(v.clone())
        torch.cuda.synchronize()
        assert wl.ws.status() == 0
        got_i = torch.cat(got_i).cpu().numpy()
        got_v = torch.cat(got_v).cpu().numpy()
        if weight == 0.0:
            # lexical / max(lexical) alone: a deterministic sum on both sides, bit-exact.
            ref_i, ref_v = orc.hybrid_topk(dense, orc.DTYPE_F16, wl.D, queries, wl.K, wl.offsets_h, docs, weights,
                                           wl.V, terms, weight, metric=orc.METRIC_COSINE)
            np.testing.assert_array_equal(got_i, ref_i)
            np.testing.assert_array_equal(got_v, ref_v)
        else:
            # Full blended score rows (the oracle's hybrid chain: dense, BM25, max, fuse).
            rows = orc.scores(dense, orc.DTYPE_F16, wl.D, queries, metric=orc.METRIC_COSINE)
            for r in range(len(sel)):
                lex = orc.bm25(wl.offsets_h, docs, weights, wl.V, terms[r], wl.N)
                rows[r] = orc.fuse(rows[r], lex, orc.max_positive(lex), weight)
            assert_topk_parity(got_i, got_v, rows, wl.K, exact=False)
