"""GPU tier: BM25 lexical scoring and the hybrid search against the CPU oracle.

The reference accumulates BM25 with float atomics and checks its GPU with a tolerance
(tests/cpp/test_lexical.cu:118-126). This build sums in (term slot, posting) order, so its
lexical scores, maxima and fused scores must equal the oracle's sequential loop bit for bit; the
hybrid top-k is bit-exact wherever the dense part is (per-row int8, or dense_weight 0) and within
1e-4 otherwise. The first cases run the reference test's own index and query
(test_lexical.cu:31-67, regenerated from its seeds).
"""

from __future__ import annotations

import numpy as np
import pytest

from conftest import assert_topk_parity

pytestmark = pytest.mark.gpu

FLT_MAX = np.finfo(np.float32).max


def dev(a, dtype=None):
    import torch

    return torch.as_tensor(np.ascontiguousarray(a), dtype=dtype).cuda()


@pytest.fixture(scope="module")
def ref_case(orc):
    import lexical_index as li

    offsets, docs, weights, terms, dense = orc.lexical_test_case()
    assert not li.postings_sorted(offsets, docs)  # the reference test's index is unsorted
    s_off, s_docs, s_w = li.sort_postings(offsets, docs, weights)
    return offsets, docs, weights, terms, dense, s_off, s_docs, s_w


def test_bm25_reference_case_bit_exact(zc, orc, ref_case):
    import torch

    offsets, docs, weights, terms, dense, s_off, s_docs, s_w = ref_case
    n = dense.size
    expected = orc.bm25(offsets, docs, weights, 3000, terms, n)  # unsorted index, reference loop order
    index = zc.LexicalIndex(s_off, s_docs, s_w)
    scores = torch.zeros(n, dtype=torch.float32, device="cuda")
    zc.bm25(index, dev(terms), scores)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(scores.cpu().numpy(), expected)


def test_bm25_accumulates_onto_existing_scores(zc, orc, ref_case):
    import torch

    offsets, docs, weights, terms, dense, s_off, s_docs, s_w = ref_case
    n = dense.size
    expected = orc.bm25(offsets, docs, weights, 3000, terms, n, init=dense)
    scores = dev(dense)
    zc.bm25(zc.LexicalIndex(s_off, s_docs, s_w), dev(terms), scores)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(scores.cpu().numpy(), expected)


def test_max_and_fuse_reference_case(zc, orc, ref_case):
    import torch

    offsets, docs, weights, terms, dense, *_ = ref_case
    n = dense.size
    lex = orc.bm25(offsets, docs, weights, 3000, terms, n)
    peak = orc.max_positive(lex)
    d_max = torch.zeros(1, dtype=torch.float32, device="cuda")
    zc.max_positive(dev(lex), d_max)
    d_dense = dev(dense)
    zc.fuse_scores(d_dense, dev(lex), d_max, 0.6)
    torch.cuda.synchronize()
    assert float(d_max.item()) == peak
    np.testing.assert_array_equal(d_dense.cpu().numpy(), orc.fuse(dense, lex, peak, 0.6))


def test_max_positive_of_negative_values_is_zero(zc):
    import torch

    d_max = torch.zeros(1, dtype=torch.float32, device="cuda")
    zc.max_positive(torch.full((1000,), -3.0, device="cuda"), d_max)
    assert float(d_max.item()) == 0.0


def zipf_case(orc, n, dim, vocab, batch, seed):
    import lexical_index as li

    offsets, docs, weights = li.synthetic_corpus(n, vocab, 40.0, 1.1, seed, k1=0.9, b=0.4)
    terms = li.synthetic_queries(batch, vocab, 1.1, seed + 1)
    corpus = orc.normal_rows(n, dim, 500 + seed)
    queries = orc.normal_rows(batch, dim, 600 + seed)
    return offsets.numpy(), docs.numpy(), weights.numpy(), terms, corpus, queries


@pytest.mark.parametrize("name,dtype", [("f16", 1), ("f32", 0), ("i8row", 4)])
@pytest.mark.parametrize("w", [0.0, 0.5, 1.0])
@pytest.mark.parametrize("batch", [1, 3])
def test_hybrid_topk(zc, orc, name, dtype, w, batch):
    import torch

    n, dim, vocab, k = 30000, 384, 3000, 10
    offsets, docs, weights, terms, corpus, queries = zipf_case(orc, n, dim, vocab, batch, 7 + batch)
    storage, scale, row_scales = orc.encode(corpus, dtype)
    st = dev(storage.view(np.int16) if storage.dtype == np.uint16 else storage)
    idx, val = zc.hybrid_topk(st, dtype, dim, dev(queries), k, zc.LexicalIndex(offsets, docs, weights),
                              dev(terms), w, scale=scale,
                              row_scales=None if row_scales is None else dev(row_scales), metric=0)
    torch.cuda.synchronize()
    ref_idx, ref_val = orc.hybrid_topk(storage, dtype, dim, queries, k, offsets, docs, weights, vocab, terms, w,
                                       scale=scale, row_scales=row_scales, metric=0)
    if name == "i8row" or w == 0.0:
        np.testing.assert_array_equal(idx.cpu().numpy(), ref_idx)
        np.testing.assert_array_equal(val.cpu().numpy(), ref_val)
    else:
        # Full fused score rows for the near-tie check.
        full = np.empty((batch, n), dtype=np.float32)
        dense = orc.scores(storage, dtype, dim, queries, scale=scale, row_scales=row_scales, metric=0)
        for q in range(batch):
            lex = orc.bm25(offsets, docs, weights, vocab, terms[q], n)
            full[q] = orc.fuse(dense[q], lex, orc.max_positive(lex), w)
        assert_topk_parity(idx.cpu().numpy(), val.cpu().numpy(), full, k, exact=False)


def test_hybrid_masked_and_edge_terms(zc, orc):
    """Masked documents keep w * -FLT_MAX + lexical (the reference fuses after masking);
    padding, out-of-vocabulary and repeated term ids; a query with no valid terms."""
    import torch

    n, dim, vocab, k, batch = 20000, 256, 2000, 50, 4
    offsets, docs, weights, terms, corpus, queries = zipf_case(orc, n, dim, vocab, batch, 21)
    terms[1, :] = -1                   # no lexical evidence: lex = 0, inverse 0
    terms[2, 0] = vocab + 5            # out of vocabulary: ignored
    terms[3, 1] = terms[3, 0]          # repeated term counts twice
    mask = np.ones(n, dtype=np.uint8)
    mask[::3] = 0
    storage, _, row_scales = orc.encode(corpus, 4)
    for w in (0.0, 0.3):
        idx, val = zc.hybrid_topk(dev(storage), 4, dim, dev(queries), k, zc.LexicalIndex(offsets, docs, weights),
                                  dev(terms), w, row_scales=dev(row_scales), mask=dev(mask))
        torch.cuda.synchronize()
        ref_idx, ref_val = orc.hybrid_topk(storage, 4, dim, queries, k, offsets, docs, weights, vocab, terms, w,
                                           row_scales=row_scales, mask=mask)
        np.testing.assert_array_equal(idx.cpu().numpy(), ref_idx)
        np.testing.assert_array_equal(val.cpu().numpy(), ref_val)


def test_hybrid_without_terms_is_dense_search(zc, orc):
    import torch

    n, dim = 5000, 128
    corpus = orc.normal_rows(n, dim, 3)
    queries = orc.normal_rows(2, dim, 4)
    storage, _, row_scales = orc.encode(corpus, 4)
    empty = zc.LexicalIndex(np.zeros(2, dtype=np.int64), np.zeros(0, dtype=np.int32), np.zeros(0, dtype=np.float32))
    idx, val = zc.hybrid_topk(dev(storage), 4, dim, dev(queries), 20, empty,
                              torch.empty((2, 0), dtype=torch.int32, device="cuda"), 0.5, row_scales=dev(row_scales))
    torch.cuda.synchronize()
    ref_idx, ref_val = orc.scan_topk(storage, 4, dim, queries, 20, row_scales=row_scales)
    np.testing.assert_array_equal(idx.cpu().numpy(), ref_idx)
    np.testing.assert_array_equal(val.cpu().numpy(), ref_val)


def test_hybrid_sorted_postings_with_runs_and_ragged_tail(zc, orc):
    """Sorted posting lists holding runs of equal documents (a hand-made index), list lengths
    that are not multiples of 4 and a total that is not either: the 16-byte posting loads, the
    run heads found across lanes and groups, and the element loads at the index's end must give
    the oracle's sequential sums bit for bit."""
    import torch

    n, dim, vocab, k, batch = 7000, 128, 40, 50, 5
    rng = np.random.default_rng(77)
    lists = []
    for t in range(vocab):
        df = int(rng.integers(1, 900)) | 1  # odd lengths
        lists.append(np.sort(rng.integers(0, n, size=df)).astype(np.int32))  # with repeats
    offsets = np.zeros(vocab + 1, dtype=np.int64)
    offsets[1:] = np.cumsum([len(x) for x in lists])
    docs = np.concatenate(lists)
    weights = rng.uniform(0.1, 3.0, size=docs.shape[0]).astype(np.float32)
    assert docs.shape[0] % 4 != 0
    terms = np.full((batch, 6), -1, dtype=np.int32)
    for q in range(batch):
        terms[q, :3 + q % 3] = rng.choice(vocab, size=3 + q % 3, replace=False)
    corpus = orc.normal_rows(n, dim, 31)
    queries = orc.normal_rows(batch, dim, 32)
    storage, _, row_scales = orc.encode(corpus, 4)
    idx, val = zc.hybrid_topk(dev(storage), 4, dim, dev(queries), k, zc.LexicalIndex(offsets, docs, weights),
                              dev(terms), 0.0, row_scales=dev(row_scales))
    torch.cuda.synchronize()
    ref_idx, ref_val = orc.hybrid_topk(storage, 4, dim, queries, k, offsets, docs, weights, vocab, terms, 0.0,
                                       row_scales=row_scales)
    np.testing.assert_array_equal(idx.cpu().numpy(), ref_idx)
    np.testing.assert_array_equal(val.cpu().numpy(), ref_val)


def _launch_counts(zc, fn):
    """Runs fn with the library's kernel timing on; returns (scan, lexical, hybrid_select) launch counts."""
    import torch

    zc.kernel_timing(True)
    try:
        fn()
        torch.cuda.synchronize()
        return tuple(zc.kernel_timing_read(t)[1] for t in ("scan", "lexical", "hybrid_select"))
    finally:
        zc.kernel_timing(False)


@pytest.mark.parametrize("k", [1, 10, 32, 33, 150, 300])
def test_hybrid_one_query_edge_cases_bit_exact(zc, orc, k):
    """One query per call takes the hybrid scan (dense rows and BM25 accumulated in the same
    CTAs) and the blend + top-k kernel for k <= 192, the lexical kernel and the blending scan
    above: masked documents, padding / out-of-vocabulary / repeated term ids and a query without
    terms, bit-exact against the oracle on the per-row int8 store (exact integer dot products)."""
    import torch

    n, dim, vocab, batch = 20000, 512, 2000, 4
    offsets, docs, weights, terms, corpus, queries = zipf_case(orc, n, dim, vocab, batch, 21)
    terms[1, :] = -1
    terms[2, 0] = vocab + 5
    terms[3, 1] = terms[3, 0]
    mask = np.ones(n, dtype=np.uint8)
    mask[::3] = 0
    storage, _, row_scales = orc.encode(corpus, 4)
    index = zc.LexicalIndex(offsets, docs, weights)
    d_storage, d_scales, d_mask, d_queries, d_terms = (dev(storage), dev(row_scales), dev(mask), dev(queries),
                                                       dev(terms))
    ws = zc.Workspace()
    fused = k <= 192
    for w in (0.0, 0.3, 1.0):
        for use_mask in (False, True):
            ref_idx, ref_val = orc.hybrid_topk(storage, 4, dim, queries, k, offsets, docs, weights, vocab, terms, w,
                                               row_scales=row_scales, mask=mask if use_mask else None)
            for q in range(batch):
                out = []
                counts = _launch_counts(zc, lambda: out.append(zc.hybrid_topk(
                    d_storage, 4, dim, d_queries[q:q + 1], k, index, d_terms[q:q + 1], w, row_scales=d_scales,
                    mask=d_mask if use_mask else None, workspace=ws)))
                assert counts == ((1, 0, 1) if fused else (1, 1, 0))
                idx, val = out[0]
                np.testing.assert_array_equal(idx.cpu().numpy()[0], ref_idx[q])
                np.testing.assert_array_equal(val.cpu().numpy()[0], ref_val[q])
    assert ws.status() == 0


@pytest.mark.parametrize("n", [1, 63, 64, 1000, 9473, 150000])
def test_hybrid_one_query_corpus_sizes(zc, orc, n):
    """Corpora of one document, less than one tile, one tile, fewer tiles than SMs, a ragged last
    tile and more tiles than SMs: the hybrid scan's CTA ranges (its BM25 accumulator spans the
    CTA's tiles) and the select kernel's ranges (n split evenly over the CTAs) differ, and every
    document must be scored once."""
    import torch

    dim, vocab = 768, 500
    k = min(10, n)
    offsets, docs, weights, terms, corpus, queries = zipf_case(orc, n, dim, vocab, 2, 41)
    storage, _, row_scales = orc.encode(corpus, 4)
    index = zc.LexicalIndex(offsets, docs, weights)
    for w in (0.0, 0.5):
        ref_idx, ref_val = orc.hybrid_topk(storage, 4, dim, queries, k, offsets, docs, weights, vocab, terms, w,
                                           row_scales=row_scales)
        for q in range(2):
            out = []
            counts = _launch_counts(zc, lambda: out.append(zc.hybrid_topk(
                dev(storage), 4, dim, dev(queries[q:q + 1]), k, index, dev(terms[q:q + 1]), w,
                row_scales=dev(row_scales))))
            assert counts == (1, 0, 1)
            idx, val = out[0]
            np.testing.assert_array_equal(idx.cpu().numpy()[0], ref_idx[q])
            np.testing.assert_array_equal(val.cpu().numpy()[0], ref_val[q])


@pytest.mark.parametrize("name,dtype,dim", [("f16", 1, 384), ("f32", 0, 256), ("i8row", 4, 768)])
def test_hybrid_one_query_runs_and_ragged_tail(zc, orc, name, dtype, dim):
    """The hand-made index with runs of equal documents and odd list lengths, one query per call
    (the hybrid scan's lexical warps): with w = 0 the result is lexical / max alone, a sequential
    sum on both sides, bit-exact for every storage type."""
    import torch

    n, vocab, k, batch = 7000, 40, 50, 5
    rng = np.random.default_rng(78)
    lists = []
    for t in range(vocab):
        df = int(rng.integers(1, 900)) | 1
        lists.append(np.sort(rng.integers(0, n, size=df)).astype(np.int32))
    offsets = np.zeros(vocab + 1, dtype=np.int64)
    offsets[1:] = np.cumsum([len(x) for x in lists])
    docs = np.concatenate(lists)
    weights = rng.uniform(0.1, 3.0, size=docs.shape[0]).astype(np.float32)
    terms = np.full((batch, 6), -1, dtype=np.int32)
    for q in range(batch):
        terms[q, :3 + q % 3] = rng.choice(vocab, size=3 + q % 3, replace=False)
    corpus = orc.normal_rows(n, dim, 33)
    queries = orc.normal_rows(batch, dim, 34)
    storage, scale, row_scales = orc.encode(corpus, dtype)
    st = dev(storage.view(np.int16) if storage.dtype == np.uint16 else storage)
    index = zc.LexicalIndex(offsets, docs, weights)
    ref_idx, ref_val = orc.hybrid_topk(storage, dtype, dim, queries, k, offsets, docs, weights, vocab, terms, 0.0,
                                       scale=scale, row_scales=row_scales, metric=0)
    for q in range(batch):
        out = []
        counts = _launch_counts(zc, lambda: out.append(zc.hybrid_topk(
            st, dtype, dim, dev(queries[q:q + 1]), k, index, dev(terms[q:q + 1]), 0.0, scale=scale,
            row_scales=None if row_scales is None else dev(row_scales), metric=0)))
        assert counts == (1, 0, 1)
        idx, val = out[0]
        np.testing.assert_array_equal(idx.cpu().numpy()[0], ref_idx[q])
        np.testing.assert_array_equal(val.cpu().numpy()[0], ref_val[q])


def test_hybrid_one_query_windowed_accumulator(zc, orc):
    """1.3M documents: a CTA's documents no longer fit the BM25 accumulator beside a four-stage
    ring, so the hybrid scan's lexical warps score them in two windows (two rounds of posting
    searches); bit-exact against the oracle on the per-row int8 store."""
    import torch

    n, dim, vocab = 1_300_000, 768, 5000
    offsets, docs, weights, terms, corpus, queries = zipf_case(orc, n, dim, vocab, 2, 51)
    storage, _, row_scales = orc.encode(corpus, 4)
    index = zc.LexicalIndex(offsets, docs, weights)
    d_storage, d_scales = dev(storage), dev(row_scales)
    for w in (0.0, 0.5):
        ref_idx, ref_val = orc.hybrid_topk(storage, 4, dim, queries, 10, offsets, docs, weights, vocab, terms, w,
                                           row_scales=row_scales)
        for q in range(2):
            out = []
            counts = _launch_counts(zc, lambda: out.append(zc.hybrid_topk(
                d_storage, 4, dim, dev(queries[q:q + 1]), 10, index, dev(terms[q:q + 1]), w, row_scales=d_scales)))
            assert counts == (1, 0, 1)
            idx, val = out[0]
            np.testing.assert_array_equal(idx.cpu().numpy()[0], ref_idx[q])
            np.testing.assert_array_equal(val.cpu().numpy()[0], ref_val[q])
