"""Pins the CPU oracle against the reference's own code (CPU tier, no GPU).

The golden fixtures were produced by tests/golden/make_golden.py from the reference's
python/zcgvs_tools/formats.py and tests/cpp/cpu_reference.hpp; the known-answer vectors below
are the ones the reference's tests/python/test_formats.py asserts.
"""

from __future__ import annotations

import zlib

import numpy as np
import pytest


def crc(a):
    return zlib.crc32(np.ascontiguousarray(a).tobytes())


def test_pack_binary_bit_order_kat(orc):
    # tests/python/test_formats.py:36-52: dims 0, 33 and 129 set in a 130-dim row.
    m = np.full((1, 130), -1.0, dtype=np.float32)
    m[0, 0] = m[0, 33] = m[0, 129] = 1.0
    packed = orc.pack_binary(m)
    assert packed.shape == (1, 5)
    assert packed[0].tolist() == [1, 2, 0, 0, 2]
    assert packed[0, 4] >> 2 == 0  # padding bits stay clear


def test_row_strides(golden):
    f = golden["formats"]
    # tests/python/test_formats.py:27-33
    assert int(f["stride_3_384"]) == 48 and int(f["stride_3_130"]) == 20
    for dim in (130, 384, 97, 1024, 33):
        assert int(f[f"stride_0_{dim}"]) == 4 * dim
        assert int(f[f"stride_1_{dim}"]) == 2 * dim
        assert int(f[f"stride_2_{dim}"]) == dim
        assert int(f[f"stride_3_{dim}"]) == 4 * ((dim + 31) // 32)


@pytest.mark.parametrize("dim", [130, 384, 97, 1024, 33])
def test_formats_conventions(orc, golden, dim):
    f = golden["formats"]
    m = orc.normal_rows(16, dim, 3 + dim)
    assert crc(m) == int(f[f"input_crc_{dim}"]), "seeded generator drifted"
    np.testing.assert_array_equal(orc.pack_binary(m), f[f"pack_{dim}"])
    scale = orc.matrix_scale(m)
    assert np.float32(scale) == f[f"q8scale_{dim}"]
    q = orc.quantize_i8(m, scale)
    np.testing.assert_array_equal(q, f[f"q8_{dim}"])
    # tests/python/test_formats.py:55-63: symmetric, bounded, error <= scale
    assert q.min() >= -127 and q.max() <= 127
    assert np.max(np.abs(q.astype(np.float32) * np.float32(scale) - m)) <= scale


def test_fp16_rounding_matches_ieee(orc):
    rng = np.random.default_rng(5)
    x = np.concatenate([rng.normal(size=20000).astype(np.float32) * 7,
                        np.array([0.0, -0.0, 6.1e-5, 6.0e-8, 2.98e-8, 65504.0, 65519.0, 1e-9], np.float32)])
    np.testing.assert_array_equal(orc.to_f16_bits(x), x.astype(np.float16).view(np.uint16))


@pytest.mark.parametrize("dim", [97, 100, 256, 384])
def test_oracle_scores_equal_reference_cpu(orc, golden, dim):
    g = golden["scan_small"]
    corpus = orc.normal_rows(512, dim, 11 + dim)
    queries = orc.normal_rows(3, dim, 97 + dim)
    assert crc(corpus) == int(g[f"crc_corpus_{dim}"]) and crc(queries) == int(g[f"crc_queries_{dim}"])
    # float32
    s = orc.scores(corpus, orc.DTYPE_F32, dim, queries)
    np.testing.assert_array_equal(s, g[f"f32_scores_{dim}"])
    np.testing.assert_array_equal(orc.topk(s, 10)[0], g[f"f32_top10_{dim}"])
    # float16 storage
    s = orc.scores(orc.to_f16_bits(corpus), orc.DTYPE_F16, dim, queries)
    np.testing.assert_array_equal(s, g[f"f16_scores_{dim}"])
    np.testing.assert_array_equal(orc.topk(s, 10)[0], g[f"f16_top10_{dim}"])
    # int8 per-matrix storage, scale 1/127 (tests/cpp/test_quantized.cu:40-44)
    scale = np.float32(1.0 / 127.0)
    s = orc.scores(orc.quantize_i8(corpus, scale), orc.DTYPE_I8, dim, queries, scale=float(scale))
    np.testing.assert_array_equal(s, g[f"i8_scores_{dim}"])
    np.testing.assert_array_equal(orc.topk(s, 10)[0], g[f"i8_top10_{dim}"])
    # binary
    packed = orc.pack_binary(corpus)
    np.testing.assert_array_equal(packed, g[f"bin_packed_{dim}"])
    s = orc.scores(packed, orc.DTYPE_BINARY, dim, queries)
    ham = g[f"bin_hamming_{dim}"]
    np.testing.assert_array_equal(s, ((dim - 2 * ham).astype(np.float32) / np.float32(dim)))


def test_reference_kats(orc, golden):
    k = golden["kat"]
    corpus = orc.normal_rows(8192, 256, 31)
    query = orc.normal_rows(1, 256, 32)
    assert (crc(corpus) ^ crc(query)) == int(k["pipeline_crc"])
    idx, _ = orc.scan_topk(corpus, orc.DTYPE_F32, 256, query, 10)
    np.testing.assert_array_equal(idx, k["pipeline_top10"])
    s = orc.uniform(5000, 7, -100.0, 100.0)
    assert crc(s) == int(k["topk5000_crc"])
    np.testing.assert_array_equal(orc.topk(s, 100)[0], k["topk5000_top100"])
    s = orc.uniform(1000000, 17, -1000.0, 1000.0)
    assert crc(s) == int(k["topk1m_crc"])
    np.testing.assert_array_equal(orc.topk(s, 512)[0], k["topk1m_top512"])


def test_per_row_int8_exactness(orc):
    x = orc.normal_rows(300, 768, 1001)
    q, s = orc.quantize_rows_i8(x)
    assert q.min() >= -127 and q.max() <= 127
    np.testing.assert_array_equal(s, np.abs(x).max(axis=1) / np.float32(127.0))
    queries = orc.normal_rows(4, 768, 1002)
    got = orc.scores(q, orc.DTYPE_I8_ROW, 768, queries, row_scales=s)
    qq, qs = orc.quantize_rows_i8(queries)
    dots = qq.astype(np.int64) @ q.astype(np.int64).T
    expect = (dots.astype(np.float32) * qs[:, None]).astype(np.float32) * s[None, :]
    np.testing.assert_array_equal(got, expect.astype(np.float32))


def test_topk_tie_order(orc):
    s = np.array([[1.0, 3.0, 3.0, -0.0, 0.0, 3.0, 2.0]], dtype=np.float32)
    idx, val = orc.topk(s, 5)
    assert idx[0].tolist() == [1, 2, 5, 6, 0]
    idx, val = orc.topk(s, 7)
    assert idx[0].tolist()[-2:] == [3, 4]  # -0.0 ties +0.0, lower id first


def test_oracle_bm25_matches_sequential_float32_loop(orc):
    """orc_bm25 against an independent float32 restatement of tests/cpp/test_lexical.cu:71-80
    on the reference test's own index (regenerated from its seeds)."""
    offsets, docs, weights, terms, dense = orc.lexical_test_case()
    assert offsets[-1] == docs.size and terms[-1] == -1 and dense.size == 20000
    expected = [np.float32(0.0)] * 20000
    for term in terms:
        if term < 0:
            continue
        for p in range(offsets[term], offsets[term + 1]):
            expected[docs[p]] = np.float32(expected[docs[p]] + weights[p])
    np.testing.assert_array_equal(orc.bm25(offsets, docs, weights, 3000, terms, 20000),
                                  np.array(expected, dtype=np.float32))


def test_oracle_fuse_order(orc):
    dense = np.array([0.5, -1.0, 0.25], dtype=np.float32)
    lex = np.array([3.0, 0.0, 1.5], dtype=np.float32)
    w = np.float32(0.6)
    inv = np.float32(1.0) / np.float32(3.0)
    expected = [np.float32(np.float32(w * d) + np.float32(np.float32(np.float32(np.float32(1.0) - w) * l) * inv))
                for d, l in zip(dense, lex)]
    np.testing.assert_array_equal(orc.fuse(dense, lex, 3.0, 0.6), np.array(expected, dtype=np.float32))
    assert orc.max_positive(np.array([-2.0, -1.0], dtype=np.float32)) == 0.0


def test_sort_postings_keeps_per_document_order():
    import lexical_index as li

    offsets = np.array([0, 4, 4, 7], dtype=np.int64)
    docs = np.array([9, 2, 9, 1, 5, 5, 0], dtype=np.int32)
    weights = np.arange(7, dtype=np.float32)
    assert not li.postings_sorted(offsets, docs)
    o, d, w = li.sort_postings(offsets, docs, weights)
    np.testing.assert_array_equal(d, [1, 2, 9, 9, 0, 5, 5])
    np.testing.assert_array_equal(w, [3, 1, 0, 2, 6, 4, 5])
    assert li.postings_sorted(o, d)


def test_bm25_weights_match_builder_formula():
    import math

    import torch

    import lexical_index as li

    # Two documents, three terms: doc 0 = [0, 0, 1], doc 1 = [1, 2].
    doc_ids = torch.tensor([0, 0, 1, 1])
    term_ids = torch.tensor([0, 1, 1, 2])
    tf = torch.tensor([2, 1, 1, 1])
    lengths = torch.tensor([3, 2])
    offsets, docs, weights = li.build_csr(doc_ids, term_ids, tf, lengths, 3, k1=0.9, b=0.4)
    avgdl = 2.5
    expected = []
    for d, t, f in [(0, 0, 2), (0, 1, 1), (1, 1, 1), (1, 2, 1)]:
        df = {0: 1, 1: 2, 2: 1}[t]
        idf = math.log(1.0 + (2 - df + 0.5) / (df + 0.5))
        norm = 0.9 * (1.0 - 0.4 + 0.4 * [3, 2][d] / avgdl)
        expected.append(np.float32(idf * (f * 1.9) / (f + norm)))
    np.testing.assert_array_equal(offsets.numpy(), [0, 1, 3, 4])
    np.testing.assert_array_equal(docs.numpy(), [0, 0, 1, 1])
    np.testing.assert_array_equal(weights.numpy(), np.array(expected, dtype=np.float32))


def test_bm25_weights_match_builder_loop_on_a_random_corpus():
    """lexical_index.build_csr against the reference builder's loop restated
    (python/zcgvs_tools/build_lexical.py:125-162: per-document term counts, document
    frequencies, idf = ln(1 + (N - df + 0.5) / (df + 0.5)), the BM25 weight in float64, stored as
    float32, postings by term then document), bit for bit, on 2,000 random documents."""
    import math
    from collections import defaultdict

    import torch

    import lexical_index as li

    rng = np.random.default_rng(11)
    n_docs, vocab, k1, b = 2000, 500, 0.9, 0.4
    lengths = rng.poisson(30, n_docs)
    docs_tokens = [rng.zipf(1.3, size=int(L)) % vocab for L in lengths]
    # The reference loop.
    tfs = []
    dfreq = defaultdict(int)
    for toks in docs_tokens:
        counts = defaultdict(int)
        for t in toks:
            counts[int(t)] += 1
        tfs.append(counts)
        for t in counts:
            dfreq[t] += 1
    lens = np.asarray([float(len(t)) for t in docs_tokens], dtype=np.float64)
    avg = float(lens.mean()) or 1.0
    postings = defaultdict(list)
    for d, counts in enumerate(tfs):
        norm = k1 * (1.0 - b + b * lens[d] / avg)
        for t, f in counts.items():
            df = dfreq[t]
            idf = math.log(1.0 + (n_docs - df + 0.5) / (df + 0.5))
            postings[t].append((d, idf * (f * (k1 + 1.0)) / (f + norm)))
    ref_off = [0]
    ref_docs, ref_w = [], []
    for t in range(vocab):
        for d, w in postings.get(t, ()):
            ref_docs.append(d)
            ref_w.append(w)
        ref_off.append(len(ref_docs))
    # The same corpus as unique (doc, term, tf) triples for build_csr.
    trip = [(d, t, f) for d, counts in enumerate(tfs) for t, f in counts.items()]
    doc_ids = torch.tensor([x[0] for x in trip])
    term_ids = torch.tensor([x[1] for x in trip])
    tf = torch.tensor([x[2] for x in trip])
    offsets, docs, weights = li.build_csr(doc_ids, term_ids, tf, torch.tensor(lengths), vocab, k1=k1, b=b)
    np.testing.assert_array_equal(offsets.numpy(), ref_off)
    np.testing.assert_array_equal(docs.numpy(), ref_docs)
    np.testing.assert_array_equal(weights.numpy(), np.asarray(ref_w, dtype=np.float32))
