"""GPU tier: fused candidate rescoring (zcgvs_rescore_topk) and the score-matrix form
(zcgvs_gather_rescore) against the CPU oracle's restatement of the reference rescore chain
(src/cuda/rescore.cu gather + second launchTopK + launchRemapIndices).

Per-row int8 stores must match the oracle bit for bit; float stores within 1e-4 (relative to
max(1, |score|)) with id sets equal modulo near-ties. The lossless case mirrors
tests/cpp/test_pipeline.cu:80-108 (fp16 coarse pass, 512 candidates, fp32 rescore to top-10
equals the exact CPU top-10).
"""

from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

FLT_MAX = np.finfo(np.float32).max
DTYPES = {"f32": 0, "f16": 1, "i8": 2, "i8row": 4}
TOL = 1e-4


def to_dev(a):
    import torch

    a = np.ascontiguousarray(a)
    if a.dtype == np.uint16:
        a = a.view(np.int16)
    elif a.dtype == np.uint32:
        a = a.view(np.int32)
    return torch.from_numpy(a).cuda()


def make_candidates(rng, n, batch, m, invalid=0.0):
    cand = np.stack([rng.choice(n, size=m, replace=False) for _ in range(batch)]).astype(np.int32)
    if invalid:
        bad = rng.random(cand.shape) < invalid
        cand[bad] = np.where(rng.random(bad.sum()) < 0.5, -1, n + rng.integers(0, 1000, bad.sum()))
    return cand


def run(zc, orc, name, n, dim, batch, m, k, metric=1, seed=0, invalid=0.0, cand=None):
    import torch

    corpus = orc.normal_rows(n, dim, 301 + dim + seed)
    queries = orc.normal_rows(batch, dim, 401 + dim + seed)
    dtype = DTYPES[name]
    storage, scale, row_scales = orc.encode(corpus, dtype)
    if cand is None:
        cand = make_candidates(np.random.default_rng(seed + m), n, batch, m, invalid)
    d_idx, d_val = zc.rescore_topk(to_dev(storage), dtype, dim, to_dev(queries), to_dev(cand), k, scale=scale,
                                   row_scales=None if row_scales is None else to_dev(row_scales), metric=metric)
    torch.cuda.synchronize()
    ref_idx, ref_val = orc.rescore_topk(storage, dtype, dim, queries, cand, k, scale=scale, row_scales=row_scales,
                                        metric=metric)
    full = orc.scores(storage, dtype, dim, queries, scale=scale, row_scales=row_scales, metric=metric)
    return d_idx.cpu().numpy(), d_val.cpu().numpy(), ref_idx, ref_val, full, cand


def check(gpu_idx, gpu_val, ref_idx, ref_val, full, cand, exact):
    if exact:
        np.testing.assert_array_equal(gpu_idx, ref_idx)
        np.testing.assert_array_equal(gpu_val, ref_val)
        return
    n = full.shape[1]
    for q in range(ref_idx.shape[0]):
        valid = cand[q][(cand[q] >= 0) & (cand[q] < n)]
        nvalid = len(valid)
        ids, vals = gpu_idx[q], gpu_val[q]
        live = ids >= 0
        assert live.sum() == min(nvalid, len(ids)), "wrong number of results"
        assert np.all(vals[~live] == -FLT_MAX) and np.all(ids[~live] == -1), "bad padding"
        assert np.isin(ids[live], valid).all(), "result id is not a candidate"
        exact_scores = full[q][ids[live]]
        assert np.all(np.abs(vals[live] - exact_scores) <= TOL * np.maximum(1.0, np.abs(exact_scores)))
        assert np.all(np.diff(vals[live]) <= TOL), "not descending"
        # Id sets agree except among near-ties at the last kept score.
        ref_live = ref_idx[q][ref_idx[q] >= 0]
        if len(ref_live):
            kth = float(ref_val[q][len(ref_live) - 1])
            band = TOL * max(1.0, abs(kth))
            for doc in set(ref_live.tolist()) ^ set(ids[live].tolist()):
                assert abs(float(full[q][doc]) - kth) <= band, f"doc {doc} differs beyond a near-tie"


SWEEP = [(name, dim, metric)
         for name in ("f32", "f16", "i8", "i8row")
         for dim in (256, 1024, 100, 97)
         for metric in (1, 2)
         if not (metric == 2 and name == "i8row")]


@pytest.mark.parametrize("name,dim,metric", SWEEP)
def test_rescore_sweep(zc, orc, name, dim, metric):
    out = run(zc, orc, name, 6000, dim, 4, 512, 10, metric=metric)
    check(*out, exact=(name == "i8row"))


@pytest.mark.parametrize("m,k,batch", [(m, k, b) for m, k in ((1, 1), (7, 7), (33, 5), (1000, 10), (1024, 1024),
                                                                (2048, 100), (8192, 1024))
                                         for b in (1, 3, 64) if not (b == 64 and m > 2048)])
def test_rescore_widths(zc, orc, m, k, batch):
    out = run(zc, orc, "f16", 10000, 1024, batch, m, k, seed=batch)
    check(*out, exact=False)


@pytest.mark.parametrize("m,k", [(1000, 10), (1024, 1024), (64, 64)])
def test_rescore_i8row_exact_widths(zc, orc, m, k):
    out = run(zc, orc, "i8row", 5000, 768, 5, m, k, seed=m)
    check(*out, exact=True)


@pytest.mark.parametrize("name", ["f32", "i8row"])
def test_rescore_invalid_candidates(zc, orc, name):
    out = run(zc, orc, name, 3000, 128, 6, 300, 50, invalid=0.3)
    check(*out, exact=(name == "i8row"))


def test_rescore_fewer_valid_than_k(zc, orc):
    cand = np.full((2, 40), -1, dtype=np.int32)
    cand[0, :5] = [10, 20, 30, 40, 50]
    out = run(zc, orc, "i8row", 1000, 64, 2, 40, 20, cand=cand)
    check(*out, exact=True)
    gpu_idx, gpu_val = out[0], out[1]
    assert (gpu_idx[1] == -1).all() and (gpu_val[1] == -FLT_MAX).all()


def test_rescore_duplicate_candidates(zc, orc):
    cand = np.array([[5, 5, 9, 9, 9, 1, 2, 3]], dtype=np.int32)
    out = run(zc, orc, "i8row", 100, 64, 1, 8, 8, cand=cand)
    check(*out, exact=True)


def test_lossless_rescore_matches_exact_search(zc, orc):
    """tests/cpp/test_pipeline.cu:80-108: fp16 coarse top-512, fp32 rescore to top-10 ==
    exact fp32 CPU top-10 (cosine on normalised rows)."""
    import torch

    n, dim, m, k = 8192, 256, 512, 10
    corpus = orc.normal_rows(n, dim, 31)
    query = orc.normal_rows(1, dim, 32)
    coarse, _, _ = orc.encode(corpus, 1)
    c_idx, _ = zc.scan_topk(to_dev(coarse), 1, dim, to_dev(query), m, metric=0)
    idx, val = zc.rescore_topk(to_dev(corpus), 0, dim, to_dev(query), c_idx, k, metric=0)
    torch.cuda.synchronize()
    ref_idx, ref_val = orc.scan_topk(corpus, 0, dim, query, k, metric=0)
    np.testing.assert_array_equal(idx.cpu().numpy(), ref_idx)
    np.testing.assert_allclose(val.cpu().numpy(), ref_val, rtol=0, atol=1e-4)


@pytest.mark.parametrize("name", ["f32", "f16", "i8", "i8row"])
def test_gather_rescore_matrix(zc, orc, name):
    import torch

    n, dim, batch, m = 4000, 200, 3, 700
    corpus = orc.normal_rows(n, dim, 77)
    queries = orc.normal_rows(batch, dim, 78)
    dtype = DTYPES[name]
    storage, scale, row_scales = orc.encode(corpus, dtype)
    cand = make_candidates(np.random.default_rng(5), n, batch, m, invalid=0.1)
    vals = zc.gather_rescore(to_dev(storage), dtype, dim, to_dev(queries), to_dev(cand), scale=scale,
                             row_scales=None if row_scales is None else to_dev(row_scales))
    torch.cuda.synchronize()
    vals = vals.cpu().numpy()
    full = orc.scores(storage, dtype, dim, queries, scale=scale, row_scales=row_scales)
    for q in range(batch):
        ok = (cand[q] >= 0) & (cand[q] < n)
        assert (vals[q][~ok] == -FLT_MAX).all()
        ref = full[q][cand[q][ok]]
        if name == "i8row":
            np.testing.assert_array_equal(vals[q][ok], ref)
        else:
            np.testing.assert_allclose(vals[q][ok], ref, rtol=0, atol=TOL)
