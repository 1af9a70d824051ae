"""GPU tier: the fused scan + top-k and the score-matrix kernels against the CPU oracle.

Cases follow the reference's own harnesses: the 44-case storage x dim x metric x mask sweep of
tests/cpp/test_scan_paths.cu (N = 20000, batch 11 = one full pass of 8 plus a ragged pass),
the batched top-k of tests/cpp/test_batched.cu, the masked -FLT_MAX contract of
tests/cpp/test_metrics_filter.cu, plus the BASELINE int8 configuration at full size.

Integer-valued paths (per-row int8, binary) must match the oracle bit for bit, ids and scores;
float paths within 1e-4 (relative to max(1, |score|)) with id sets equal modulo near-ties.
"""

from __future__ import annotations

import numpy as np
import pytest

from conftest import assert_topk_parity

pytestmark = pytest.mark.gpu

FLT_MAX = np.finfo(np.float32).max
DTYPES = {"f32": 0, "f16": 1, "i8": 2, "bin": 3, "i8row": 4}


def to_dev(a):
    import torch

    a = np.ascontiguousarray(a)
    if a.dtype == np.uint16:
        a = a.view(np.int16)
    elif a.dtype == np.uint32:
        a = a.view(np.int32)
    return torch.from_numpy(a).cuda()


def make_store(orc, name, corpus):
    dtype = DTYPES[name]
    scale = np.float32(1.0 / 127.0) if name == "i8" else None
    storage, s, row_scales = orc.encode(corpus, dtype, scale=None if scale is None else float(scale))
    return dtype, storage, float(s), row_scales


def run_topk(zc, orc, name, n, dim, batch, k, metric=0, mask_every=0, seed=0, id_base=0):
    import torch

    corpus = orc.normal_rows(n, dim, 11 + dim + seed)
    queries = orc.normal_rows(batch, dim, 97 + dim + seed)
    dtype, storage, scale, row_scales = make_store(orc, name, corpus)
    mask = None
    if mask_every:
        mask = np.ones(n, dtype=np.uint8)
        mask[::mask_every] = 0
    d_idx, d_val = zc.scan_topk(to_dev(storage), dtype, dim, to_dev(queries), k, scale=scale,
                                row_scales=None if row_scales is None else to_dev(row_scales),
                                mask=None if mask is None else to_dev(mask), metric=metric,
                                id_base=id_base)
    torch.cuda.synchronize()
    ref = orc.scores(storage, dtype, dim, queries, scale=scale, row_scales=row_scales, mask=mask,
                     metric=metric)
    return d_idx.cpu().numpy(), d_val.cpu().numpy(), ref, name in ("bin", "i8row")


SWEEP = [(name, dim, metric, mask_every)
         for dim in (384, 768, 100, 97)
         for name in ("f32", "f16", "i8", "bin", "i8row")
         for metric, mask_every in ((1, 0), (1, 7), (2, 7))
         if not (metric == 2 and name in ("bin", "i8row"))]


@pytest.mark.parametrize("name,dim,metric,mask_every", SWEEP)
def test_scan_topk_sweep(zc, orc, name, dim, metric, mask_every):
    idx, val, ref, exact = run_topk(zc, orc, name, 20000, dim, 11, 64, metric, mask_every)
    assert_topk_parity(idx, val, ref, 64, exact=exact)


@pytest.mark.parametrize("name", ["f32", "f16", "i8", "bin", "i8row"])
@pytest.mark.parametrize("batch", [1, 2, 3, 8, 16])
def test_scan_topk_batches(zc, orc, name, batch):
    idx, val, ref, exact = run_topk(zc, orc, name, 8192, 256, batch, 10, seed=batch)
    assert_topk_parity(idx, val, ref, 10, exact=exact)


@pytest.mark.parametrize("name", ["f32", "i8row", "bin"])
@pytest.mark.parametrize("n,k", [(37, 37), (100, 100), (5000, 1024), (4099, 513), (1, 1)])
def test_scan_topk_edges(zc, orc, name, n, k):
    idx, val, ref, exact = run_topk(zc, orc, name, n, 128, 3, k)
    assert_topk_parity(idx, val, ref, k, exact=exact)


def test_scan_topk_id_base_and_mask_everything_but_few(zc, orc):
    n, dim, k = 3000, 64, 16
    idx, val, ref, _ = run_topk(zc, orc, "i8row", n, dim, 2, k, id_base=1000000)
    assert_topk_parity(idx, val, ref, k, exact=True, id_base=1000000)
    # Only 5 documents allowed: the other 11 slots are masked documents at -FLT_MAX, lowest id first.
    import torch

    corpus = orc.normal_rows(n, dim, 5)
    queries = orc.normal_rows(1, dim, 6)
    storage, _, rs = orc.encode(corpus, orc.DTYPE_I8_ROW)
    mask = np.zeros(n, dtype=np.uint8)
    allowed = [7, 123, 999, 2048, 2999]
    mask[allowed] = 1
    d_idx, d_val = zc.scan_topk(to_dev(storage), zc.DTYPE_I8_ROW, dim, to_dev(queries), k,
                                row_scales=to_dev(rs), mask=to_dev(mask))
    torch.cuda.synchronize()
    got = d_idx.cpu().numpy()[0]
    assert sorted(got[:5].tolist()) == allowed
    assert got[5:].tolist() == [i for i in range(n) if i not in allowed][:11]
    assert (d_val.cpu().numpy()[0, 5:] == -FLT_MAX).all()


def test_int8_per_row_baseline_config_full_size(zc, orc):
    """BASELINE config 2 at full size: 1,000,000 x 768 per-row int8, top-100, batches 1 and 16."""
    import torch

    n, dim = 1_000_000, 768
    corpus = orc.normal_rows(n, dim, 2001)
    storage, _, rs = orc.encode(corpus, orc.DTYPE_I8_ROW)
    d_store, d_rs = to_dev(storage), to_dev(rs)
    for batch, seed in ((1, 2002), (16, 2003)):
        queries = orc.normal_rows(batch, dim, seed)
        d_idx, d_val = zc.scan_topk(d_store, zc.DTYPE_I8_ROW, dim, to_dev(queries), 100, row_scales=d_rs)
        torch.cuda.synchronize()
        ridx, rval = orc.scan_topk(storage, orc.DTYPE_I8_ROW, dim, queries, 100, row_scales=rs)
        np.testing.assert_array_equal(d_idx.cpu().numpy(), ridx)
        np.testing.assert_array_equal(d_val.cpu().numpy(), rval)


def test_repeat_calls_are_deterministic_and_reuse_workspace(zc, orc):
    import torch

    n, dim = 50000, 384
    corpus = orc.normal_rows(n, dim, 77)
    queries = orc.normal_rows(4, dim, 78)
    f16 = to_dev(orc.to_f16_bits(corpus))
    q = to_dev(queries)
    ws = zc.Workspace()
    first = [t.clone() for t in zc.scan_topk(f16, zc.DTYPE_F16, dim, q, 100, workspace=ws)]
    for _ in range(5):
        again = zc.scan_topk(f16, zc.DTYPE_F16, dim, q, 100, workspace=ws)
        torch.cuda.synchronize()
        assert torch.equal(first[0], again[0]) and torch.equal(first[1], again[1])
    assert ws.status() == 0


@pytest.mark.parametrize("name,dim,metric,mask_every", SWEEP)
def test_similarity_matrix_sweep(zc, orc, name, dim, metric, mask_every):
    """tests/cpp/test_scan_paths.cu:109-166: every score of [11, 20000] within 1e-4, masked
    documents exactly -FLT_MAX."""
    import torch

    n, batch = 20000, 11
    corpus = orc.normal_rows(n, dim, 11 + dim)
    queries = orc.normal_rows(batch, dim, 97 + dim)
    dtype, storage, scale, row_scales = make_store(orc, name, corpus)
    mask = None
    if mask_every:
        mask = np.ones(n, dtype=np.uint8)
        mask[::mask_every] = 0
    q_dev = to_dev(orc.pack_binary(queries)) if name == "bin" else to_dev(queries)
    out = zc.similarity(to_dev(storage), dtype, dim, q_dev, scale=scale,
                        row_scales=None if row_scales is None else to_dev(row_scales),
                        mask=None if mask is None else to_dev(mask), metric=metric)
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    ref = orc.scores(storage, dtype, dim, queries, scale=scale, row_scales=row_scales, mask=mask, metric=metric)
    if mask is not None:
        assert (got[:, mask == 0] == -FLT_MAX).all()
        assert (got[:, mask == 1] != -FLT_MAX).all()
    if name in ("bin", "i8row"):
        np.testing.assert_array_equal(got, ref)
    else:
        np.testing.assert_allclose(got, ref, rtol=0, atol=1e-4)


FAST_CASES = [(name, dim) for name, dims in (("i8row", (512, 768, 1024, 1536, 2048)),
                                             ("f32", (384, 512)),
                                             ("f16", (384, 768, 1024)),
                                             ("i8", (512, 768, 1024)))
              for dim in dims]


@pytest.mark.parametrize("name,dim", FAST_CASES)
@pytest.mark.parametrize("n,k,mask_every", [(100000, 100, 0), (33333, 256, 5), (4097, 1, 0), (70001, 10, 3)])
def test_single_query_warp_specialised_path(zc, orc, name, dim, n, k, mask_every):
    """Batch 1 over 16-byte-multiple rows takes the warp-specialised kernel (scan_fast.cuh):
    every storage, sweep depth 2-8, ragged corpus sizes, masks and k from 1 to 256."""
    idx, val, ref, exact = run_topk(zc, orc, name, n, dim, 1, k, 1, mask_every, seed=dim + k)
    assert_topk_parity(idx, val, ref, k, exact=exact)


@pytest.mark.parametrize("order", ["ascending", "descending", "constant"])
def test_single_query_adversarial_orders_spill_and_ties(zc, orc, order):
    """Ascending scores make every row beat the running threshold, so every CTA overflows its
    shared candidate buffer into the global spill area; constant scores make every row tie and
    the order is decided by id alone."""
    import torch

    n, dim, k = 600_000, 128, 100
    q = orc.normal_rows(1, dim, 4242)
    if order == "constant":
        t = np.ones(n, dtype=np.float32)
    else:
        t = np.linspace(0.0, 1.0, n, dtype=np.float32)
        if order == "descending":
            t = t[::-1].copy()
    corpus = (t[:, None] * q).astype(np.float32)
    d_idx, d_val = zc.scan_topk(to_dev(corpus), zc.DTYPE_F32, dim, to_dev(q), k)
    torch.cuda.synchronize()
    ref = orc.scores(corpus, orc.DTYPE_F32, dim, q)
    assert_topk_parity(d_idx.cpu().numpy(), d_val.cpu().numpy(), ref, k, exact=False)
    if order == "constant":
        assert d_idx.cpu().numpy()[0].tolist() == list(range(k))
