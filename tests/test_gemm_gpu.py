"""GPU tier: the tensor-core batched search (tcgen05 / TMEM / TMA) against the CPU oracle.

Per-row int8 corpora score an exact int32 dot, and 1-bit corpora an exact integer dot of sign
vectors (their Hamming score), so the tensor-core score matrix and top-k must equal the oracle
(and zcgvs_scan_topk) bit for bit. fp16 corpora take fp16 queries (the tests
round their queries to fp16 first, as BASELINE's fp16 workloads draw them) and accumulate in
fp32 in the tensor core's order: scores within 1e-4, id sets equal modulo near-ties. Shapes cover
partial query blocks (batch not a multiple of 128), partial document tiles (N not a multiple
of 256), masks, id_base and k from 1 to 1024.
"""

from __future__ import annotations

import numpy as np
import pytest

from conftest import assert_topk_parity

pytestmark = pytest.mark.gpu

FLT_MAX = np.finfo(np.float32).max


def dev(a):
    import torch

    a = np.ascontiguousarray(a)
    if a.dtype == np.uint16:
        a = a.view(np.int16)
    elif a.dtype == np.uint32:
        a = a.view(np.int32)
    return torch.from_numpy(a).cuda()


def fp16_round(orc, x):
    bits = orc.to_f16_bits(x)
    return bits.view(np.float16).astype(np.float32)


def case(orc, dtype, n, dim, batch, seed):
    corpus = orc.normal_rows(n, dim, 700 + seed)
    queries = orc.normal_rows(batch, dim, 800 + seed)
    if dtype == 1:
        queries = fp16_round(orc, queries)
    storage, _, row_scales = orc.encode(corpus, dtype)
    return storage, row_scales, queries


@pytest.mark.parametrize("n,dim,batch", [(1000, 256, 200), (777, 128, 5), (3000, 768, 130)])
def test_gemm_similarity_i8row_exact(zc, orc, n, dim, batch):
    import torch

    storage, row_scales, queries = case(orc, 4, n, dim, batch, 1)
    mask = np.ones(n, dtype=np.uint8)
    mask[::5] = 0
    out = zc.gemm_similarity(dev(storage), 4, dim, dev(queries), row_scales=dev(row_scales), mask=dev(mask))
    torch.cuda.synchronize()
    ref = orc.scores(storage, 4, dim, queries, row_scales=row_scales, mask=mask)
    np.testing.assert_array_equal(out.cpu().numpy(), ref)


@pytest.mark.parametrize("n,dim,batch", [(1000, 256, 200), (600, 64, 3), (2000, 768, 129)])
def test_gemm_similarity_f16(zc, orc, n, dim, batch):
    import torch

    storage, _, queries = case(orc, 1, n, dim, batch, 2)
    out = zc.gemm_similarity(dev(storage), 1, dim, dev(queries))
    torch.cuda.synchronize()
    ref = orc.scores(storage, 1, dim, queries)
    np.testing.assert_allclose(out.cpu().numpy(), ref, rtol=0, atol=1e-4)


@pytest.mark.parametrize("n,dim,batch,k", [(5000, 256, 130, 10), (20000, 768, 256, 100), (3000, 128, 7, 1),
                                           (5000, 128, 64, 1024), (70000, 384, 300, 100)])
def test_gemm_topk_i8row_exact(zc, orc, n, dim, batch, k):
    import torch

    storage, row_scales, queries = case(orc, 4, n, dim, batch, 3)
    ws = zc.Workspace()
    idx, val = zc.gemm_topk(dev(storage), 4, dim, dev(queries), k, row_scales=dev(row_scales), workspace=ws)
    torch.cuda.synchronize()
    ref_i, ref_v = orc.scan_topk(storage, 4, dim, queries, k, row_scales=row_scales)
    np.testing.assert_array_equal(idx.cpu().numpy(), ref_i)
    np.testing.assert_array_equal(val.cpu().numpy(), ref_v)
    assert ws.status() == 0


def test_gemm_topk_i8row_mask_and_id_base(zc, orc):
    import torch

    n, dim, batch, k = 9000, 256, 150, 40
    storage, row_scales, queries = case(orc, 4, n, dim, batch, 4)
    mask = np.ones(n, dtype=np.uint8)
    mask[1::3] = 0
    idx, val = zc.gemm_topk(dev(storage), 4, dim, dev(queries), k, row_scales=dev(row_scales), mask=dev(mask),
                            id_base=1000)
    torch.cuda.synchronize()
    ref_i, ref_v = orc.scan_topk(storage, 4, dim, queries, k, row_scales=row_scales, mask=mask, id_base=1000)
    np.testing.assert_array_equal(idx.cpu().numpy(), ref_i)
    np.testing.assert_array_equal(val.cpu().numpy(), ref_v)


def test_gemm_topk_equals_streaming_scan(zc, orc):
    """Same per-row int8 search through the CUDA-core scan and the tensor-core scan."""
    import torch

    n, dim, batch, k = 30000, 768, 160, 100
    storage, row_scales, queries = case(orc, 4, n, dim, batch, 5)
    a = zc.gemm_topk(dev(storage), 4, dim, dev(queries), k, row_scales=dev(row_scales))
    b = zc.scan_topk(dev(storage), 4, dim, dev(queries), k, row_scales=dev(row_scales))
    torch.cuda.synchronize()
    np.testing.assert_array_equal(a[0].cpu().numpy(), b[0].cpu().numpy())
    np.testing.assert_array_equal(a[1].cpu().numpy(), b[1].cpu().numpy())


@pytest.mark.parametrize("n,dim,batch,k", [(20000, 384, 300, 50), (6000, 768, 128, 100), (4000, 64, 20, 10)])
def test_gemm_topk_f16(zc, orc, n, dim, batch, k):
    import torch

    storage, _, queries = case(orc, 1, n, dim, batch, 6)
    idx, val = zc.gemm_topk(dev(storage), 1, dim, dev(queries), k)
    torch.cuda.synchronize()
    ref = orc.scores(storage, 1, dim, queries)
    assert_topk_parity(idx.cpu().numpy(), val.cpu().numpy(), ref, k, exact=False)


def test_gemm_rejects_unsupported(zc):
    import torch

    x = torch.zeros((100, 100), dtype=torch.int8, device="cuda")
    q = torch.zeros((2, 100), device="cuda")
    with pytest.raises(zc.ZcgvsError):
        zc.gemm_topk(x, 4, 100, q, 5, row_scales=torch.ones(100, device="cuda"))  # 100-byte rows
    with pytest.raises(zc.ZcgvsError):
        zc.gemm_topk(torch.zeros((100, 128), device="cuda"), 0, 128, torch.zeros((2, 128), device="cuda"), 5)


def test_gemm_topk_overflow_retry_is_exact(zc, orc):
    """A corpus where every document scores the same: the threshold keeps all of them, the
    16384-slot candidate buffer overflows, and the retry pass must still return the exact
    (score desc, id asc) top-k."""
    import torch

    n, dim, batch, k = 40000, 128, 3, 50
    storage = np.ones((n, dim), dtype=np.int8)
    row_scales = np.full(n, 0.01, dtype=np.float32)
    queries = np.ones((batch, dim), dtype=np.float32)
    ws = zc.Workspace()
    idx, val = zc.gemm_topk(dev(storage), 4, dim, dev(queries), k, row_scales=dev(row_scales), workspace=ws)
    torch.cuda.synchronize()
    ref_i, ref_v = orc.scan_topk(storage, 4, dim, queries, k, row_scales=row_scales)
    np.testing.assert_array_equal(idx.cpu().numpy(), ref_i)
    np.testing.assert_array_equal(val.cpu().numpy(), ref_v)
    assert ws.status() == 0


def test_gemm_topk_statistical_bound_fallback_is_exact(zc, orc):
    """The threshold sample (the first tiles) holds 20 documents far above the rest, one per
    chunk: the statistical bound (16th chunk maximum) lets only those 20 through (< k), the safe
    bound keeps every document (fewer sample chunks than k) and overflows the candidate buffer,
    and the raised bound of the second retry must still return the exact top-k."""
    import torch

    n, dim, batch, k = 40000, 128, 3, 100
    rng = np.random.default_rng(9)
    storage = rng.integers(-20, 21, size=(n, dim), dtype=np.int8)
    v = rng.integers(60, 127, size=dim).astype(np.int8)
    for i in range(20):
        storage[32 * i] = v
    row_scales = np.full(n, 0.01, dtype=np.float32)
    queries = np.tile(v.astype(np.float32) / 127.0, (batch, 1))
    ws = zc.Workspace()
    idx, val = zc.gemm_topk(dev(storage), 4, dim, dev(queries), k, row_scales=dev(row_scales), workspace=ws)
    torch.cuda.synchronize()
    ref_i, ref_v = orc.scan_topk(storage, 4, dim, queries, k, row_scales=row_scales)
    np.testing.assert_array_equal(idx.cpu().numpy(), ref_i)
    np.testing.assert_array_equal(val.cpu().numpy(), ref_v)
    assert ws.status() == 0


def test_scan_topk_dispatches_large_int8_batches_exactly(zc, orc):
    """zcgvs_scan_topk on a per-row int8 corpus with >= 64 queries and >= 65536 rows runs on the
    tensor cores; the result must still equal the oracle bit for bit."""
    import torch

    n, dim, batch, k = 100000, 256, 96, 100
    storage, row_scales, queries = case(orc, 4, n, dim, batch, 11)
    idx, val = zc.scan_topk(dev(storage), 4, dim, dev(queries), k, row_scales=dev(row_scales))
    torch.cuda.synchronize()
    ref_i, ref_v = orc.scan_topk(storage, 4, dim, queries, k, row_scales=row_scales)
    np.testing.assert_array_equal(idx.cpu().numpy(), ref_i)
    np.testing.assert_array_equal(val.cpu().numpy(), ref_v)


# ----------------------------------------------------------------------------------------
# 1-bit corpora: sign bits expanded to int8 on chip, exact Hamming scores
# ----------------------------------------------------------------------------------------
BIN = 3


@pytest.mark.parametrize("n,dim,batch", [(1000, 256, 200), (777, 128, 5), (3000, 1024, 130)])
def test_gemm_similarity_binary_exact(zc, orc, n, dim, batch):
    import torch

    storage, _, queries = case(orc, BIN, n, dim, batch, 21)
    mask = np.ones(n, dtype=np.uint8)
    mask[::5] = 0
    out = zc.gemm_similarity(dev(storage), BIN, dim, dev(queries), mask=dev(mask))
    torch.cuda.synchronize()
    ref = orc.scores(storage, BIN, dim, queries, mask=mask)
    np.testing.assert_array_equal(out.cpu().numpy(), ref)


@pytest.mark.parametrize("n,dim,batch,k", [(5000, 1024, 64, 1000), (20000, 384, 130, 10), (3000, 128, 7, 1),
                                           (70000, 768, 20, 100), (4000, 256, 300, 1024)])
def test_gemm_topk_binary_exact(zc, orc, n, dim, batch, k):
    import torch

    storage, _, queries = case(orc, BIN, n, dim, batch, 22)
    ws = zc.Workspace()
    idx, val = zc.gemm_topk(dev(storage), BIN, dim, dev(queries), k, workspace=ws)
    torch.cuda.synchronize()
    ref_i, ref_v = orc.scan_topk(storage, BIN, dim, queries, k)
    np.testing.assert_array_equal(idx.cpu().numpy(), ref_i)
    np.testing.assert_array_equal(val.cpu().numpy(), ref_v)
    assert ws.status() == 0


def test_gemm_topk_binary_mask_id_base_and_l2(zc, orc):
    """Masked documents never appear, ids are offset by id_base, and the L2 metric scores a
    1-bit corpus by Hamming distance like any other metric."""
    import torch

    n, dim, batch, k = 9000, 256, 150, 40
    storage, _, queries = case(orc, BIN, n, dim, batch, 23)
    mask = np.ones(n, dtype=np.uint8)
    mask[1::3] = 0
    for metric in (zc.METRIC_DOT, zc.METRIC_L2):
        idx, val = zc.gemm_topk(dev(storage), BIN, dim, dev(queries), k, mask=dev(mask), id_base=1000,
                                metric=metric)
        torch.cuda.synchronize()
        ref_i, ref_v = orc.scan_topk(storage, BIN, dim, queries, k, mask=mask, id_base=1000)
        np.testing.assert_array_equal(idx.cpu().numpy(), ref_i)
        np.testing.assert_array_equal(val.cpu().numpy(), ref_v)


def test_gemm_topk_binary_all_ties_is_exact(zc, orc):
    """Every row holds the same bits: all documents tie, the candidate buffer overflows and the
    raised bound of the retry must return ids 0 .. k-1 in order."""
    import torch

    n, dim, batch, k = 40000, 128, 3, 50
    rng = np.random.default_rng(5)
    row = rng.standard_normal(dim).astype(np.float32)
    storage = orc.pack_binary(np.tile(row, (n, 1)))
    queries = rng.standard_normal((batch, dim)).astype(np.float32)
    ws = zc.Workspace()
    idx, val = zc.gemm_topk(dev(storage), BIN, dim, dev(queries), k, workspace=ws)
    torch.cuda.synchronize()
    ref_i, ref_v = orc.scan_topk(storage, BIN, dim, queries, k)
    np.testing.assert_array_equal(idx.cpu().numpy(), ref_i)
    np.testing.assert_array_equal(val.cpu().numpy(), ref_v)
    assert ws.status() == 0


def test_scan_topk_dispatches_binary_batches_exactly(zc, orc):
    """zcgvs_scan_topk on a 1-bit corpus with >= 16 queries and >= 65536 rows runs on the tensor
    cores (the BASELINE 1-bit shape: 1024 dimensions, top-1,000); bit-exact against the oracle
    and against the streaming scan of the same queries one at a time."""
    import torch

    n, dim, batch, k = 100000, 1024, 64, 1000
    storage, _, queries = case(orc, BIN, n, dim, batch, 24)
    idx, val = zc.scan_topk(dev(storage), BIN, dim, dev(queries), k)
    torch.cuda.synchronize()
    ref_i, ref_v = orc.scan_topk(storage, BIN, dim, queries, k)
    np.testing.assert_array_equal(idx.cpu().numpy(), ref_i)
    np.testing.assert_array_equal(val.cpu().numpy(), ref_v)
    one_i, one_v = zc.scan_topk(dev(storage), BIN, dim, dev(queries[:8]), k)  # below the batch cut: streaming
    torch.cuda.synchronize()
    np.testing.assert_array_equal(one_i.cpu().numpy(), ref_i[:8])
    np.testing.assert_array_equal(one_v.cpu().numpy(), ref_v[:8])
