"""GPU: zcgvs_scan_topk_noalloc, the fused search for callers that cannot allocate device
memory (hosts that own all GPU memory and forbid cudaMalloc in plug-ins, or paths where an
allocation's implicit synchronisation is not allowed). It keeps its scratch in a static
device array inside the library instead of a caller workspace.

Checked through the C ABI against the existing entry point, zcgvs_scan_topk, on two calls in a
row (the static scratch keeps the previous call's contents, which must not leak into the next
result). Both entry points run the same deterministic kernels, so the results must be identical
bit for bit on every path: the streaming scans (per-row int8, fp16) and the tensor-core route
that zcgvs_scan_topk takes for large per-row int8 and 1-bit batches, whose scratch layout and
status header differ. The status word of the static scratch is read back through
zcgvs_scan_topk_noalloc_status, including after a search made to overflow its candidate buffer.
Collected last so a stop-at-first-failure run has already run every other test.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

SCRATCH_BYTES = 32 << 20


def _dev(a):
    import torch

    a = np.ascontiguousarray(a)
    if a.dtype == np.uint16:
        a = a.view(np.int16)
    elif a.dtype == np.uint32:
        a = a.view(np.int32)
    return torch.from_numpy(a).cuda()


def _both_entry_points_agree(zc, d_store, dtype, dim, queries, k, d_rs=None, call=0):
    import torch

    q = _dev(queries)
    ref_idx, ref_val = zc.scan_topk(d_store, dtype, dim, q, k, row_scales=d_rs)
    got_idx, got_val = zc.scan_topk_noalloc(d_store, dtype, dim, q, k, row_scales=d_rs)
    torch.cuda.synchronize()
    assert torch.equal(got_idx, ref_idx), f"call {call}: ids differ"
    assert torch.equal(got_val, ref_val), f"call {call}: scores differ"
    assert zc.noalloc_status() == 0


@pytest.mark.parametrize("name", ["i8row", "f16"])
def test_noalloc_matches_workspace_entry_point_twice(zc, orc, name):
    n, dim, k = 200_000, 768, 100
    corpus = orc.normal_rows(n, dim, 5151)
    if name == "i8row":
        dtype, (storage, _, row_scales) = zc.DTYPE_I8_ROW, orc.encode(corpus, orc.DTYPE_I8_ROW)
    else:
        dtype, (storage, _, row_scales) = zc.DTYPE_F16, orc.encode(corpus, orc.DTYPE_F16)
    d_store = _dev(storage)
    d_rs = None if row_scales is None else _dev(row_scales)
    for call, (batch, seed) in enumerate(((1, 6161), (3, 7171))):
        _both_entry_points_agree(zc, d_store, dtype, dim, orc.normal_rows(batch, dim, seed), k, d_rs, call)


def _tensor_core_shape(zc, dtype, dim, batch, k):
    """The largest row count (>= 65,536, where zcgvs_scan_topk takes the tensor-core route) whose
    search fits the static scratch."""
    for n in (200_000, 131_072, 65_536):
        if zc.scan_topk_workspace_bytes(dtype, n, dim, batch, k) <= SCRATCH_BYTES:
            return n
    pytest.fail(f"no tensor-core shape of dtype {dtype}, batch {batch}, k {k} fits the static scratch")


@pytest.mark.parametrize("name,batch", [("i8row", 64), ("bin", 16)])
def test_noalloc_tensor_core_route_matches_twice(zc, orc, name, batch):
    dim, k = 1024, 10
    dtype = zc.DTYPE_I8_ROW if name == "i8row" else zc.DTYPE_BINARY
    n = _tensor_core_shape(zc, dtype, dim, batch, k)
    corpus = orc.normal_rows(n, dim, 8181)
    storage, _, row_scales = orc.encode(corpus, orc.DTYPE_I8_ROW if name == "i8row" else orc.DTYPE_BINARY)
    d_store = _dev(storage)
    d_rs = None if row_scales is None else _dev(row_scales)
    for call, seed in enumerate((8282, 8383)):
        _both_entry_points_agree(zc, d_store, dtype, dim, orc.normal_rows(batch, dim, seed), k, d_rs, call)


def test_noalloc_status_reports_an_overflowed_search_then_clears(zc, orc):
    """The candidate buffer of the tensor-core route is capped (test hook, host-side) below k, so
    the search ends incomplete and sets the overflow bit in the static scratch's status word; the
    reader returns it and the binding raises. The next call clears the word."""
    import torch

    dim, batch, k = 1024, 16, 10
    n = _tensor_core_shape(zc, zc.DTYPE_BINARY, dim, batch, k)
    corpus = orc.normal_rows(n, dim, 9191)
    d_store = _dev(orc.encode(corpus, orc.DTYPE_BINARY)[0])
    q = _dev(orc.normal_rows(batch, dim, 9292))
    zc.set_test_candidate_cap(5)
    try:
        zc.scan_topk_noalloc(d_store, zc.DTYPE_BINARY, dim, q, k, check_status=False)
        word = zc.noalloc_status()
        assert word & zc.DEVICE_CANDIDATE_OVERFLOW, hex(word)
        with pytest.raises(zc.DeviceStatusError, match="more candidates than its buffer holds"):
            zc.scan_topk_noalloc(d_store, zc.DTYPE_BINARY, dim, q, k)
    finally:
        zc.set_test_candidate_cap(0)
    ids, vals = zc.scan_topk_noalloc(d_store, zc.DTYPE_BINARY, dim, q, k)
    torch.cuda.synchronize()
    assert zc.noalloc_status() == 0
    ref_idx, ref_val = zc.scan_topk(d_store, zc.DTYPE_BINARY, dim, q, k)
    assert torch.equal(ids, ref_idx) and torch.equal(vals, ref_val)


def test_noalloc_rejects_searches_beyond_its_static_scratch(zc):
    # 8 M rows at batch 1 needs > 32 MiB of scratch (one spill slot per row): rejected before
    # any device work, with a message pointing at the workspace entry point.
    fake = ctypes.c_void_p(256)
    status = zc.lib().zcgvs_scan_topk_noalloc(fake, zc.DTYPE_I8_ROW, 1.0, fake, 8_000_000, 768, fake, 1, None,
                                              zc.METRIC_DOT, 100, 0, fake, fake, None)
    assert status == zc.ERR_INVALID_ARG
    assert "zcgvs_scan_topk with a caller-provided workspace" in zc.lib().zcgvs_last_error_message().decode()
