"""GPU tier: failure reporting without a GPU fault.

Every wait in the library's kernels is bounded; when one runs out, the kernel sets a bit in the
workspace's device status word and returns. These tests drive the two ways a search can end
incomplete and check that the caller sees it:

* a bounded wait that runs out: zcgvs_check_bounded_wait waits, through the kernels' own wait
  helper, on a barrier nothing completes (nothing is in flight); after the 2 s budget the
  timeout bit is set and the context stays usable;
* a candidate buffer that overflows: the test hook caps the tensor-core path's per-query buffer
  below k (host-side), so the search ends incomplete with the overflow bit set. The Python
  helpers that own their workspace raise DeviceStatusError; a caller-owned workspace keeps the
  word for the caller to read (the C++ Searcher's exception is tested in test_store_cpp_gpu.py).
"""

from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _dev(a):
    import torch

    a = np.ascontiguousarray(a)
    if a.dtype == np.uint32:
        a = a.view(np.int32)
    return torch.from_numpy(a).cuda()


def test_bounded_wait_runs_out_sets_status_and_context_survives(zc, orc):
    import torch

    ws = zc.Workspace()
    ws.get(256)
    zc.check_bounded_wait(ws)
    assert ws.status() == zc.DEVICE_TILE_WAIT_TIMEOUT
    with pytest.raises(zc.DeviceStatusError, match="corpus tile ran out"):
        ws.raise_on_status()
    assert ws.status() == 0
    # The context is still usable: a search on the same workspace is exact.
    corpus = orc.normal_rows(5000, 64, 1)
    q = orc.normal_rows(2, 64, 2)
    storage, _, rs = orc.encode(corpus, orc.DTYPE_I8_ROW)
    idx, val = zc.scan_topk(_dev(storage), zc.DTYPE_I8_ROW, 64, _dev(q), 10, row_scales=_dev(rs), workspace=ws)
    torch.cuda.synchronize()
    ridx, rval = orc.scan_topk(storage, orc.DTYPE_I8_ROW, 64, q, 10, row_scales=rs)
    np.testing.assert_array_equal(idx.cpu().numpy(), ridx)
    np.testing.assert_array_equal(val.cpu().numpy(), rval)
    assert ws.status() == 0


@pytest.mark.parametrize("name", ["i8row", "bin"])
def test_overflow_reaches_the_caller(zc, orc, name):
    import torch

    n, dim, batch, k = 70_000, 256, 64, 10
    dtype = zc.DTYPE_I8_ROW if name == "i8row" else zc.DTYPE_BINARY
    storage, _, rs = orc.encode(orc.normal_rows(n, dim, 31), orc.DTYPE_I8_ROW if name == "i8row" else orc.DTYPE_BINARY)
    d_store, d_rs = _dev(storage), (None if rs is None else _dev(rs))
    q = _dev(orc.normal_rows(batch, dim, 32))
    zc.set_test_candidate_cap(5)
    try:
        # Helper-owned workspace: the helper reads the word and raises.
        with pytest.raises(zc.DeviceStatusError, match="more candidates than its buffer holds"):
            zc.gemm_topk(d_store, dtype, dim, q, k, row_scales=d_rs)
        with pytest.raises(zc.DeviceStatusError):
            zc.scan_topk(d_store, dtype, dim, q, k, row_scales=d_rs)
        # Caller-owned workspace: the word stays for the caller.
        ws = zc.Workspace()
        zc.scan_topk(d_store, dtype, dim, q, k, row_scales=d_rs, workspace=ws)
        assert ws.status() & zc.DEVICE_CANDIDATE_OVERFLOW
        ws.clear_status()
    finally:
        zc.set_test_candidate_cap(0)
    idx, val = zc.scan_topk(d_store, dtype, dim, q, k, row_scales=d_rs, workspace=ws)
    torch.cuda.synchronize()
    assert ws.status() == 0
    ridx, rval = orc.scan_topk(storage, orc.DTYPE_I8_ROW if name == "i8row" else orc.DTYPE_BINARY, dim,
                               q.cpu().numpy(), k, row_scales=rs)
    np.testing.assert_array_equal(idx.cpu().numpy(), ridx)
    np.testing.assert_array_equal(val.cpu().numpy(), rval)
