"""GPU: zcgvs_scan_topk_noalloc, the fused search for callers that cannot allocate device
memory (hosts that own all GPU memory and forbid cudaMalloc in plug-ins, or paths where an
allocation's implicit synchronisation is not allowed). It keeps its scratch in a static
device array inside the library instead of a caller workspace.

Checked through the C ABI against the existing entry point, zcgvs_scan_topk, on two calls in a
row (the static scratch keeps the previous call's contents, which must not leak into the next
result): bit-exact for per-row int8, within the float paths' 1e-4 for fp16. Collected last so a
stop-at-first-failure run has already run every other test.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _dev(a):
    import torch

    a = np.ascontiguousarray(a)
    if a.dtype == np.uint16:
        a = a.view(np.int16)
    return torch.from_numpy(a).cuda()


@pytest.mark.parametrize("name", ["i8row", "f16"])
def test_noalloc_matches_workspace_entry_point_twice(zc, orc, name):
    import torch

    n, dim, k = 200_000, 768, 100
    corpus = orc.normal_rows(n, dim, 5151)
    if name == "i8row":
        dtype, (storage, _, row_scales) = zc.DTYPE_I8_ROW, orc.encode(corpus, orc.DTYPE_I8_ROW)
    else:
        dtype, (storage, _, row_scales) = zc.DTYPE_F16, orc.encode(corpus, orc.DTYPE_F16)
    d_store = _dev(storage)
    d_rs = None if row_scales is None else _dev(row_scales)
    for call, (batch, seed) in enumerate(((1, 6161), (3, 7171))):
        q = _dev(orc.normal_rows(batch, dim, seed))
        ref_idx, ref_val = zc.scan_topk(d_store, dtype, dim, q, k, row_scales=d_rs)
        got_idx, got_val = zc.scan_topk_noalloc(d_store, dtype, dim, q, k, row_scales=d_rs)
        torch.cuda.synchronize()
        if name == "i8row":
            assert torch.equal(got_idx, ref_idx), f"call {call}: ids differ"
            assert torch.equal(got_val, ref_val), f"call {call}: scores differ"
        else:
            np.testing.assert_allclose(got_val.cpu().numpy(), ref_val.cpu().numpy(), rtol=0, atol=1e-4)
            same = (got_idx.cpu().numpy() == ref_idx.cpu().numpy()).mean()
            assert same > 0.99, f"call {call}: id agreement {same}"


def test_noalloc_rejects_searches_beyond_its_static_scratch(zc):
    # 8 M rows at batch 1 needs > 32 MiB of scratch (one spill slot per row): rejected before
    # any device work, with a message pointing at the workspace entry point.
    fake = ctypes.c_void_p(256)
    status = zc.lib().zcgvs_scan_topk_noalloc(fake, zc.DTYPE_I8_ROW, 1.0, fake, 8_000_000, 768, fake, 1, None,
                                              zc.METRIC_DOT, 100, 0, fake, fake, None)
    assert status == zc.ERR_INVALID_ARG
    assert "zcgvs_scan_topk with a caller-provided workspace" in zc.lib().zcgvs_last_error_message().decode()
