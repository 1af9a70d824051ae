"""GPU tier: the store converters (fp32 rows on the device -> fp16 / per-matrix int8 / per-row
int8 / sign bits), bit-exact against the oracle's restatement of the reference quantisers
(src/cuda/convert.cu:17-53, python/zcgvs_tools/formats.py:65-91, the per-row extension used by
DTYPE_I8_ROW). Shapes cover odd dims (scalar path), dims that are multiples of 4 (vector path),
all-zero rows (scale 1), ties at .5 (round half to even) and values that clamp."""

from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _dev(a):
    import torch

    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _rows(rows, dim, seed):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((rows, dim), dtype=np.float32) * rng.uniform(0.01, 10.0, (rows, 1)).astype(np.float32)
    if rows > 3:
        x[1] = 0.0                                   # all-zero row: scale 1, codes 0
        x[2, : min(dim, 4)] = [127.0, -63.5, 0.5, -0.5][: min(dim, 4)]  # halves round to even
    return x


@pytest.mark.parametrize("rows,dim", [(1, 1), (7, 33), (1000, 384), (513, 768), (64, 1027), (4096, 128)])
def test_convert_i8_rows_matches_oracle(zc, orc, rows, dim):
    x = _rows(rows, dim, 7 + dim)
    codes, scales = zc.convert_i8_rows(_dev(x))
    ref_codes, ref_scales = orc.quantize_rows_i8(x)
    np.testing.assert_array_equal(scales.cpu().numpy(), ref_scales)
    np.testing.assert_array_equal(codes.cpu().numpy(), ref_codes)


def test_convert_i8_rows_unaligned_source_takes_scalar_path(zc, orc):
    """A source that is not 16-byte aligned (a view one float in) must still be exact."""
    import torch

    x = _rows(65, 256, 3)
    flat = torch.zeros(65 * 256 + 1, dtype=torch.float32, device="cuda")
    flat[1:] = _dev(x).reshape(-1)
    codes, scales = zc.convert_i8_rows(flat[1:].view(65, 256))
    ref_codes, ref_scales = orc.quantize_rows_i8(x)
    np.testing.assert_array_equal(scales.cpu().numpy(), ref_scales)
    np.testing.assert_array_equal(codes.cpu().numpy(), ref_codes)


def test_convert_i8_rows_store_searches_like_the_oracle(zc, orc):
    """The converter's output is a DTYPE_I8_ROW store: searching it equals the oracle search."""
    x = orc.normal_rows(20000, 256, 17)
    q = orc.normal_rows(3, 256, 18)
    codes, scales = zc.convert_i8_rows(_dev(x))
    ids, vals = zc.scan_topk(codes, zc.DTYPE_I8_ROW, 256, _dev(q), 50, row_scales=scales)
    ref_codes, ref_scales = orc.quantize_rows_i8(x)
    ref_i, ref_s = orc.scan_topk(ref_codes, orc.DTYPE_I8_ROW, 256, q, 50, row_scales=ref_scales)
    np.testing.assert_array_equal(ids.cpu().numpy(), ref_i)
    np.testing.assert_array_equal(vals.cpu().numpy(), ref_s)


@pytest.mark.parametrize("count", [1, 1000, 333333])
def test_convert_f16_and_i8_match_oracle(zc, orc, count):
    x = _rows(1, count, count)[0]
    np.testing.assert_array_equal(zc.convert_f16(_dev(x)).cpu().numpy().view(np.uint16), orc.to_f16_bits(x))
    s = orc.matrix_scale(x)
    np.testing.assert_array_equal(zc.convert_i8(_dev(x), s).cpu().numpy(), orc.quantize_i8(x, s))


@pytest.mark.parametrize("rows,dim", [(1, 1), (5, 33), (1000, 1024), (77, 130)])
def test_pack_binary_matches_oracle(zc, orc, rows, dim):
    x = _rows(rows, dim, 11 + dim)
    x[0, 0] = -0.0                                   # -0.0 >= 0: bit set
    got = zc.pack_binary(_dev(x)).cpu().numpy().view(np.uint32)
    np.testing.assert_array_equal(got, orc.pack_binary(x))


def test_converters_reject_null_and_accept_empty(zc):
    import torch

    with pytest.raises(zc.InvalidArgument):
        zc.check(zc.lib().zcgvs_convert_i8_rows(None, None, None, 4, 4, None))
    empty = torch.empty((0, 8), dtype=torch.float32, device="cuda")
    codes, scales = zc.convert_i8_rows(empty)
    assert codes.shape == (0, 8) and scales.shape == (0,)
