"""CPU tier: ZCVE / ZCVL files (formats.py). The writer must produce the reference writer's bytes
for every reference dtype (tests/golden/files.npz holds files the reference's
python/zcgvs_tools/formats.py wrote), the readers must decode them, version 1 files stay
readable, and the version-3 per-row int8 extension round-trips with the same arithmetic as the
oracle's per-row quantiser (which the device converter is tested against on the GPU). Row
strides follow the reference's tests/python/test_formats.py:27-33."""

from __future__ import annotations

import struct

import numpy as np
import pytest

from conftest import ROOT

import formats  # noqa: E402  (the package directory is on sys.path through conftest)

GOLDEN = np.load(ROOT / "tests" / "golden" / "files.npz")


@pytest.mark.parametrize("dtype", ["float32", "float16", "int8", "binary"])
def test_writer_matches_reference_bytes(tmp_path, dtype):
    path = tmp_path / "e.zcve"
    formats.write_embeddings(path, GOLDEN["matrix"], normalized=(dtype != "int8"), dtype=dtype)
    assert path.read_bytes() == GOLDEN[f"zcve_{dtype}"].tobytes()


def test_writer_default_dtype_follows_input_precision(tmp_path):
    path = tmp_path / "e.zcve"
    formats.write_embeddings(path, GOLDEN["matrix"].astype(np.float16), normalized=True)
    assert path.read_bytes() == GOLDEN["zcve_default16"].tobytes()


@pytest.mark.parametrize("dtype", ["float32", "float16", "int8", "binary"])
def test_reader_decodes_reference_files(tmp_path, dtype):
    path = tmp_path / "e.zcve"
    path.write_bytes(GOLDEN[f"zcve_{dtype}"].tobytes())
    h, storage, row_scales = formats.read_encoded_embeddings(path)
    m = GOLDEN["matrix"]
    assert (h["version"], h["doc_count"], h["dim"], h["dtype"]) == (2, 9, 70, dtype)
    assert h["normalized"] == (dtype != "int8") and row_scales is None
    expect, _, scale, _ = formats.encode_matrix(m, dtype)
    np.testing.assert_array_equal(storage, expect)
    assert np.float32(h["scale"]) == np.float32(scale)
    decoded, _ = formats.read_embeddings(path)
    if dtype == "int8":
        assert np.max(np.abs(decoded - m)) <= h["scale"]


def test_row_strides_match_reference():
    # tests/python/test_formats.py:27-33 of the reference
    assert formats.row_stride(formats.DTYPE_BINARY, 384) == 48
    assert formats.row_stride(formats.DTYPE_BINARY, 130) == 20
    assert formats.row_stride(formats.DTYPE_FLOAT16, 384) == 768
    assert formats.row_stride(formats.DTYPE_INT8, 384) == 384
    assert formats.row_stride(formats.DTYPE_INT8_ROW, 384) == 384
    assert formats.row_stride(formats.DTYPE_FLOAT32, 384) == 1536


def test_version1_file_is_readable(tmp_path):
    m = GOLDEN["matrix"]
    path = tmp_path / "v1.zcve"
    path.write_bytes(struct.pack("<4sIIqii", b"ZCVE", 1, 1, 9, 70, 1) + m.astype(np.float16).tobytes())
    h, storage, _ = formats.read_encoded_embeddings(path)
    assert (h["version"], h["scale"], h["row_stride"]) == (1, 1.0, 140)
    np.testing.assert_array_equal(storage, m.astype(np.float16))


def test_int8_row_version3_round_trip_matches_oracle(tmp_path, orc):
    m = np.concatenate([GOLDEN["matrix"], orc.normal_rows(50, 70, 5) * 3.0])
    path = tmp_path / "r.zcve"
    formats.write_embeddings(path, m, normalized=False, dtype="int8_row")
    h, storage, row_scales = formats.read_encoded_embeddings(path)
    assert (h["version"], h["dtype_code"], h["row_stride"]) == (3, formats.DTYPE_INT8_ROW, 70)
    ref_q, ref_s = orc.quantize_rows_i8(m)
    np.testing.assert_array_equal(storage, ref_q)
    np.testing.assert_array_equal(row_scales, ref_s)
    assert row_scales[4] == 1.0  # the all-zero row
    assert path.stat().st_size == 36 + m.shape[0] * (70 + 4)


def test_per_matrix_int8_and_pack_match_oracle(orc):
    m = orc.normal_rows(40, 130, 9)
    q, s = formats.quantize_int8(m)
    assert np.float32(s) == np.float32(orc.matrix_scale(m))
    np.testing.assert_array_equal(q, orc.quantize_i8(m, s))
    np.testing.assert_array_equal(formats.pack_binary(m), orc.pack_binary(m))


def test_lexical_index_round_trip_and_reference_bytes(tmp_path):
    path = tmp_path / "i.zcvl"
    formats.write_lexical_index(path, 9, 5, GOLDEN["lex_offsets"], GOLDEN["lex_docs"], GOLDEN["lex_weights"],
                                0.9, 0.4, 12.5)
    assert path.read_bytes() == GOLDEN["zcvl"].tobytes()
    got = formats.read_lexical_index(path)
    assert (got["doc_count"], got["vocab_size"], got["nnz"]) == (9, 5, 11)
    np.testing.assert_array_equal(got["offsets"], GOLDEN["lex_offsets"])
    np.testing.assert_array_equal(got["posting_docs"], GOLDEN["lex_docs"])
    np.testing.assert_array_equal(got["posting_weights"], GOLDEN["lex_weights"])


@pytest.mark.parametrize("mutate,match", [
    (lambda b: b"ZCVX" + b[4:], "not a zcgvs"),
    (lambda b: b[:4] + struct.pack("<I", 7) + b[8:], "version"),
    (lambda b: b[:24] + struct.pack("<i", 4) + b[28:], "not valid in a version 2"),
    (lambda b: b[:32] + struct.pack("<i", 71) + b[36:], "row stride"),
])
def test_reader_rejects_malformed_headers(tmp_path, mutate, match):
    path = tmp_path / "bad.zcve"
    path.write_bytes(mutate(GOLDEN["zcve_float32"].tobytes()))
    with pytest.raises(ValueError, match=match):
        formats.read_embedding_header(path)


def test_reader_rejects_truncated_payload(tmp_path):
    path = tmp_path / "short.zcve"
    path.write_bytes(GOLDEN["zcve_float32"].tobytes()[:-1])
    with pytest.raises(ValueError, match="ends early"):
        formats.read_encoded_embeddings(path)


def test_writer_rejects_inconsistent_row_scales(tmp_path):
    with pytest.raises(ValueError):
        formats.write_encoded_embeddings(tmp_path / "x.zcve", np.zeros((2, 4), np.int8), formats.DTYPE_INT8_ROW, 4,
                                         False)
    with pytest.raises(ValueError):
        formats.write_encoded_embeddings(tmp_path / "x.zcve", np.zeros((2, 4), np.int8), formats.DTYPE_INT8, 4,
                                         False, row_scales=np.ones(2, np.float32))
