"""ZCVE embedding, ZCVM metadata and ZCVL lexical-index files: writers and readers.

The byte layouts are the reference's (include/zcgvs/data/binary_format.hpp:12-47; its Python
counterpart python/zcgvs_tools/formats.py), all scalars little-endian, so files move between
the reference and this library in both directions:

  ZCVE  magic 'ZCVE', u32 version, u32 flags (bit 0: rows L2-normalised), i64 doc_count,
        i32 dim, i32 dtype; version >= 2: f32 scale, i32 row_stride; then the row-major matrix.
        Version 3 (this library's extension, dtype 4 = int8 with one scale per row) appends the
        [doc_count] f32 row scales after the matrix. Writers emit version 2 for the reference's
        dtypes (0-3) and version 3 only for dtype 4.
  ZCVM  magic 'ZCVM', u32 version 1, i64 doc_count, then per document u32 length + UTF-8 id
        and u32 length + UTF-8 passage text.
  ZCVL  magic 'ZCVL', u32 version 1, i64 doc_count, i32 vocab, i64 nnz, f32 k1, f32 b,
        f32 average_doc_length, i64 offsets[vocab + 1], i32 docs[nnz], f32 weights[nnz].

Encoders (fp32 arithmetic): fp16 round-to-nearest-even; sign bit b of word w = dimension
32 w + b, set when x >= 0; scale = max|x| / 127 (1 when the maximum is 0). Per-matrix int8 rounds
as the reference's writer does, clamp(rint(x / scale), +-127) (formats.py:85-91), so int8 files
are byte-identical to the reference's; per-row int8 rounds as zcgvs_convert_i8_rows and the
reference's CUDA converter do, clamp(rint(x * (1 / scale)), +-127), so a host-written int8_row
file equals a store converted on the device. The C++ loaders are EmbeddingStore::loadFromFile /
LexicalIndex::loadFromFile and Corpus::load (include/zcgvs/data/).
"""

from __future__ import annotations

import struct
from pathlib import Path

import numpy as np

EMBEDDING_MAGIC = b"ZCVE"
LEXICAL_MAGIC = b"ZCVL"
METADATA_MAGIC = b"ZCVM"
METADATA_VERSION = 1
EMBEDDING_VERSION = 2          # what the reference writes and reads
EMBEDDING_VERSION_ROW_SCALES = 3
LEXICAL_VERSION = 1
FLAG_NORMALIZED = 1

DTYPE_FLOAT32, DTYPE_FLOAT16, DTYPE_INT8, DTYPE_BINARY, DTYPE_INT8_ROW = 0, 1, 2, 3, 4
DTYPE_NAMES = {"float32": DTYPE_FLOAT32, "float16": DTYPE_FLOAT16, "int8": DTYPE_INT8, "binary": DTYPE_BINARY,
               "int8_row": DTYPE_INT8_ROW}
DTYPE_CODE_NAMES = {code: name for name, code in DTYPE_NAMES.items()}
_ELEMENT = {DTYPE_FLOAT32: np.float32, DTYPE_FLOAT16: np.float16, DTYPE_INT8: np.int8, DTYPE_BINARY: np.uint32,
            DTYPE_INT8_ROW: np.int8}

_HEAD = struct.Struct("<4sIIqii")          # magic, version, flags, doc_count, dim, dtype
_HEAD_V2 = struct.Struct("<fi")            # scale, row_stride
_LEX_HEAD = struct.Struct("<4sIqiqfff")    # magic, version, doc_count, vocab, nnz, k1, b, avgdl


def binary_words(dim: int) -> int:
    return (dim + 31) // 32


def row_stride(dtype_code: int, dim: int) -> int:
    """Bytes of one stored row."""
    if dtype_code not in _ELEMENT:
        raise ValueError(f"unknown dtype code {dtype_code}")
    if dtype_code == DTYPE_BINARY:
        return 4 * binary_words(dim)
    return dim * np.dtype(_ELEMENT[dtype_code]).itemsize


# ------------------------------------------------------------------------------------------
# Encoders (host, fp32 arithmetic)
# ------------------------------------------------------------------------------------------
def _scale_of(peak: np.ndarray) -> np.ndarray:
    peak = np.asarray(peak, dtype=np.float32)
    return np.where(peak > 0, peak / np.float32(127.0), np.float32(1.0)).astype(np.float32)


def quantize_int8(matrix: np.ndarray) -> tuple[np.ndarray, float]:
    """One scale for the matrix: (codes, scale), codes = clamp(rint(x / scale), +-127)."""
    x = np.ascontiguousarray(matrix, dtype=np.float32)
    scale = _scale_of(np.abs(x).max() if x.size else 0.0)
    return np.clip(np.rint(x / scale), -127, 127).astype(np.int8), float(scale)


def quantize_int8_rows(matrix: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """One scale per row: (codes [N, d], scales [N] fp32), codes = clamp(rint(x * (1 / scale)), +-127)."""
    x = np.ascontiguousarray(matrix, dtype=np.float32)
    scales = _scale_of(np.abs(x).max(axis=1) if x.shape[1] else np.zeros(x.shape[0], np.float32))
    inverse = (np.float32(1.0) / scales).astype(np.float32)
    return np.clip(np.rint(x * inverse[:, None]), -127, 127).astype(np.int8), scales


def pack_binary(matrix: np.ndarray) -> np.ndarray:
    """Sign bits: [N, d] -> [N, ceil(d / 32)] uint32, bit b of word w = dimension 32 w + b."""
    x = np.ascontiguousarray(matrix, dtype=np.float32)
    rows, dim = x.shape
    words = binary_words(dim)
    bits = np.zeros((rows, words * 32), dtype=np.uint8)
    bits[:, :dim] = x >= 0
    # little-endian bit order within bytes, then bytes into little-endian words
    return np.packbits(bits, axis=1, bitorder="little").view("<u4").reshape(rows, words)


def encode_matrix(matrix: np.ndarray, dtype: str):
    """fp32 rows -> (storage array, dtype code, scale, row scales or None)."""
    if dtype not in DTYPE_NAMES:
        raise ValueError(f"unknown storage dtype '{dtype}'")
    code = DTYPE_NAMES[dtype]
    x = np.ascontiguousarray(matrix, dtype=np.float32)
    if code == DTYPE_FLOAT32:
        return x, code, 1.0, None
    if code == DTYPE_FLOAT16:
        return x.astype(np.float16), code, 1.0, None
    if code == DTYPE_INT8:
        q, s = quantize_int8(x)
        return q, code, s, None
    if code == DTYPE_INT8_ROW:
        q, s = quantize_int8_rows(x)
        return q, code, 1.0, s
    return pack_binary(x), code, 1.0, None


# ------------------------------------------------------------------------------------------
# ZCVE
# ------------------------------------------------------------------------------------------
def write_embeddings(path: str | Path, matrix: np.ndarray, normalized: bool, dtype: str | None = None) -> None:
    """Encodes a float [doc_count, dim] matrix as `dtype` (default: float16 for a float16 input,
    else float32) and writes it: version 2, or version 3 for int8_row."""
    src = np.asarray(matrix)
    if src.ndim != 2:
        raise ValueError("embedding matrix must be 2-D [doc_count, dim]")
    if dtype is None:
        dtype = "float16" if src.dtype == np.float16 else "float32"
    storage, code, scale, row_scales = encode_matrix(src, dtype)
    write_encoded_embeddings(path, storage, code, src.shape[1], normalized, scale, row_scales)


def write_encoded_embeddings(path: str | Path, storage: np.ndarray, dtype_code: int, dim: int, normalized: bool,
                             scale: float = 1.0, row_scales: np.ndarray | None = None) -> None:
    """Writes an already-encoded matrix (e.g. the output of the device converters)."""
    storage = np.ascontiguousarray(storage)
    doc_count = storage.shape[0]
    stride = row_stride(dtype_code, dim)
    if storage.nbytes != doc_count * stride:
        raise ValueError("storage bytes do not match doc_count x row stride")
    per_row = dtype_code == DTYPE_INT8_ROW
    if per_row != (row_scales is not None):
        raise ValueError("row scales are required for int8_row and only for it")
    version = EMBEDDING_VERSION_ROW_SCALES if per_row else EMBEDDING_VERSION
    with open(path, "wb") as f:
        f.write(_HEAD.pack(EMBEDDING_MAGIC, version, FLAG_NORMALIZED if normalized else 0, doc_count, dim, dtype_code))
        f.write(_HEAD_V2.pack(float(scale), stride))
        f.write(storage.tobytes())
        if per_row:
            scales = np.ascontiguousarray(row_scales, dtype="<f4")
            if scales.shape != (doc_count,):
                raise ValueError("row scales must hold one value per row")
            f.write(scales.tobytes())


def read_embedding_header(path: str | Path) -> dict:
    with open(path, "rb") as f:
        raw = f.read(_HEAD.size + _HEAD_V2.size)
    if len(raw) < _HEAD.size:
        raise ValueError("embedding file ends inside its header")
    magic, version, flags, doc_count, dim, code = _HEAD.unpack_from(raw)
    if magic != EMBEDDING_MAGIC:
        raise ValueError("not a zcgvs embedding file")
    if version not in (1, 2, 3):
        raise ValueError(f"unsupported embedding file version {version}")
    if code not in _ELEMENT or (code == DTYPE_INT8_ROW and version < 3) or (version == 1 and code > DTYPE_FLOAT16):
        raise ValueError(f"dtype {code} is not valid in a version {version} file")
    if version == 1:
        scale, stride, offset = 1.0, row_stride(code, dim), _HEAD.size
    else:
        scale, stride = _HEAD_V2.unpack_from(raw, _HEAD.size)
        offset = _HEAD.size + _HEAD_V2.size
        if stride != row_stride(code, dim):
            raise ValueError("embedding row stride does not match dtype and dim")
    return {"version": version, "normalized": bool(flags & FLAG_NORMALIZED), "doc_count": doc_count, "dim": dim,
            "dtype": DTYPE_CODE_NAMES[code], "dtype_code": code, "scale": scale, "row_stride": stride,
            "bytes": doc_count * stride, "offset": offset}


def read_encoded_embeddings(path: str | Path):
    """(header, storage array in its stored element type, row scales or None), no decoding."""
    h = read_embedding_header(path)
    element = np.dtype(_ELEMENT[h["dtype_code"]]).newbyteorder("<")
    columns = h["row_stride"] // element.itemsize
    with open(path, "rb") as f:
        f.seek(h["offset"])
        data = f.read(h["bytes"])
        scales = f.read(4 * h["doc_count"]) if h["dtype_code"] == DTYPE_INT8_ROW else None
    if len(data) != h["bytes"] or (scales is not None and len(scales) != 4 * h["doc_count"]):
        raise ValueError("embedding file ends early")
    storage = np.frombuffer(data, dtype=element).reshape(h["doc_count"], columns)
    row_scales = None if scales is None else np.frombuffer(scales, dtype="<f4")
    return h, storage, row_scales


def read_embeddings(path: str | Path) -> tuple[np.ndarray, bool]:
    """(matrix, normalized) as the reference reader returns it: fp32 / fp16 as stored, int8
    dequantised to fp32 (per row for int8_row), binary as its packed uint32 words."""
    h, storage, row_scales = read_encoded_embeddings(path)
    if h["dtype_code"] == DTYPE_INT8:
        return storage.astype(np.float32) * np.float32(h["scale"]), h["normalized"]
    if h["dtype_code"] == DTYPE_INT8_ROW:
        return storage.astype(np.float32) * row_scales[:, None], h["normalized"]
    return storage, h["normalized"]


# ------------------------------------------------------------------------------------------
# ZCVL
# ------------------------------------------------------------------------------------------
def write_lexical_index(path: str | Path, doc_count: int, vocab_size: int, offsets: np.ndarray,
                        posting_docs: np.ndarray, posting_weights: np.ndarray, k1: float, b: float,
                        average_doc_length: float) -> None:
    offsets = np.ascontiguousarray(offsets, dtype="<i8")
    docs = np.ascontiguousarray(posting_docs, dtype="<i4")
    weights = np.ascontiguousarray(posting_weights, dtype="<f4")
    if offsets.shape != (vocab_size + 1,):
        raise ValueError("offsets must hold vocab_size + 1 entries")
    if docs.shape != weights.shape:
        raise ValueError("posting arrays must have equal length")
    nnz = docs.shape[0]
    if offsets[0] != 0 or offsets[-1] != nnz:
        raise ValueError("CSR offsets are inconsistent with the posting count")
    with open(path, "wb") as f:
        f.write(_LEX_HEAD.pack(LEXICAL_MAGIC, LEXICAL_VERSION, int(doc_count), int(vocab_size), nnz, float(k1),
                               float(b), float(average_doc_length)))
        for part in (offsets, docs, weights):
            f.write(part.tobytes())


def read_lexical_index(path: str | Path) -> dict:
    with open(path, "rb") as f:
        raw = f.read(_LEX_HEAD.size)
        if len(raw) < _LEX_HEAD.size:
            raise ValueError("lexical index ends inside its header")
        magic, version, doc_count, vocab, nnz, k1, b, avgdl = _LEX_HEAD.unpack(raw)
        if magic != LEXICAL_MAGIC:
            raise ValueError("not a zcgvs lexical index")
        if version != LEXICAL_VERSION:
            raise ValueError(f"unsupported lexical index version {version}")
        parts = []
        for count, dtype in ((vocab + 1, "<i8"), (nnz, "<i4"), (nnz, "<f4")):
            data = f.read(count * 4 if dtype != "<i8" else count * 8)
            if len(data) != count * np.dtype(dtype).itemsize:
                raise ValueError("lexical index ends early")
            parts.append(np.frombuffer(data, dtype=dtype))
    return {"doc_count": doc_count, "vocab_size": vocab, "nnz": nnz, "k1": k1, "b": b, "average_doc_length": avgdl,
            "offsets": parts[0], "posting_docs": parts[1], "posting_weights": parts[2]}


_META_HEAD = struct.Struct("<4sIq")        # magic, version, doc_count
_U32 = struct.Struct("<I")


def write_metadata(path: str | Path, doc_ids: list[str], texts: list[str]) -> None:
    """The corpus metadata file: one (id, passage text) pair per document, in corpus order."""
    if len(doc_ids) != len(texts):
        raise ValueError(f"{len(doc_ids)} document ids but {len(texts)} texts")
    parts = [_META_HEAD.pack(METADATA_MAGIC, METADATA_VERSION, len(doc_ids))]
    for doc_id, text in zip(doc_ids, texts):
        for field in (doc_id.encode("utf-8"), text.encode("utf-8")):
            parts.append(_U32.pack(len(field)))
            parts.append(field)
    Path(path).write_bytes(b"".join(parts))


def read_metadata(path: str | Path) -> tuple[list[str], list[str]]:
    raw = Path(path).read_bytes()
    if len(raw) < _META_HEAD.size:
        raise ValueError(f"{path}: shorter than a metadata header")
    magic, version, count = _META_HEAD.unpack_from(raw, 0)
    if magic != METADATA_MAGIC:
        raise ValueError(f"{path}: not a metadata file (magic {magic!r})")
    if version != METADATA_VERSION:
        raise ValueError(f"{path}: unsupported metadata version {version}")
    at = _META_HEAD.size
    ids: list[str] = []
    texts: list[str] = []
    for _ in range(count):
        fields = []
        for _ in range(2):
            if at + 4 > len(raw):
                raise ValueError(f"{path}: ends inside document {len(ids)}")
            (length,) = _U32.unpack_from(raw, at)
            at += 4
            if at + length > len(raw):
                raise ValueError(f"{path}: ends inside document {len(ids)}")
            fields.append(raw[at:at + length].decode("utf-8"))
            at += length
        ids.append(fields[0])
        texts.append(fields[1])
    return ids, texts
