"""Python access to the CPU oracle. TEST INFRASTRUCTURE ONLY.

Wraps ``oracle/liboracle.so`` (the C restatement in ``oracle.c`` plus the seeded generators in
``gen.cpp``) and, when built, ``oracle/_ref/libzcgvs_refcpu.so`` (the reference's own CPU code,
``tests/cpp/cpu_reference.hpp``). Only tests/, ``__graft_entry__.smoke()`` and bench.py's
cpu_baseline leg import this module, and only as the checker / CPU baseline.
"""

from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "liboracle.so"
REF_CPU_PATH = HERE / "_ref" / "libzcgvs_refcpu.so"

DTYPE_F32, DTYPE_F16, DTYPE_I8, DTYPE_BINARY, DTYPE_I8_ROW = 0, 1, 2, 3, 4
METRIC_COSINE, METRIC_DOT, METRIC_L2 = 0, 1, 2

_P = ctypes.c_void_p
_lib = None
_ref = None


def reference_root() -> Path | None:
    """The reference checkout: $ZCGVS_REFERENCE, else a `reference` directory beside this
    repository; None when neither holds the reference's tests/cpp (e.g. on a GPU box, which
    uses the prebuilt oracle/_ref)."""
    env = os.environ.get("ZCGVS_REFERENCE")
    candidates = [Path(env)] if env else [HERE.parents[1] / "reference"]
    for path in candidates:
        if (path / "tests" / "cpp").is_dir():
            return path.resolve()
    return None


def build() -> None:
    """Compiles liboracle.so and, when the reference checkout is found (reference_root), the
    reference CPU library and (once the CUDA library is built) the reference's C++ programs
    linked against it."""
    subprocess.run(["make", "-s", "-C", str(HERE), "liboracle.so"], check=True)
    ref = reference_root()
    if ref is not None:
        subprocess.run(["make", "-s", "-C", str(HERE), "ref", f"REF={ref}"], check=True)
        if (HERE.parent / "zero-copy-gpu-vector-search-re-ranking-engine_b200" / "libzcgvs_sm100.so").exists():
            subprocess.run(["make", "-s", "-j8", "-C", str(HERE), "reftests", f"REF={ref}"], check=True)


def lib():
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            build()
        _lib = ctypes.CDLL(str(LIB_PATH))
        i64, i32, f32, u32 = ctypes.c_int64, ctypes.c_int, ctypes.c_float, ctypes.c_uint32
        _lib.orc_set_threads.argtypes = [i32]
        _lib.orc_f32_to_f16.restype = ctypes.c_uint16
        _lib.orc_f32_to_f16.argtypes = [f32]
        _lib.orc_convert_f16.argtypes = [_P, ctypes.c_size_t, _P]
        _lib.orc_matrix_scale.restype = f32
        _lib.orc_matrix_scale.argtypes = [_P, ctypes.c_size_t]
        _lib.orc_quantize_i8.argtypes = [_P, ctypes.c_size_t, f32, _P]
        _lib.orc_quantize_rows_i8.argtypes = [_P, i64, i32, _P, _P]
        _lib.orc_pack_binary.argtypes = [_P, i64, i32, _P]
        _lib.orc_hamming.restype = i32
        _lib.orc_hamming.argtypes = [_P, _P, i32]
        _lib.orc_scores.argtypes = [i32, _P, f32, _P, i64, i32, _P, i32, _P, i32, _P]
        _lib.orc_topk.argtypes = [_P, i64, i32, i32, i32, _P, _P]
        _lib.orc_scan_topk.argtypes = [i32, _P, f32, _P, i64, i32, _P, i32, _P, i32, i32, i32, _P, _P]
        _lib.orc_rescore_topk.restype = i32
        _lib.orc_rescore_topk.argtypes = [i32, _P, f32, _P, i64, i32, _P, i32, _P, i32, i32, i32, _P, _P]
        _lib.orc_bm25.argtypes = [_P, _P, _P, i32, _P, i32, i64, _P]
        _lib.orc_max_positive.restype = f32
        _lib.orc_max_positive.argtypes = [_P, i64]
        _lib.orc_fuse.argtypes = [_P, _P, f32, f32, i64]
        _lib.orc_hybrid_topk.argtypes = [i32, _P, f32, _P, i64, i32, _P, i32, _P, i32, _P, _P, _P, i32, _P, i32,
                                         f32, i32, _P, _P]
        _lib.orc_gen_lexical_test.argtypes = [u32, i32, i32, i32, f32, f32, u32, i32, _P, _P, _P, _P, _P, _P]
        _lib.orc_gen_normal_rows.argtypes = [i64, i32, u32, i32, _P]
        _lib.orc_gen_uniform.argtypes = [ctypes.c_size_t, u32, f32, f32, _P]
    return _lib


def ref_lib():
    """The reference's own CPU code, or None when oracle/_ref was not built."""
    global _ref
    if _ref is None and REF_CPU_PATH.exists():
        _ref = ctypes.CDLL(str(REF_CPU_PATH))
        i32 = ctypes.c_int
        _ref.refcpu_scores.argtypes = [_P, i32, i32, _P, i32, _P]
        _ref.refcpu_topk.argtypes = [_P, i32, i32, i32, _P]
        _ref.refcpu_quantize_dequantize_i8.argtypes = [_P, ctypes.c_size_t, ctypes.c_float, _P]
        _ref.refcpu_pack_binary.argtypes = [_P, i32, i32, _P]
        _ref.refcpu_hamming.restype = i32
        _ref.refcpu_hamming.argtypes = [_P, _P, i32]
        _ref.refcpu_l2_normalize.argtypes = [_P, i32]
        _ref.refcpu_search.restype = ctypes.c_double
        _ref.refcpu_search.argtypes = [_P, i32, i32, _P, i32, i32, i32, _P]
    return _ref


def set_threads(threads: int) -> None:
    """Host threads for the oracle's row loops (1 = sequential, the default). Rows are scored
    independently, so the results do not depend on it."""
    lib().orc_set_threads(int(threads))


def _ptr(a: np.ndarray | None):
    return None if a is None else a.ctypes.data_as(_P)


# ----------------------------------------------------------------------------------------
# Generators (bit-identical to the reference harnesses' std::mt19937 inputs)
# ----------------------------------------------------------------------------------------
def normal_rows(rows: int, dim: int, seed: int, normalize: bool = True) -> np.ndarray:
    out = np.empty((rows, dim), dtype=np.float32)
    lib().orc_gen_normal_rows(rows, dim, seed, 1 if normalize else 0, _ptr(out))
    return out


def uniform(count: int, seed: int, lo: float, hi: float) -> np.ndarray:
    out = np.empty(count, dtype=np.float32)
    lib().orc_gen_uniform(count, seed, lo, hi, _ptr(out))
    return out


# ----------------------------------------------------------------------------------------
# Storage conversions
# ----------------------------------------------------------------------------------------
def to_f16_bits(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.shape, dtype=np.uint16)
    lib().orc_convert_f16(_ptr(x), x.size, _ptr(out))
    return out


def matrix_scale(x: np.ndarray) -> float:
    x = np.ascontiguousarray(x, dtype=np.float32)
    return float(lib().orc_matrix_scale(_ptr(x), x.size))


def quantize_i8(x: np.ndarray, scale: float) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.shape, dtype=np.int8)
    lib().orc_quantize_i8(_ptr(x), x.size, scale, _ptr(out))
    return out


def quantize_rows_i8(x: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    x = np.ascontiguousarray(x, dtype=np.float32)
    rows, dim = x.shape
    q = np.empty((rows, dim), dtype=np.int8)
    s = np.empty(rows, dtype=np.float32)
    lib().orc_quantize_rows_i8(_ptr(x), rows, dim, _ptr(q), _ptr(s))
    return q, s


def pack_binary(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    rows, dim = x.shape
    out = np.empty((rows, (dim + 31) // 32), dtype=np.uint32)
    lib().orc_pack_binary(_ptr(x), rows, dim, _ptr(out))
    return out


def encode(x: np.ndarray, dtype: int, scale: float | None = None):
    """Stores a float32 matrix in `dtype` form. Returns (storage, scale, row_scales)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    if dtype == DTYPE_F32:
        return x, 1.0, None
    if dtype == DTYPE_F16:
        return to_f16_bits(x), 1.0, None
    if dtype == DTYPE_I8:
        s = matrix_scale(x) if scale is None else scale
        return quantize_i8(x, s), s, None
    if dtype == DTYPE_I8_ROW:
        q, s = quantize_rows_i8(x)
        return q, 1.0, s
    if dtype == DTYPE_BINARY:
        return pack_binary(x), 1.0, None
    raise ValueError(f"unknown dtype {dtype}")


# ----------------------------------------------------------------------------------------
# Scoring and selection
# ----------------------------------------------------------------------------------------
def scores(storage, dtype, dim, queries, scale=1.0, row_scales=None, mask=None, metric=METRIC_DOT):
    storage = np.ascontiguousarray(storage)
    queries = np.ascontiguousarray(queries, dtype=np.float32).reshape(-1, dim)
    n = storage.shape[0]
    out = np.empty((queries.shape[0], n), dtype=np.float32)
    rs = None if row_scales is None else np.ascontiguousarray(row_scales, dtype=np.float32)
    m = None if mask is None else np.ascontiguousarray(mask, dtype=np.uint8)
    lib().orc_scores(dtype, _ptr(storage), scale, _ptr(rs), n, dim, _ptr(queries),
                     queries.shape[0], _ptr(m), metric, _ptr(out))
    return out


def topk(score_matrix: np.ndarray, k: int, id_base: int = 0):
    s = np.ascontiguousarray(score_matrix, dtype=np.float32)
    if s.ndim == 1:
        s = s[None, :]
    batch, n = s.shape
    idx = np.empty((batch, k), dtype=np.int32)
    val = np.empty((batch, k), dtype=np.float32)
    lib().orc_topk(_ptr(s), n, batch, k, id_base, _ptr(idx), _ptr(val))
    return idx, val


def scan_topk(storage, dtype, dim, queries, k, scale=1.0, row_scales=None, mask=None,
              metric=METRIC_DOT, id_base=0):
    storage = np.ascontiguousarray(storage)
    queries = np.ascontiguousarray(queries, dtype=np.float32).reshape(-1, dim)
    batch = queries.shape[0]
    idx = np.empty((batch, k), dtype=np.int32)
    val = np.empty((batch, k), dtype=np.float32)
    rs = None if row_scales is None else np.ascontiguousarray(row_scales, dtype=np.float32)
    m = None if mask is None else np.ascontiguousarray(mask, dtype=np.uint8)
    lib().orc_scan_topk(dtype, _ptr(storage), scale, _ptr(rs), storage.shape[0], dim,
                        _ptr(queries), batch, _ptr(m), metric, k, id_base, _ptr(idx), _ptr(val))
    return idx, val


def rescore_topk(storage, dtype, dim, queries, candidates, k, scale=1.0, row_scales=None,
                 metric=METRIC_DOT):
    """Gather-rescore + second top-k + id remap over candidate ids [batch, m]."""
    storage = np.ascontiguousarray(storage)
    queries = np.ascontiguousarray(queries, dtype=np.float32).reshape(-1, dim)
    batch = queries.shape[0]
    cand = np.ascontiguousarray(candidates, dtype=np.int32).reshape(batch, -1)
    idx = np.empty((batch, k), dtype=np.int32)
    val = np.empty((batch, k), dtype=np.float32)
    rs = None if row_scales is None else np.ascontiguousarray(row_scales, dtype=np.float32)
    rc = lib().orc_rescore_topk(dtype, _ptr(storage), scale, _ptr(rs), storage.shape[0], dim,
                                _ptr(queries), batch, _ptr(cand), cand.shape[1], metric, k,
                                _ptr(idx), _ptr(val))
    if rc != 0:
        raise ValueError("rescore store must hold float32, float16 or int8 rows")
    return idx, val


# ----------------------------------------------------------------------------------------
# Lexical scoring
# ----------------------------------------------------------------------------------------
def lexical_test_case(index_seed=41, doc_count=20000, vocab=3000, max_postings=400, wlo=0.01, whi=8.0,
                      query_seed=42, term_count=24):
    """The index, query terms and dense scores of tests/cpp/test_lexical.cu:31-67."""
    nnz = ctypes.c_int64(0)
    lib().orc_gen_lexical_test(index_seed, doc_count, vocab, max_postings, wlo, whi, query_seed, term_count,
                               None, None, None, ctypes.byref(nnz), None, None)
    offsets = np.empty(vocab + 1, dtype=np.int64)
    docs = np.empty(nnz.value, dtype=np.int32)
    weights = np.empty(nnz.value, dtype=np.float32)
    terms = np.empty(term_count, dtype=np.int32)
    dense = np.empty(doc_count, dtype=np.float32)
    lib().orc_gen_lexical_test(index_seed, doc_count, vocab, max_postings, wlo, whi, query_seed, term_count,
                               _ptr(offsets), _ptr(docs), _ptr(weights), ctypes.byref(nnz), _ptr(terms),
                               _ptr(dense))
    return offsets, docs, weights, terms, dense


def bm25(offsets, docs, weights, vocab, terms, n, init=None):
    out = np.zeros(n, dtype=np.float32) if init is None else np.array(init, dtype=np.float32)
    terms = np.ascontiguousarray(terms, dtype=np.int32)
    lib().orc_bm25(_ptr(np.ascontiguousarray(offsets, dtype=np.int64)), _ptr(np.ascontiguousarray(docs, dtype=np.int32)),
                   _ptr(np.ascontiguousarray(weights, dtype=np.float32)), vocab, _ptr(terms), terms.size, n, _ptr(out))
    return out


def max_positive(values) -> float:
    v = np.ascontiguousarray(values, dtype=np.float32)
    return float(lib().orc_max_positive(_ptr(v), v.size))


def fuse(dense, lex, peak, w):
    out = np.array(dense, dtype=np.float32)
    lex = np.ascontiguousarray(lex, dtype=np.float32)
    lib().orc_fuse(_ptr(out), _ptr(lex), peak, w, out.size)
    return out


def hybrid_topk(storage, dtype, dim, queries, k, offsets, docs, weights, vocab, terms, dense_weight, scale=1.0,
                row_scales=None, mask=None, metric=METRIC_DOT):
    storage = np.ascontiguousarray(storage)
    queries = np.ascontiguousarray(queries, dtype=np.float32).reshape(-1, dim)
    batch = queries.shape[0]
    terms = np.ascontiguousarray(terms, dtype=np.int32).reshape(batch, -1)
    idx = np.empty((batch, k), dtype=np.int32)
    val = np.empty((batch, k), dtype=np.float32)
    rs = None if row_scales is None else np.ascontiguousarray(row_scales, dtype=np.float32)
    m = None if mask is None else np.ascontiguousarray(mask, dtype=np.uint8)
    lib().orc_hybrid_topk(dtype, _ptr(storage), scale, _ptr(rs), storage.shape[0], dim, _ptr(queries), batch, _ptr(m),
                          metric, _ptr(np.ascontiguousarray(offsets, dtype=np.int64)),
                          _ptr(np.ascontiguousarray(docs, dtype=np.int32)),
                          _ptr(np.ascontiguousarray(weights, dtype=np.float32)), vocab, _ptr(terms), terms.shape[1],
                          dense_weight, k, _ptr(idx), _ptr(val))
    return idx, val
