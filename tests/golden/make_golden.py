"""Generates tests/golden/*.npz from the reference's own code. Run in a container that has the
reference tree (its path in ZCGVS_REFERENCE):

    ZCGVS_REFERENCE=<reference checkout> python tests/golden/make_golden.py

Sources of truth (nothing from the reference is copied; it is imported / linked read-only):
  * python/zcgvs_tools/formats.py  - sign packing, per-matrix int8 quantisation, row strides
  * tests/cpp/cpu_reference.hpp    - cpuCosineSimilarity, cpuTopKIndices,
    cpuQuantizeDequantizeInt8, cpuPackBinary, cpuHamming (through oracle/_ref/libzcgvs_refcpu.so,
    built by `make -C oracle ref REF=<reference checkout>`)

Inputs are regenerated from seeds with the oracle's std::mt19937 generators (oracle/gen.cpp),
which reproduce the reference harnesses' randomMatrix; a CRC of every input is stored so a
drifting generator is caught.
"""

from __future__ import annotations

import ctypes
import os
import sys
import zlib
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
if not os.environ.get("ZCGVS_REFERENCE"):
    sys.exit("set ZCGVS_REFERENCE to the reference checkout (the script imports its Python tools)")
REF = Path(os.environ["ZCGVS_REFERENCE"])
sys.path.insert(0, str(ROOT / "oracle"))
sys.path.insert(0, str(REF / "python"))

import oracle  # noqa: E402
from zcgvs_tools import formats  # noqa: E402

P = ctypes.c_void_p


def crc(a: np.ndarray) -> int:
    return zlib.crc32(np.ascontiguousarray(a).tobytes())


def ref_scores(ref, corpus, queries):
    n, dim = corpus.shape
    out = np.empty((queries.shape[0], n), dtype=np.float32)
    ref.refcpu_scores(corpus.ctypes.data_as(P), n, dim, queries.ctypes.data_as(P), queries.shape[0],
                      out.ctypes.data_as(P))
    return out


def ref_topk(ref, scores, k):
    batch, n = scores.shape
    out = np.empty((batch, k), dtype=np.int32)
    ref.refcpu_topk(np.ascontiguousarray(scores).ctypes.data_as(P), n, batch, k, out.ctypes.data_as(P))
    return out


def main() -> None:
    oracle.build()
    ref = oracle.ref_lib()
    if ref is None:
        raise SystemExit("oracle/_ref/libzcgvs_refcpu.so missing: run make -C oracle ref REF=<reference checkout>")

    # 1. Format conventions from formats.py.
    fmt = {}
    for dim in (130, 384, 97, 1024, 33):
        m = oracle.normal_rows(16, dim, 3 + dim)
        fmt[f"pack_{dim}"] = formats.pack_binary(m)
        q, s = formats.quantize_int8(m)
        fmt[f"q8_{dim}"] = q
        fmt[f"q8scale_{dim}"] = np.float32(s)
        fmt[f"input_crc_{dim}"] = np.int64(crc(m))
        for code in (formats.DTYPE_FLOAT32, formats.DTYPE_FLOAT16, formats.DTYPE_INT8, formats.DTYPE_BINARY):
            fmt[f"stride_{code}_{dim}"] = np.int64(formats.row_stride(code, dim))
    np.savez_compressed(HERE / "formats.npz", **fmt)

    # 2. Scores + top-k of the reference CPU code over each storage form, small seeded cases.
    scan = {}
    for dim in (97, 100, 256, 384):
        corpus = oracle.normal_rows(512, dim, 11 + dim)
        queries = oracle.normal_rows(3, dim, 97 + dim)
        scan[f"crc_corpus_{dim}"] = np.int64(crc(corpus))
        scan[f"crc_queries_{dim}"] = np.int64(crc(queries))
        # float32 rows
        s = ref_scores(ref, corpus, queries)
        scan[f"f32_scores_{dim}"] = s
        scan[f"f32_top10_{dim}"] = ref_topk(ref, s, 10)
        # float16 storage: the reference test's __half2float(__float2half_rn(x)) rounding
        stored16 = corpus.astype(np.float16).astype(np.float32)
        s = ref_scores(ref, stored16, queries)
        scan[f"f16_scores_{dim}"] = s
        scan[f"f16_top10_{dim}"] = ref_topk(ref, s, 10)
        # int8 storage, scale 1/127, dequantised by cpuQuantizeDequantizeInt8
        scale = np.float32(1.0 / 127.0)
        deq = np.empty(corpus.size, dtype=np.float32)
        ref.refcpu_quantize_dequantize_i8(corpus.ctypes.data_as(P), corpus.size, ctypes.c_float(scale),
                                          deq.ctypes.data_as(P))
        deq = deq.reshape(corpus.shape)
        s = ref_scores(ref, deq, queries)
        scan[f"i8_scores_{dim}"] = s
        scan[f"i8_top10_{dim}"] = ref_topk(ref, s, 10)
        # binary: cpuPackBinary + cpuHamming, score (dim - 2h) / dim
        words = (dim + 31) // 32
        pc = np.empty((512, words), dtype=np.uint32)
        pq = np.empty((3, words), dtype=np.uint32)
        ref.refcpu_pack_binary(corpus.ctypes.data_as(P), 512, dim, pc.ctypes.data_as(P))
        ref.refcpu_pack_binary(queries.ctypes.data_as(P), 3, dim, pq.ctypes.data_as(P))
        ham = np.empty((3, 512), dtype=np.int32)
        for q in range(3):
            for i in range(512):
                ham[q, i] = ref.refcpu_hamming(pc[i].ctypes.data_as(P), pq[q].ctypes.data_as(P), words)
        scan[f"bin_hamming_{dim}"] = ham
        scan[f"bin_packed_{dim}"] = pc
    np.savez_compressed(HERE / "scan_small.npz", **scan)

    # 3. Known-answer tests of the reference harnesses.
    kat = {}
    # test_pipeline.cu: the exact CPU top-10 of a seed-31 corpus (8192 x 256) and seed-32 query.
    corpus = oracle.normal_rows(8192, 256, 31)
    query = oracle.normal_rows(1, 256, 32)
    s = ref_scores(ref, corpus, query)
    kat["pipeline_top10"] = ref_topk(ref, s, 10)
    kat["pipeline_crc"] = np.int64(crc(corpus) ^ crc(query))
    # test_topk.cu: 5000 uniform(-100, 100) scores, seed 7, k = 100.
    scores = oracle.uniform(5000, 7, -100.0, 100.0)
    kat["topk5000_top100"] = ref_topk(ref, scores[None, :], 100)
    kat["topk5000_crc"] = np.int64(crc(scores))
    # test_topk_large.cu: 1e6 uniform(-1000, 1000) scores, seed 17, k = 512.
    scores = oracle.uniform(1000000, 17, -1000.0, 1000.0)
    kat["topk1m_top512"] = ref_topk(ref, scores[None, :], 512)
    kat["topk1m_crc"] = np.int64(crc(scores))
    np.savez_compressed(HERE / "kat.npz", **kat)

    for name in ("formats.npz", "scan_small.npz", "kat.npz"):
        print(name, (HERE / name).stat().st_size, "bytes")


if __name__ == "__main__":
    main()
