"""Generates tests/golden/files.npz: ZCVE and ZCVL files written by the reference's own writer
(python/zcgvs_tools/formats.py, imported read-only from the reference tree), stored as byte
arrays beside the inputs they encode. The format tests check that this library's writer produces
the same bytes and that its readers (Python and C++) decode them. Run in a container that has
the reference tree (its path in ZCGVS_REFERENCE):

    ZCGVS_REFERENCE=<reference checkout> python tests/golden/make_format_files.py
"""

from __future__ import annotations

import os
import sys
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
if not os.environ.get("ZCGVS_REFERENCE"):
    sys.exit("set ZCGVS_REFERENCE to the reference checkout (the script imports its Python tools)")
REF = Path(os.environ["ZCGVS_REFERENCE"])
sys.path.insert(0, str(REF / "python"))

from zcgvs_tools import formats  # noqa: E402


def main() -> None:
    rng = np.random.default_rng(2024)
    matrix = rng.standard_normal((9, 70)).astype(np.float32)
    matrix /= np.linalg.norm(matrix, axis=1, keepdims=True).astype(np.float32)
    matrix[4] = 0.0  # an all-zero row
    out = {"matrix": matrix}
    with tempfile.TemporaryDirectory() as tmp:
        for dtype in ("float32", "float16", "int8", "binary"):
            path = Path(tmp) / f"{dtype}.zcve"
            formats.write_embeddings(path, matrix, normalized=(dtype != "int8"), dtype=dtype)
            out[f"zcve_{dtype}"] = np.frombuffer(path.read_bytes(), dtype=np.uint8)
        # A float16 input with the default dtype (float16 storage).
        path = Path(tmp) / "default16.zcve"
        formats.write_embeddings(path, matrix.astype(np.float16), normalized=True)
        out["zcve_default16"] = np.frombuffer(path.read_bytes(), dtype=np.uint8)

        offsets = np.array([0, 3, 3, 7, 8, 11], dtype=np.int64)
        docs = np.array([0, 4, 8, 1, 2, 3, 8, 5, 0, 6, 7], dtype=np.int32)
        weights = rng.uniform(0.1, 4.0, docs.shape[0]).astype(np.float32)
        path = Path(tmp) / "index.zcvl"
        formats.write_lexical_index(path, 9, 5, offsets, docs, weights, 0.9, 0.4, 12.5)
        out["zcvl"] = np.frombuffer(path.read_bytes(), dtype=np.uint8)
        out["lex_offsets"], out["lex_docs"], out["lex_weights"] = offsets, docs, weights
    np.savez_compressed(HERE / "files.npz", **out)
    print("files.npz", (HERE / "files.npz").stat().st_size, "bytes")


if __name__ == "__main__":
    main()
