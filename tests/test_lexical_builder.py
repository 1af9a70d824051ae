"""The offline BM25 index builder (lexical_index.build_csr) against the reference's own builder.

tests/golden/lexical.npz holds indexes written by the reference's unmodified
python/zcgvs_tools/build_lexical.py (run by tests/golden/make_lexical.py on a seeded synthetic
corpus, with its own WordPiece pass giving each document's term ids): the default BM25
parameters, BASELINE config 5's (k1 0.9, b 0.4), a 24-token document cap, and a corpus of
empty documents (the builder's average-length fallback of 1). build_csr on the same term ids
must write the same offsets, documents and fp32 weights, and the same header, bit for bit; on
CPU tensors here, and on the GPU in the gpu tier (its per-posting float64 operations run on the
device).
"""

from __future__ import annotations

import numpy as np
import pytest

from conftest import ROOT

import formats  # noqa: E402
import lexical_index as li  # noqa: E402

GOLDEN = np.load(ROOT / "tests" / "golden" / "lexical.npz")
CASES = ["default", "cfg5", "capped", "empty_default"]


def _docs(case):
    if case.startswith("empty_"):
        return [[] for _ in range(5)]
    offsets, tokens = GOLDEN["doc_offsets"], GOLDEN["doc_tokens"]
    return [tokens[offsets[i]:offsets[i + 1]] for i in range(offsets.size - 1)]


def _check(case, device, tmp_path):
    import torch

    vocab = int(GOLDEN["vocab_size"])
    k1, b, cap = GOLDEN[f"{case}_params"]
    docs, terms, tf, lengths = li.token_counts(_docs(case), vocab, int(cap))
    t = lambda a: torch.from_numpy(a).to(device)  # noqa: E731
    offsets, pdocs, weights = li.build_csr(t(docs), t(terms), t(tf), t(lengths), vocab, k1=float(k1), b=float(b))
    path = tmp_path / "ours.lex"
    formats.write_lexical_index(path, len(lengths), vocab, offsets.cpu().numpy(), pdocs.cpu().numpy(),
                                weights.cpu().numpy(), float(k1), float(b), li.average_length(lengths))
    ref = GOLDEN[f"{case}_lex"].tobytes()
    ours = path.read_bytes()
    if ours != ref:
        (tmp_path / "ref.lex").write_bytes(ref)
        a, b2 = formats.read_lexical_index(tmp_path / "ref.lex"), formats.read_lexical_index(path)
        for key in a:
            if isinstance(a[key], np.ndarray):
                diff = np.flatnonzero(a[key] != b2[key])
                assert diff.size == 0, f"{key}: {diff.size} entries differ, first at {diff[:5]}"
            else:
                assert a[key] == b2[key], key
    assert ours == ref


@pytest.mark.parametrize("case", CASES)
def test_build_csr_writes_the_reference_builders_index(case, tmp_path):
    _check(case, "cpu", tmp_path)


@pytest.mark.gpu
@pytest.mark.parametrize("case", CASES)
def test_build_csr_on_the_gpu_writes_the_reference_builders_index(zc, case, tmp_path):
    _check(case, "cuda", tmp_path)
