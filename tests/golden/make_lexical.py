"""Generates tests/golden/lexical.npz by running the reference's own BM25 index builder,
python/zcgvs_tools/build_lexical.py, unchanged on a small seeded corpus. Run where the reference
tree exists (its path in ZCGVS_REFERENCE):

    ZCGVS_REFERENCE=<reference checkout> python tests/golden/make_lexical.py

The corpus is synthetic: a WordPiece vocabulary of made-up words and suffixes, and documents
drawn from it with a seeded generator (mixed case, punctuation, unknown words, an empty
document, documents longer than the token cap). The reference writes its metadata file with its
formats.write_metadata and builds the index with its command line (built-in WordPiece pass,
default and BASELINE config 5 BM25 parameters); its own tokenizer (build_tokenizer) gives each
document's term ids. A corpus of empty documents covers the builder's average-length fallback.
The fixture stores the vocabulary size, every document's term ids, and the .lex bytes per
parameter set.
"""

from __future__ import annotations

import os
import subprocess
import sys
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
if not os.environ.get("ZCGVS_REFERENCE"):
    sys.exit("set ZCGVS_REFERENCE to the reference checkout (the script runs its Python tools)")
REF = Path(os.environ["ZCGVS_REFERENCE"])
PARAMS = {"default": (1.2, 0.75, 512), "cfg5": (0.9, 0.4, 512), "capped": (1.2, 0.75, 24)}


def vocabulary(rng) -> list[str]:
    specials = ["[PAD]", "[UNK]", "[CLS]", "[SEP]", "[MASK]"]
    consonants, vowels = "bcdfghklmnprstvz", "aeiou"
    words = set()
    while len(words) < 300:
        n = int(rng.integers(1, 4))
        words.add("".join(rng.choice(list(consonants)) + rng.choice(list(vowels)) for _ in range(n)))
    suffixes = ["##s", "##ed", "##ing", "##er", "##ly", "##a", "##o"]
    punctuation = [".", ",", "!", "?", "-", "(", ")"]
    return specials + sorted(words) + suffixes + punctuation


def documents(rng, vocab: list[str], count: int) -> list[str]:
    words = [w for w in vocab if not w.startswith("[") and not w.startswith("##") and w.isalpha()]
    suffixes = [w[2:] for w in vocab if w.startswith("##")]
    weights = 1.0 / np.arange(1, len(words) + 1) ** 1.1
    weights /= weights.sum()
    docs = []
    for d in range(count):
        if d == 7:
            docs.append("")
            continue
        n = int(rng.poisson(30 if d % 5 else 70))
        parts = []
        for _ in range(n):
            w = words[int(rng.choice(len(words), p=weights))]
            r = rng.random()
            if r < 0.15:
                w += suffixes[int(rng.integers(len(suffixes)))]
            elif r < 0.2:
                w = w.upper()
            elif r < 0.23:
                w = "qxj" + w  # no WordPiece cover: [UNK]
            parts.append(w)
            if rng.random() < 0.1:
                parts.append(str(rng.choice(list(".,!?"))))
        docs.append(" ".join(parts))
    return docs


def main() -> None:
    sys.path.insert(0, str(REF / "python"))
    from zcgvs_tools import build_lexical, formats

    rng = np.random.default_rng(20261202)
    vocab = vocabulary(rng)
    texts = documents(rng, vocab, 240)
    out = {"vocab_size": np.array(len(vocab))}
    with tempfile.TemporaryDirectory() as tmp:
        tmp = Path(tmp)
        (tmp / "vocab.txt").write_text("\n".join(vocab) + "\n", encoding="utf-8")
        encode = build_lexical.build_tokenizer(tmp / "vocab.txt", None)
        ids = [encode(t) for t in texts]
        out["doc_offsets"] = np.cumsum([0] + [len(x) for x in ids]).astype(np.int64)
        out["doc_tokens"] = np.array([i for x in ids for i in x], dtype=np.int32)
        env = dict(os.environ, PYTHONPATH=str(REF / "python"))
        for corpus, doc_texts in (("", texts), ("empty_", [""] * 5)):
            formats.write_metadata(tmp / "c.meta", [f"d{i}" for i in range(len(doc_texts))], doc_texts)
            for name, (k1, b, cap) in PARAMS.items():
                if corpus and name != "default":
                    continue
                lex = tmp / f"{corpus}{name}.lex"
                subprocess.run([sys.executable, "-m", "zcgvs_tools.build_lexical", "--metadata", str(tmp / "c.meta"),
                                "--vocab", str(tmp / "vocab.txt"), "--output", str(lex), "--k1", str(k1), "--b", str(b),
                                "--max-doc-tokens", str(cap)], check=True, env=env, capture_output=True)
                out[f"{corpus}{name}_lex"] = np.frombuffer(lex.read_bytes(), dtype=np.uint8)
                out[f"{corpus}{name}_params"] = np.array([k1, b, cap], dtype=np.float64)
    np.savez_compressed(HERE / "lexical.npz", **out)
    print("lexical.npz", (HERE / "lexical.npz").stat().st_size, "bytes")


if __name__ == "__main__":
    main()
