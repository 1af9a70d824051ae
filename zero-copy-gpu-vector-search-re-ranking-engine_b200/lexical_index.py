"""Host-side helpers for the BM25 inverted index the hybrid search consumes.

The index is the reference's CSR layout (include/zcgvs/data/lexical_index.hpp:14-46):
``offsets`` [vocab + 1] int64, ``docs`` int32 and ``weights`` fp32 per posting, postings grouped
by term. The CUDA kernels need each term's postings sorted by document id, which the reference
builder already guarantees (python/zcgvs_tools/build_lexical.py:143-162); ``sort_postings``
establishes it for any other index without changing a single score (the sort is stable, so the
additions per document keep their order).

``build_csr`` computes the reference builder's BM25 weights from token counts
(build_lexical.py:143-154): idf = ln(1 + (N - df + 0.5) / (df + 0.5)),
w = idf * tf * (k1 + 1) / (tf + k1 * (1 - b + b * len / avgdl)), in float64, stored as fp32, with
the builder's operation order and its average-length fallback (1 when the mean length is 0), so
the weights equal the reference builder's bit for bit (tests/golden/lexical.npz holds indexes
written by the reference builder itself). ``token_counts`` turns tokenised documents into its
inputs the way the builder counts them.
``synthetic_corpus`` / ``synthetic_queries`` draw the seeded hybrid workload (Poisson document
lengths, Zipf term frequencies) on any torch device.
"""

from __future__ import annotations

import math

import numpy as np


def sort_postings(offsets, docs, weights):
    """Stable sort of every term's postings by document id. numpy arrays in, numpy arrays out."""
    offsets = np.asarray(offsets, dtype=np.int64)
    docs = np.asarray(docs, dtype=np.int32)
    weights = np.asarray(weights, dtype=np.float32)
    term_of = np.repeat(np.arange(offsets.size - 1, dtype=np.int64), np.diff(offsets))
    order = np.lexsort((docs, term_of))  # last key is primary; lexsort is stable
    return offsets.copy(), docs[order], weights[order]


def postings_sorted(offsets, docs) -> bool:
    """True when every term's postings are non-decreasing in document id."""
    offsets = np.asarray(offsets, dtype=np.int64)
    docs = np.asarray(docs, dtype=np.int64)
    if docs.size < 2:
        return True
    drops = np.flatnonzero(np.diff(docs) < 0) + 1  # positions where a document id decreases
    starts = np.zeros(docs.size, dtype=bool)
    starts[offsets[1:-1][offsets[1:-1] < docs.size]] = True
    return bool(starts[drops].all())


def average_length(lengths) -> float:
    """The builder's average document length (build_lexical.py:139-142): the float64 mean of the
    token counts, 1.0 when it is not positive (an empty corpus, or only empty documents)."""
    values = np.asarray(lengths.cpu() if hasattr(lengths, "cpu") else lengths, dtype=np.float64)
    mean = float(values.mean()) if values.size else 0.0
    return mean if mean > 0.0 else 1.0


def token_counts(doc_tokens, vocab: int, max_doc_tokens: int = 512):
    """(doc_ids, term_ids, tf, lengths) numpy int64 arrays from per-document token id lists, as
    the builder counts them (build_lexical.py:127-137): each document cut to max_doc_tokens
    tokens, its length the number kept, and one (doc, term, tf) entry per distinct in-vocabulary
    term."""
    docs, terms, counts, lengths = [], [], [], []
    for d, tokens in enumerate(doc_tokens):
        kept = np.asarray(tokens, dtype=np.int64)[:max_doc_tokens]
        lengths.append(kept.size)
        kept = kept[(kept >= 0) & (kept < vocab)]
        uniq, tf = np.unique(kept, return_counts=True)
        docs.append(np.full(uniq.size, d, dtype=np.int64))
        terms.append(uniq)
        counts.append(tf)
    cat = (lambda parts: np.concatenate(parts) if parts else np.zeros(0, dtype=np.int64))
    return cat(docs), cat(terms), cat(counts).astype(np.int64), np.asarray(lengths, dtype=np.int64)


def build_csr(doc_ids, term_ids, tf, lengths, vocab: int, k1: float = 1.2, b: float = 0.75):
    """BM25 CSR index from unique (doc, term) pairs with term frequencies.

    doc_ids, term_ids, tf: torch int64 tensors of the pairs (any order); lengths: torch tensor
    [n_docs] of document token counts. Returns torch (offsets int64 [vocab + 1], docs int32,
    weights fp32) on the inputs' device, postings sorted by (term, doc).

    The per-posting arithmetic runs as float64 torch operations on the inputs' device, each one
    rounded on its own in the builder's order; the two values torch could round differently from
    the builder are taken as the builder takes them: idf from Python's math.log once per
    document frequency, and the mean length from numpy (average_length).
    """
    import torch

    n_docs = lengths.numel()
    key = term_ids * n_docs + doc_ids
    order = torch.argsort(key)
    doc_ids, term_ids, tf = doc_ids[order], term_ids[order], tf[order].to(torch.float64)
    df_count = torch.bincount(term_ids, minlength=vocab)
    avgdl = average_length(lengths)
    df_host = df_count.cpu().numpy()
    idf_host = np.zeros(vocab, dtype=np.float64)
    for value in np.unique(df_host[df_host > 0]):
        idf_host[df_host == value] = math.log(1.0 + (n_docs - int(value) + 0.5) / (int(value) + 0.5))
    idf = torch.from_numpy(idf_host).to(doc_ids.device)
    norm = k1 * (1.0 - b + b * lengths.to(torch.float64)[doc_ids] / avgdl)
    weights = (idf[term_ids] * (tf * (k1 + 1.0)) / (tf + norm)).to(torch.float32)
    offsets = torch.zeros(vocab + 1, dtype=torch.int64, device=doc_ids.device)
    offsets[1:] = torch.cumsum(df_count, 0)
    return offsets, doc_ids.to(torch.int32), weights


def zipf_probs(vocab: int, s: float, device=None):
    import torch

    ranks = torch.arange(1, vocab + 1, dtype=torch.float64, device=device)
    p = ranks.pow(-s)
    return p / p.sum()


def synthetic_corpus(n_docs: int, vocab: int, mean_len: float, zipf_s: float, seed: int, device=None,
                     k1: float = 1.2, b: float = 0.75, chunk_tokens: int = 1 << 27):
    """Seeded BM25 index: lengths ~ Poisson(mean_len), tokens ~ Zipf(zipf_s) over the vocabulary
    (term id = rank - 1). Returns torch (offsets, docs, weights) on `device`."""
    import torch

    gen = torch.Generator(device=device or "cpu")
    gen.manual_seed(seed)
    rate = torch.full((n_docs,), float(mean_len), dtype=torch.float64, device=device)
    lengths = torch.poisson(rate, generator=gen).to(torch.int64)
    cdf = torch.cumsum(zipf_probs(vocab, zipf_s, device), 0)
    cdf[-1] = 1.0
    starts = torch.cumsum(lengths, 0) - lengths
    pairs = []
    # Draw tokens in chunks of whole documents so the (doc, term) keys fit memory.
    doc0 = 0
    while doc0 < n_docs:
        doc1 = int(torch.searchsorted(starts, (starts[doc0] + chunk_tokens).reshape(1), right=True)[0])
        doc1 = max(doc1, doc0 + 1)
        count = int(lengths[doc0:doc1].sum())
        if count:
            # Inverse-CDF draws: term = first rank whose cumulative probability exceeds u.
            u = torch.rand(count, dtype=torch.float64, device=device, generator=gen)
            tokens = torch.searchsorted(cdf, u, right=True).clamp_(max=vocab - 1)
            owner = torch.repeat_interleave(torch.arange(doc0, doc1, device=device), lengths[doc0:doc1])
            key, tf = torch.unique(owner * vocab + tokens, return_counts=True)
            pairs.append((key // vocab, key % vocab, tf))
        doc0 = doc1
    doc_ids = torch.cat([p[0] for p in pairs]) if pairs else torch.empty(0, dtype=torch.int64, device=device)
    term_ids = torch.cat([p[1] for p in pairs]) if pairs else torch.empty(0, dtype=torch.int64, device=device)
    tf = torch.cat([p[2] for p in pairs]) if pairs else torch.empty(0, dtype=torch.int64, device=device)
    return build_csr(doc_ids, term_ids, tf, lengths, vocab, k1, b)


def synthetic_queries(batch: int, vocab: int, zipf_s: float, seed: int, min_terms: int = 3, max_terms: int = 12):
    """[batch, max_terms] int32 numpy term ids: a U{min..max} count of Zipf-drawn terms per query,
    de-duplicated in first-occurrence order (Engine::lexicalTerms, src/engine/engine.cpp:150-172)
    and padded with -1."""
    rng = np.random.default_rng(seed)
    ranks = np.arange(1, vocab + 1, dtype=np.float64)
    p = ranks ** (-zipf_s)
    p /= p.sum()
    out = np.full((batch, max_terms), -1, dtype=np.int32)
    for q in range(batch):
        count = int(rng.integers(min_terms, max_terms + 1))
        drawn = rng.choice(vocab, size=count, p=p)
        _, first = np.unique(drawn, return_index=True)
        uniq = drawn[np.sort(first)]
        out[q, : uniq.size] = uniq
    return out
