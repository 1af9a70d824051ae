"""Results written straight into pinned host memory. Under unified addressing the kernels can
write a search's (id, score) pairs into pinned host buffers themselves (the end-to-end path of
bench.py and the C++ Searcher for small results do this instead of copying them back). The
three routes that write final results (the streaming scan's last CTA, the tensor-core path's
selection and the hybrid select kernel) must give exactly what they give in device buffers."""

from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def pinned_out(torch, batch, k):
    return (torch.empty((batch, k), dtype=torch.int32).pin_memory(),
            torch.empty((batch, k), dtype=torch.float32).pin_memory())


@pytest.mark.parametrize("n,batch,k", [(200_000, 1, 100), (100_000, 64, 10), (5_183, 1, 10)])
def test_scan_topk_into_pinned_host_memory(zc, orc, n, batch, k):
    import torch

    dim = 768
    corpus = orc.normal_rows(n, dim, 91)
    queries = orc.normal_rows(batch, dim, 92)
    storage, _, row_scales = orc.encode(corpus, 4)
    st, sc, q = torch.from_numpy(storage).cuda(), torch.from_numpy(row_scales).cuda(), torch.from_numpy(queries).cuda()
    ws = zc.Workspace()
    dev_i, dev_v = zc.scan_topk(st, 4, dim, q, k, row_scales=sc, workspace=ws)
    for _ in range(2):
        host = pinned_out(torch, batch, k)
        zc.scan_topk(st, 4, dim, q, k, row_scales=sc, workspace=ws, out=host)
        torch.cuda.synchronize()
        np.testing.assert_array_equal(host[0].numpy(), dev_i.cpu().numpy())
        np.testing.assert_array_equal(host[1].numpy(), dev_v.cpu().numpy())
    assert ws.status() == 0


def test_hybrid_topk_into_pinned_host_memory(zc, orc):
    import torch
    import lexical_index as li

    n, dim, vocab, k = 50_000, 384, 3000, 10
    offsets, docs, weights = li.synthetic_corpus(n, vocab, 40.0, 1.1, 93, k1=0.9, b=0.4)
    terms = torch.from_numpy(li.synthetic_queries(2, vocab, 1.1, 94)).cuda()
    corpus = orc.normal_rows(n, dim, 95)
    queries = torch.from_numpy(orc.normal_rows(2, dim, 96)).cuda()
    storage, _, _ = orc.encode(corpus, 1)
    st = torch.from_numpy(storage.view(np.int16)).cuda()
    index = zc.LexicalIndex(offsets.numpy(), docs.numpy(), weights.numpy())
    ws = zc.Workspace()
    for q in range(2):
        dev_i, dev_v = zc.hybrid_topk(st, 1, dim, queries[q:q + 1], k, index, terms[q:q + 1], 0.5, metric=0,
                                      workspace=ws)
        host = pinned_out(torch, 1, k)
        zc.hybrid_topk(st, 1, dim, queries[q:q + 1], k, index, terms[q:q + 1], 0.5, metric=0, workspace=ws, out=host)
        torch.cuda.synchronize()
        np.testing.assert_array_equal(host[0].numpy(), dev_i.cpu().numpy())
        np.testing.assert_array_equal(host[1].numpy(), dev_v.cpu().numpy())
    assert ws.status() == 0
