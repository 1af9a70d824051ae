"""Row-sharded search across the GPUs of one node (one process per GPU, torch.distributed).

The reference runs on one GPU. For corpora that do not fit one GPU (50M x 768 fp16 is 77 GB)
or to scale one query stream over 8 GPUs, rows are split into P contiguous shards, one per
rank. Every rank searches its shard with ``id_base`` = its first row, so its [B, k] result
carries global ids; one NCCL all-gather brings every shard's result to every rank; and
``zcgvs_merge_topk`` selects the global top-k under (score desc, id asc). The union of per-shard
top-k lists contains the global top-k and the order is total, so the result is identical to a
single-GPU search over the whole corpus.

The exchange is [P, B, k] ids and score bits (B x k x 8 bytes per rank): latency-bound, so one
all-gather of a packed int32 tensor is used, capturable in a CUDA graph. A coarse search with
rescoring (ShardedRescoreSearch) exchanges twice: the coarse top-M, then the rescored top-k.
"""

from __future__ import annotations


def shard_bounds(n: int, world: int, rank: int) -> tuple[int, int]:
    """Rows [begin, end) of shard `rank` when n rows are split as evenly as possible."""
    base, extra = divmod(n, world)
    begin = rank * base + min(rank, extra)
    return begin, begin + base + (1 if rank < extra else 0)


class ShardedSearch:
    """One rank's part of a row-sharded top-k search over rows [shard_begin, shard_end).

    local_search(queries, k, id_base) -> (ids int32 [B, k], scores fp32 [B, k]) searches this
    rank's shard; merge(ids [P, B, k], scores [P, B, k], k) -> ([B, k], [B, k]) merges. The
    defaults are the CUDA library's zcgvs_scan_topk and zcgvs_merge_topk; the all-gather goes
    through torch.distributed (NCCL on GPUs).
    """

    def __init__(self, shard_begin: int, shard_end: int, local_search, merge=None, group=None):
        self.shard_begin = shard_begin
        self.shard_end = shard_end
        self.local_search = local_search
        if merge is None:
            import zcgvs_sm100 as zc

            merge = zc.merge_topk
        self.merge = merge
        self.group = group

    def search(self, queries, k: int):
        # Every shard returns its own top-k, so k must fit the shard (a one-GPU search over the
        # whole corpus would accept a larger k; say why it fails here).
        if not 0 < k <= self.shard_end - self.shard_begin:
            raise ValueError(f"sharded search needs 0 < k <= rows per shard; got k={k}, shard rows "
                             f"{self.shard_end - self.shard_begin}")
        ids, scores = self.local_search(queries, k, self.shard_begin)
        return gather_merge(ids, scores, k, self.merge, self.group)


def gather_merge(ids, scores, k: int, merge, group=None):
    """Every rank's [B, k_in] (global ids, scores) -> the global top-k on every rank: one
    all-gather of ids and score bits packed side by side, then `merge` over [P, B, k_in]."""
    import torch
    import torch.distributed as dist

    world = dist.get_world_size(group)
    packed = torch.stack([ids, scores.view(torch.int32)])            # [2, B, k_in]
    # Concatenated along dim 0 (the layout every backend accepts), then viewed per rank.
    gathered = torch.empty((world * 2,) + tuple(packed.shape[1:]), dtype=packed.dtype, device=packed.device)
    dist.all_gather_into_tensor(gathered, packed, group=group)
    gathered = gathered.view((world, 2) + tuple(packed.shape[1:]))
    all_ids = gathered[:, 0].contiguous()                              # [P, B, k_in]
    all_scores = gathered[:, 1].contiguous().view(torch.float32)
    return merge(all_ids, all_scores, k)


class ShardedRescoreSearch:
    """One rank's part of a row-sharded coarse search with exact rescoring (
    1-bit top-M, fp16 rescore to top-k), with the reference's semantics: the rescore sees the
    global top-M.

    1. coarse_search(queries, m, id_base) -> [B, m] (global ids, scores) over this rank's codes;
    2. all-gather and merge: every rank holds the same global top-m;
    3. rescore(queries, local_candidates [B, m], k) -> [B, k] (local ids, scores) over this
       rank's rows of the rescore store, for the candidates it owns (the others are -1, which
       the rescore drops);
    4. all-gather and merge of the per-rank top-k.

    Each step's result is the single-GPU one (unions of per-shard top lists contain the global
    ones, the order is total), so the search equals the one-GPU pipeline bit for bit.
    """

    def __init__(self, shard_begin: int, shard_end: int, coarse_search, rescore, merge=None, group=None):
        self.shard_begin = shard_begin
        self.shard_end = shard_end
        self.coarse_search = coarse_search
        self.rescore = rescore
        if merge is None:
            import zcgvs_sm100 as zc

            merge = zc.merge_topk
        self.merge = merge
        self.group = group

    def search(self, queries, m: int, k: int):
        import torch

        # Every shard returns m coarse candidates (the per-shard search, like the reference's
        # top-k, rejects m above its row count), and the rescore keeps k of the m.
        if not 0 < k <= m <= self.shard_end - self.shard_begin:
            raise ValueError(f"sharded rescore search needs 0 < k <= m <= rows per shard; got k={k}, m={m}, "
                             f"shard rows {self.shard_end - self.shard_begin}")
        ids, scores = self.coarse_search(queries, m, self.shard_begin)
        cand, _ = gather_merge(ids, scores, m, self.merge, self.group)
        mine = (cand >= self.shard_begin) & (cand < self.shard_end)
        local = torch.where(mine, cand - self.shard_begin, torch.full_like(cand, -1))
        r_ids, r_scores = self.rescore(queries, local, k)
        r_ids = torch.where(r_ids >= 0, r_ids + self.shard_begin, r_ids)
        return gather_merge(r_ids, r_scores, k, self.merge, self.group)


def scan_shard_search(corpus_shard, dtype: int, dim: int, *, scale: float = 1.0, row_scales=None, mask=None,
                      metric: int = 1, workspace=None):
    """local_search for ShardedSearch over a device-resident shard with zcgvs_scan_topk."""
    import zcgvs_sm100 as zc

    ws = workspace or zc.Workspace(corpus_shard.device)

    def run(queries, k, id_base):
        return zc.scan_topk(corpus_shard, dtype, dim, queries, k, scale=scale, row_scales=row_scales, mask=mask,
                            metric=metric, id_base=id_base, workspace=ws)

    return run
