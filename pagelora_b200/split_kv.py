"""Host side of split-KV decode across GPUs (long contexts, config 5).

Every row's context pages are cut into `world` contiguous ranges; shard i
holds range i and the last shard also owns the growing tail (new decode
tokens append there).  Each shard computes the partial attention state
(O fp32, LSE) of its range; the partials are all-gathered over NCCL and
merged by log-sum-exp on every shard, so all shards continue the layer with
the same attention output.  There is no reference counterpart: the
reference decodes a sequence on one GPU.
"""

from __future__ import annotations


def shard_page_range(n_pages: int, rank: int, world: int) -> tuple[int, int]:
    """[p0, p1) of a row's n_pages pages held by shard `rank` of `world`."""

    if not 0 <= rank < world:
        raise ValueError("rank must satisfy 0 <= rank < world")
    return n_pages * rank // world, n_pages * (rank + 1) // world


def shard_row(n_tokens: int, page_size: int, rank: int, world: int) -> tuple[int, int, int]:
    """(p0, p1, tokens in the shard's last page) of a row of n_tokens tokens.

    Shards other than the last hold only full pages of the middle of the
    context, so their last page is full; the last shard holds the tail."""

    n_pages = -(-n_tokens // page_size)
    p0, p1 = shard_page_range(n_pages, rank, world)
    if rank == world - 1:
        last = n_tokens - (n_pages - 1) * page_size if n_pages else 0
    else:
        last = page_size if p1 > p0 else 0
    return p0, p1, last
