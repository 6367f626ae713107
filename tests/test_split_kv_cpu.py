"""Split-KV decode across ranks, host side, on CPU with gloo (world size 2 and 3).

Each rank takes its page range of every row (pagelora_b200.split_kv), computes
the oracle's partial attention state over those pages, all-gathers the
partials and merges them by log-sum-exp.  The merged output must equal the
oracle's single-device paged decode, and the ranges must partition every
row with the tail (last page) on the last rank.
"""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle.paged_decode import attend, merge_states, paged_decode
from pagelora_b200.split_kv import shard_row


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _case(seed=0):
    rng = np.random.default_rng(seed)
    ps, hq, hkv, d = 16, 8, 2, 64
    lengths = [1, 15, 16, 17, 100, 260, 33]
    pages_per_row = [-(-n // ps) for n in lengths]
    pool = sum(pages_per_row) + 4
    cache = rng.normal(size=(pool, 2, ps, hkv, d)).astype(np.float32)
    perm = rng.permutation(pool)
    indptr = np.cumsum([0] + pages_per_row)
    indices = perm[: indptr[-1]]
    last = np.array([n - (p - 1) * ps for n, p in zip(lengths, pages_per_row)])
    q = rng.normal(size=(len(lengths), hq, d)).astype(np.float32)
    return lengths, ps, cache, indptr, indices, last, q


def _worker(rank, world, port, results):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        lengths, ps, cache, indptr, indices, last, q = _case()
        rows, hq, d = q.shape
        hkv = cache.shape[3]
        part_o = np.zeros((rows, hq, d))
        part_lse = np.full((rows, hq), -np.inf)
        ranges = []
        for b, n in enumerate(lengths):
            p0, p1, kept_last = shard_row(n, ps, rank, world)
            ranges.append((p0, p1, kept_last))
            pages = indices[indptr[b] + p0: indptr[b] + p1]
            if len(pages) == 0:
                continue
            k = cache[pages, 0].reshape(-1, hkv, d).astype(np.float64)
            v = cache[pages, 1].reshape(-1, hkv, d).astype(np.float64)
            keep = (len(pages) - 1) * ps + kept_last
            part_o[b], part_lse[b] = attend(q[b].astype(np.float64), k[:keep], v[:keep], 1.0 / np.sqrt(d))
        # all-gather partials (packed [O | LSE]) and the ranges
        packed = torch.from_numpy(np.concatenate([part_o.reshape(-1), part_lse.reshape(-1)]))
        bufs = [torch.empty_like(packed) for _ in range(world)]
        dist.all_gather(bufs, packed)
        all_ranges = [None] * world
        dist.all_gather_object(all_ranges, ranges)
        nd = rows * hq * d
        v_all = np.stack([t[:nd].numpy().reshape(rows * hq, d) for t in bufs])   # [W, rows*hq, d]
        lse_all = np.stack([t[nd:].numpy().reshape(rows * hq) for t in bufs])    # [W, rows*hq]
        merged, _ = merge_states(v_all, lse_all)
        if rank == 0:
            full, _ = paged_decode(q, cache, indptr.tolist(), indices.tolist(), last.tolist())
            results["err"] = float(np.max(np.abs(merged.reshape(rows, hq, d) - full)))
            results["ranges"] = all_ranges
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_split_kv_partials_merge_to_full_decode(world):
    ctx = mp.get_context("spawn")
    with ctx.Manager() as mgr:
        results = mgr.dict()
        port = _free_port()
        procs = [ctx.Process(target=_worker, args=(r, world, port, results)) for r in range(world)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout=120)
            assert p.exitcode == 0
        err = results["err"]
        ranges = results["ranges"]
    assert err < 1e-9, err
    lengths, ps = _case()[0], _case()[1]
    for b, n in enumerate(lengths):
        n_pages = -(-n // ps)
        spans = [ranges[r][b] for r in range(world)]
        assert spans[0][0] == 0 and spans[-1][1] == n_pages
        for (a0, a1, _), (b0, _, _) in zip(spans, spans[1:]):
            assert a1 == b0  # contiguous, disjoint
        assert spans[-1][2] == n - (n_pages - 1) * ps  # the tail is on the last rank
        for r in range(world - 1):
            assert spans[r][2] in (0, ps)
