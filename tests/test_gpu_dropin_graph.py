"""The drop-in attention backend inside a captured CUDA graph, the way the
reference's decode runner uses FlashInfer's wrapper.

The reference captures a whole decode step whose attention launches were
planned by ``plan_decode`` (model/flashinfer/cuda_graph.py:222-263), keyed by
``DecodeGraphKey`` (cuda_graph.py:76-93, 277-295), which folds in the page-table
buffer pointers and the backend's ``decode_graph_signature()``.  Between
replays it only replans: the new page table is copied into the persistent
graph-safe buffers (attention_backend.py:198-221), and a new graph is captured
when the key changes.  These tests do the same with ``B200AttentionBackend``
and check every replay against the fp64 oracle.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle.numerics import bf16
from oracle.paged_decode import paged_decode as o_decode

pytestmark = pytest.mark.gpu


def _table(rng, lens, pool, ps=16):
    npg = [-(-L // ps) for L in lens]
    assert sum(npg) <= pool
    indices = rng.permutation(pool)[: sum(npg)].tolist()
    indptr = np.cumsum([0] + npg).tolist()
    last = [L - (n - 1) * ps for L, n in zip(lens, npg)]
    return indptr, indices, last


def _plan(be, indptr, indices, last, pinned):
    def host(a):
        t = torch.tensor(a, dtype=torch.int32)
        return t.pin_memory() if pinned else t.cuda()

    be.plan_decode(paged_kv_indptr=host(indptr), paged_kv_indices=host(indices), paged_kv_last_page_len=host(last),
                   q_data_type=torch.bfloat16, kv_data_type=torch.bfloat16)


@pytest.mark.parametrize("pinned", [False, True])
def test_captured_run_decode_follows_replans(cuda_device, pinned):
    from pagelora_b200.attention_backend import FlashInferAttentionBackend

    rng = np.random.default_rng(4)
    hq, hkv, d, ps, pool = 32, 8, 128, 16, 600
    cache_np = bf16(rng.normal(size=(pool, 2, ps, hkv, d)))
    cache = torch.tensor(cache_np, device="cuda").bfloat16()
    q_buf = torch.zeros((3, hq, 1, d), dtype=torch.bfloat16, device="cuda")
    be = FlashInferAttentionBackend(device=cuda_device, workspace_mb=32, num_qo_heads=hq, num_kv_heads=hkv,
                                    head_dim=d, page_size=ps)

    graphs: dict[tuple, tuple[torch.cuda.CUDAGraph, torch.Tensor]] = {}

    def capture_or_get():
        key = (be.decode_graph_signature(), cache.data_ptr(), tuple(q_buf.shape))
        if key not in graphs:
            side = torch.cuda.Stream()
            side.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(side):
                be.run_decode(q_buf, cache)  # warm-up launch outside the capture
            torch.cuda.current_stream().wait_stream(side)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                out = be.run_decode(q_buf, cache)
            graphs[key] = (g, out)
        return graphs[key]

    # A sequence of steps: contexts grow token by token (the same buffers and
    # split count, so one graph serves them), then jump far enough that the
    # plan changes and a second graph is captured.
    lens = [700, 33, 1500]
    steps = [[L + t for L in lens] for t in range(4)] + [[L + 1800 for L in lens]]
    for step_lens in steps:
        indptr, indices, last = _table(rng, step_lens, pool)
        _plan(be, indptr, indices, last, pinned)
        q_np = bf16(rng.normal(size=(3, hq, d)) * 2.0)
        q_buf.copy_(torch.tensor(q_np, device="cuda").bfloat16()[:, :, None])
        g, out = capture_or_get()
        g.replay()
        torch.cuda.synchronize()
        ref, _ = o_decode(q_np, cache_np, indptr, indices, last)
        err = float(np.max(np.abs(out[:, :, 0].float().cpu().numpy() - ref)))
        assert err <= 2e-2, (step_lens, err)
        assert int(be.status.item()) == 0
    # Token-by-token growth reused one graph; the jump made a second one.
    assert len(graphs) == 2, len(graphs)


def test_signature_tracks_plan_values(cuda_device):
    """A replan that changes a value baked into the launch (split count, row
    count, buffer pointers) changes the signature; one that only changes the
    page table contents does not (attention_backend.py:223-227)."""

    from pagelora_b200.attention_backend import FlashInferAttentionBackend

    rng = np.random.default_rng(1)
    be = FlashInferAttentionBackend(device=cuda_device, workspace_mb=32, num_qo_heads=32, num_kv_heads=8,
                                    head_dim=128, page_size=16)
    _plan(be, *_table(rng, [300, 40], 200), pinned=False)
    s0 = be.decode_graph_signature()
    _plan(be, *_table(rng, [301, 41], 200), pinned=False)
    assert be.decode_graph_signature() == s0
    _plan(be, *_table(rng, [300, 40, 5], 200), pinned=False)
    assert be.decode_graph_signature() != s0
