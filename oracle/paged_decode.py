"""Restatement of paged GQA decode attention (test oracle, float64 math).

Follows model/flashinfer/attention_backend.py:
  * plan_decode: sm_scale = query_rescale / sqrt(D)            :97
  * run_decode:  wrapper.run(q / query_rescale, layer_cache)    :127-131
so O = softmax((q/16) . K^T * 16/sqrt(D)) . V = softmax(q . K^T / sqrt(D)) . V,
with query head h reading kv head h // (Hq/Hkv).  The page pool layout is
[P, 2, page_size, Hkv, D] with K at [:, 0] and V at [:, 1]
(model/kvcache/paged_kv_store.py:559-570); a row's tokens are its pages
indices[indptr[b]:indptr[b+1]] in order with last_page_len[b] valid tokens
in the final page (model/kvcache/flashinfer_page_table.py:200-221).
The LSE is returned in natural log; an empty row gives O = 0, LSE = -inf.
"""

from __future__ import annotations

import math

import numpy as np


def row_kv(kv_cache: np.ndarray, indptr, indices, last_page_len, b: int) -> tuple[np.ndarray, np.ndarray]:
    """K, V of row b as [n_tokens, Hkv, D] float64."""

    pages = np.asarray(indices[indptr[b]: indptr[b + 1]], dtype=np.int64)
    _, _, ps, hkv, d = kv_cache.shape
    if pages.size == 0:
        empty = np.zeros((0, hkv, d))
        return empty, empty
    n_tok = (pages.size - 1) * ps + int(last_page_len[b])
    k = kv_cache[pages, 0].reshape(-1, hkv, d)[:n_tok].astype(np.float64)
    v = kv_cache[pages, 1].reshape(-1, hkv, d)[:n_tok].astype(np.float64)
    return k, v


def attend(q: np.ndarray, k: np.ndarray, v: np.ndarray, sm_scale: float) -> tuple[np.ndarray, np.ndarray]:
    """q [Hq, D], k/v [N, Hkv, D] -> (O [Hq, D], LSE [Hq]) in float64."""

    hq, d = q.shape
    n, hkv, _ = k.shape
    group = hq // hkv
    out = np.zeros((hq, d))
    lse = np.full(hq, -np.inf)
    if n == 0:
        return out, lse
    for h in range(hq):
        kh = k[:, h // group, :]
        vh = v[:, h // group, :]
        s = (kh @ q[h].astype(np.float64)) * sm_scale
        m = s.max()
        p = np.exp(s - m)
        l = p.sum()
        out[h] = (p @ vh) / l
        lse[h] = m + math.log(l)
    return out, lse


def paged_decode(q, kv_cache, indptr, indices, last_page_len, *, query_rescale: float = 16.0
                 ) -> tuple[np.ndarray, np.ndarray]:
    """Decode attention for every row: q [B, Hq, D] -> (O [B, Hq, D], LSE [B, Hq])."""

    q = np.asarray(q, dtype=np.float64)
    b_sz, hq, d = q.shape
    sm_scale = query_rescale / math.sqrt(d)
    out = np.zeros((b_sz, hq, d))
    lse = np.full((b_sz, hq), -np.inf)
    for b in range(b_sz):
        k, v = row_kv(kv_cache, indptr, indices, last_page_len, b)
        out[b], lse[b] = attend(q[b] / query_rescale, k, v, sm_scale)
    return out, lse


def split_states(q, kv_cache, indptr, indices, last_page_len, b: int, num_splits: int
                 ) -> tuple[np.ndarray, np.ndarray]:
    """Partial (O, LSE) of row b over num_splits contiguous page ranges
    (ceil(n_pages / num_splits) pages each, the last ones possibly empty)."""

    q = np.asarray(q, dtype=np.float64)
    _, hq, d = q.shape
    _, _, ps, hkv, _ = kv_cache.shape
    pages = list(indices[indptr[b]: indptr[b + 1]])
    n = len(pages)
    pps = -(-n // num_splits) if n else 0
    outs = np.zeros((num_splits, hq, d))
    lses = np.full((num_splits, hq), -np.inf)
    for s in range(num_splits):
        p0, p1 = min(s * pps, n), min(s * pps + pps, n)
        if p1 <= p0:
            continue
        sub = np.asarray(pages[p0:p1], dtype=np.int64)
        k = kv_cache[sub, 0].reshape(-1, hkv, d).astype(np.float64)
        v = kv_cache[sub, 1].reshape(-1, hkv, d).astype(np.float64)
        if p1 == n:
            keep = (p1 - p0 - 1) * ps + int(last_page_len[b])
            k, v = k[:keep], v[:keep]
        outs[s], lses[s] = attend(q[b], k, v, 1.0 / math.sqrt(d))
    return outs, lses


def merge_states(v: np.ndarray, lse: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """Log-sum-exp merge of partial states: v [S, ..., D], lse [S, ...]."""

    v = np.asarray(v, dtype=np.float64)
    lse = np.asarray(lse, dtype=np.float64)
    m = np.max(lse, axis=0)
    finite = np.isfinite(m)
    m_safe = np.where(finite, m, 0.0)
    w = np.where(np.isfinite(lse), np.exp(lse - m_safe[None]), 0.0)
    total = w.sum(axis=0)
    out = np.where(total[..., None] > 0, (w[..., None] * v).sum(axis=0) / np.maximum(total, 1e-300)[..., None], 0.0)
    out_lse = np.where(total > 0, m_safe + np.log(np.maximum(total, 1e-300)), -np.inf)
    return out, out_lse
