"""Restatement of ragged paged prefill attention (test oracle, float64 math).

Test infrastructure only: the product path never imports this module.

Follows model/flashinfer/attention_backend.py:
  * plan_prefill: sm_scale = query_rescale / sqrt(D), causal, no RoPE  :133-170
  * run_prefill:  wrapper.run(q / query_rescale, layer_cache), NHD q
                  [sum(qo_len), Hq, D] or BHSD [B, Hq, S, D]           :172-190
and its callers model/flashinfer/generation.py:250-275 (one request) and
:278-308 (packed batch): request b's page table lists its prefix spans and
then its new spans, and qo_indptr counts only the new tokens, so the
queries are the LAST qo_len positions of the request's kv_len keys.  With
FlashInfer's causal mask query i (0-based among the new tokens) attends to
keys 0 .. kv_len - qo_len + i.

Each query reduces to the decode oracle's `attend` over its visible keys
(oracle/paged_decode.py, pinned by the decode golden vectors), so the
prefill restatement shares that pinning.  A query with no visible key gives
O = 0 and LSE = -inf.
"""

from __future__ import annotations

import math

import numpy as np

from oracle.paged_decode import attend, row_kv


def paged_prefill(q, kv_cache, qo_indptr, kv_indptr, kv_indices, kv_last_page_len, *, causal: bool = True,
                  query_rescale: float = 16.0) -> tuple[np.ndarray, np.ndarray]:
    """q [total_q, Hq, D] -> (O [total_q, Hq, D], LSE [total_q, Hq]) in float64."""

    q = np.asarray(q, dtype=np.float64)
    total_q, hq, d = q.shape
    sm_scale = query_rescale / math.sqrt(d)
    out = np.zeros((total_q, hq, d))
    lse = np.full((total_q, hq), -np.inf)
    qo_indptr = [int(v) for v in qo_indptr]
    for b in range(len(qo_indptr) - 1):
        k, v = row_kv(kv_cache, kv_indptr, kv_indices, kv_last_page_len, b)
        n_kv = k.shape[0]
        q0, q1 = qo_indptr[b], qo_indptr[b + 1]
        n_q = q1 - q0
        for i in range(n_q):
            vis = n_kv - n_q + i + 1 if causal else n_kv
            vis = max(0, min(vis, n_kv))
            out[q0 + i], lse[q0 + i] = attend(q[q0 + i] / query_rescale, k[:vis], v[:vis], sm_scale)
    return out, lse


def paged_prefill_bhsd(q, kv_cache, qo_indptr, kv_indptr, kv_indices, kv_last_page_len, *, causal: bool = True,
                       query_rescale: float = 16.0) -> np.ndarray:
    """BHSD form of run_prefill (attention_backend.py:177-183): q [B, Hq, S, D]
    with every request S tokens long -> O [B, Hq, S, D]."""

    q = np.asarray(q, dtype=np.float64)
    bsz, hq, s, d = q.shape
    nhd = q.transpose(0, 2, 1, 3).reshape(bsz * s, hq, d)
    o, _ = paged_prefill(nhd, kv_cache, qo_indptr, kv_indptr, kv_indices, kv_last_page_len, causal=causal,
                         query_rescale=query_rescale)
    return o.reshape(bsz, s, hq, d).transpose(0, 2, 1, 3)
