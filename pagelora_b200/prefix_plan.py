"""Prefix reuse and page admission arithmetic of the paged KV manager.

A request whose prompt starts with tokens already in the radix prefix cache
reuses their KV pages.  The radix tree lookup itself stays the reference's
(``model/kvcache/radix_cache.py``: host metadata a drop-in user keeps); what
decides the page tables the decode kernels see is the arithmetic after it,
restated here so that the batch engine shares exactly the pages the
reference would:

* ``plan_prefix`` -- ``FlashInferPagedKVCacheManager._begin_request_unchecked``
  (``model/kvcache/paged_kvcache_manager.py:304-351``): clamp the match to
  the prompt, replay the last prompt token on a full hit, keep only the
  longest run of whole pages from offset 0 (``_flashinfer_usable_prefix_len``,
  ``:763-778``), slice and coalesce those spans;
* ``estimate_request_new_pages`` / ``can_fit_request`` /
  ``max_decode_tokens_that_fit`` -- the admission estimate
  (``paged_kvcache_manager.py:133-175``, used by
  ``model/kvcache/page_admission.py:45-139``).

Spans are anything with ``block_id``, ``start`` and ``length`` (the
reference's ``KVBlockSpan`` or :class:`pagelora_b200.page_table.KVBlockSpan`).
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Sequence

from pagelora_b200.page_table import KVBlockSpan


def _fields(span) -> tuple[int, int, int]:
    return int(span.block_id), int(span.start), int(span.length)


def slice_block_spans(spans: Sequence, start: int, length: int | None = None) -> list[KVBlockSpan]:
    """Spans covering tokens ``[start, start + length)`` of the concatenated
    spans (``model/kvcache/radix_storage.py:40-74``; same errors)."""

    if start < 0:
        raise ValueError("span slice start must be non-negative")
    total = sum(_fields(s)[2] for s in spans)
    if length is None:
        length = total - start
    if length < 0 or start + length > total:
        raise ValueError("block span slice out of range")
    out: list[KVBlockSpan] = []
    skip, left = start, length
    for s in spans:
        if left == 0:
            break
        bid, st, ln = _fields(s)
        if skip >= ln:
            skip -= ln
            continue
        take = min(ln - skip, left)
        out.append(KVBlockSpan(bid, st + skip, take))
        left -= take
        skip = 0
    return out


def coalesce_block_spans(spans: Sequence) -> list[KVBlockSpan]:
    """Drop empty slices and merge adjacent slices of one page
    (``model/kvcache/flashinfer_page_table.py:184-197``)."""

    out: list[KVBlockSpan] = []
    for s in spans:
        bid, st, ln = _fields(s)
        if ln <= 0:
            continue
        if out and out[-1].block_id == bid and out[-1].start + out[-1].length == st:
            out[-1] = KVBlockSpan(bid, out[-1].start, out[-1].length + ln)
        else:
            out.append(KVBlockSpan(bid, st, ln))
    return out


def usable_prefix_len(spans: Sequence, desired_len: int, page_size: int) -> int:
    """Longest prefix, at most ``desired_len`` tokens, made of whole pages from
    offset 0 (``paged_kvcache_manager.py:763-778``)."""

    if desired_len <= 0:
        return 0
    usable = 0
    for s in coalesce_block_spans(slice_block_spans(spans, 0, desired_len)):
        if s.start != 0 or s.length != page_size:
            break
        usable += s.length
    return min(usable, desired_len)


@dataclass(frozen=True)
class PrefixPlan:
    """What a new request reuses: ``match_len`` cached tokens, of which
    ``prefill_from`` are consumed through ``prefix_spans`` (whole pages);
    prefill recomputes tokens ``prefill_from..prompt_len``."""

    match_len: int
    prefill_from: int
    prefix_spans: list[KVBlockSpan]


def plan_prefix(prompt_len: int, key_match_len: int, key_spans: Sequence, page_size: int) -> PrefixPlan:
    """Prefix reuse of one request from its radix lookup result (the
    ``key_match_len`` and ``key_spans`` of the adapter's full-cache key;
    ``paged_kvcache_manager.py:304-351``)."""

    match_len = min(int(prompt_len), int(key_match_len))
    prefill_from = match_len
    if prompt_len > 0 and match_len == prompt_len:
        prefill_from = prompt_len - 1  # a full hit replays the last token for its logits
    prefill_from = usable_prefix_len(key_spans, prefill_from, page_size)
    spans = coalesce_block_spans(slice_block_spans(key_spans, 0, prefill_from))
    return PrefixPlan(match_len=match_len, prefill_from=prefill_from, prefix_spans=spans)


def estimate_request_new_pages(prefill_tokens: int, max_decode_tokens: int, page_size: int) -> int:
    """Conservative page count of one request's new tokens
    (``paged_kvcache_manager.py:133-148``)."""

    tokens = max(0, int(prefill_tokens)) + max(0, int(max_decode_tokens))
    return 0 if tokens == 0 else (tokens + page_size - 1) // page_size


def can_fit_request(prefill_tokens: int, max_decode_tokens: int, page_size: int, available_pages: int,
                    reserve_pages: int = 4) -> bool:
    """Admission test (``paged_kvcache_manager.py:150-163``)."""

    need = estimate_request_new_pages(prefill_tokens, max_decode_tokens, page_size)
    return need + max(0, int(reserve_pages)) <= available_pages


def max_decode_tokens_that_fit(prefill_tokens: int, requested_decode_tokens: int, page_size: int,
                               available_pages: int, reserve_pages: int = 4) -> int:
    """Decode budget left after the prefill (``paged_kvcache_manager.py:165-175``)."""

    budget = max(0, available_pages - max(0, int(reserve_pages))) * page_size
    return max(0, min(int(requested_decode_tokens), budget - max(0, int(prefill_tokens))))
