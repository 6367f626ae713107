"""Restatement of the reference's CSR page-table builder (test oracle).

Follows model/kvcache/flashinfer_page_table.py:
  * _coalesce_block_spans            :184-197
  * _validate_and_collect_page_table :200-221
  * build_flashinfer_batch_page_table :160-181
Spans are (block_id, start, length) triples (radix_types.py:30-36).
"""

from __future__ import annotations

from typing import Iterable, Sequence

ERR_START = "FlashInfer page spans must start at page offset 0"
ERR_LENGTH = "FlashInfer page span length is out of range"
ERR_NOT_FULL = "non-last FlashInfer page spans must be full pages"


def coalesce(spans: Iterable[Sequence[int]]) -> list[tuple[int, int, int]]:
    """Merge adjacent slices of one physical page; drop empty slices (:184-197)."""

    merged: list[tuple[int, int, int]] = []
    for block_id, start, length in spans:
        if length <= 0:
            continue
        if merged:
            pb, ps, pl = merged[-1]
            if pb == block_id and ps + pl == start:
                merged[-1] = (pb, ps, pl + length)
                continue
        merged.append((int(block_id), int(start), int(length)))
    return merged


def collect_row(spans: Iterable[Sequence[int]], page_size: int) -> tuple[list[int], int]:
    """Page ids and last-page length of one row; ValueError on bad spans (:200-221)."""

    if page_size <= 0:
        raise ValueError("page_size must be positive")
    merged = coalesce(spans)
    indices: list[int] = []
    last = 0
    for idx, (block_id, start, length) in enumerate(merged):
        if start != 0:
            raise ValueError(ERR_START)
        if length <= 0 or length > page_size:
            raise ValueError(ERR_LENGTH)
        if idx < len(merged) - 1 and length != page_size:
            raise ValueError(ERR_NOT_FULL)
        indices.append(block_id)
        last = length
    return indices, last


def build_batch(batch_spans: Sequence[Sequence[Sequence[int]]], page_size: int
                ) -> tuple[list[int], list[int], list[int]]:
    """(indptr, indices, last_page_len) of a batch (:160-181)."""

    indptr = [0]
    indices: list[int] = []
    last: list[int] = []
    for spans in batch_spans:
        row, ll = collect_row(spans, page_size)
        indices.extend(row)
        indptr.append(len(indices))
        last.append(ll)
    return indptr, indices, last


def advance(row_pages: list[list[int]], last_page_len: list[int], new_page_ids: Sequence[int], page_size: int
            ) -> tuple[list[int], list[int], list[int]]:
    """One decode token per row: reserve a slot, appending a page when the last
    is full (paged_kv_store.py:113-190 reserve_spans for a one-token chunk).
    Returns (slot_page, slot_offset, position) and mutates the row state."""

    slot_page, slot_off, pos = [], [], []
    for r, pages in enumerate(row_pages):
        if not pages or last_page_len[r] >= page_size:
            pages.append(int(new_page_ids[r]))
            last_page_len[r] = 1
        else:
            last_page_len[r] += 1
        slot_page.append(pages[-1])
        slot_off.append(last_page_len[r] - 1)
        pos.append((len(pages) - 1) * page_size + last_page_len[r] - 1)
    return slot_page, slot_off, pos
