"""Drop-in page-table builders on the device.

Mirrors model/kvcache/flashinfer_page_table.py (FlashInferPageTable :12-18,
FlashInferPageTableBuffer :21-65, FlashInferBatchPageTableBuffer :68-134,
build_flashinfer_page_table :137-157, build_flashinfer_batch_page_table
:160-181): the same names, arguments, reusable grow-only buffers and
ValueError messages, but the coalescing, validation and CSR construction
run in one kernel (pl_page_table_build).  The spans are flattened on the
host into one pinned int32 array, copied with one H2D transfer, and the
kernel's status word plus the table length come back in one small D2H read
(the reference's torch.tensor uploads are synchronous too).  A span is any
object with block_id / start / length attributes (radix_types.KVBlockSpan)
or a (block_id, start, length) tuple.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Sequence

import torch

from pagelora_b200 import kernels as K
from pagelora_b200._capi import SPAN_ERROR_MESSAGES


@dataclass(frozen=True)
class KVBlockSpan:
    """Slice into a KV block (radix_types.py:30-36)."""

    block_id: int
    start: int
    length: int


@dataclass(frozen=True)
class FlashInferPageTable:
    paged_kv_indptr: torch.Tensor
    paged_kv_indices: torch.Tensor
    paged_kv_last_page_len: torch.Tensor


def _span_fields(span) -> tuple[int, int, int]:
    if isinstance(span, (tuple, list)):
        return int(span[0]), int(span[1]), int(span[2])
    return int(span.block_id), int(span.start), int(span.length)


class _DeviceBuilder:
    """Staging buffers + one kernel launch per build."""

    def __init__(self, device: torch.device) -> None:
        if torch.device(device).type != "cuda":
            raise RuntimeError("page tables are built by a CUDA kernel (no CPU path)")
        self.device = torch.device(device)
        self.status = torch.zeros(2, dtype=torch.int32, device=self.device)
        self.readback = torch.zeros(2, dtype=torch.int32, pin_memory=True)

    def build(self, batch_spans: Sequence[Sequence], page_size: int, out_indptr: torch.Tensor,
              out_indices: torch.Tensor, out_last: torch.Tensor) -> int:
        if page_size <= 0:
            raise ValueError("page_size must be positive")
        n_rows = len(batch_spans)
        flat: list[int] = []
        counts = [0]
        for row in batch_spans:
            for span in row:
                flat.extend(_span_fields(span))
            counts.append(counts[-1] + len(row))
        n_spans = counts[-1]
        # one pinned host block: [blk | start | length] (span-major) + row indptr
        host = torch.empty(3 * max(1, n_spans) + n_rows + 1, dtype=torch.int32, pin_memory=True)
        if n_spans:
            fl = torch.tensor(flat, dtype=torch.int32).view(n_spans, 3).t().contiguous().view(-1)
            host[: 3 * n_spans] = fl
        host[3 * max(1, n_spans):] = torch.tensor(counts, dtype=torch.int32)
        dev = host.to(self.device, non_blocking=True)
        s = max(1, n_spans)
        self.status.zero_()
        K.page_table_build(dev[0:s], dev[s:2 * s], dev[2 * s:3 * s], dev[3 * s:], page_size, out_indptr,
                           out_indices, out_last, self.status[0:1], self.status[1:2])
        # status and table length in one D2H read
        self.readback[0:1].copy_(self.status[0:1], non_blocking=True)
        self.readback[1:2].copy_(out_indptr[n_rows: n_rows + 1], non_blocking=True)
        torch.cuda.current_stream(self.device).synchronize()
        code = int(self.readback[0])
        if code in SPAN_ERROR_MESSAGES:
            raise ValueError(SPAN_ERROR_MESSAGES[code])
        if code != 0:
            raise RuntimeError(f"page-table build failed with status {code}")
        return int(self.readback[1])


_builders: dict[torch.device, _DeviceBuilder] = {}


def _builder(device) -> _DeviceBuilder:
    dev = torch.device(device)
    if dev.type == "cuda" and dev.index is None:
        dev = torch.device("cuda", torch.cuda.current_device())
    b = _builders.get(dev)
    if b is None:
        b = _builders[dev] = _DeviceBuilder(dev)
    return b


def _span_count(batch_spans) -> int:
    return sum(len(r) for r in batch_spans)


class FlashInferPageTableBuffer:
    """Reusable single-request page-table buffers (:21-65)."""

    def __init__(self, *, page_size: int, device: torch.device, initial_capacity: int = 16) -> None:
        if page_size <= 0:
            raise ValueError("page_size must be positive")
        self.page_size = int(page_size)
        self.device = torch.device(device)
        capacity = max(1, int(initial_capacity))
        self.paged_kv_indptr = torch.empty(2, device=self.device, dtype=torch.int32)
        self.paged_kv_last_page_len = torch.empty(1, device=self.device, dtype=torch.int32)
        self.paged_kv_indices = torch.empty(capacity, device=self.device, dtype=torch.int32)

    def update_from_spans(self, spans) -> FlashInferPageTable:
        self._ensure_capacity(len(spans))
        n = _builder(self.device).build([spans], self.page_size, self.paged_kv_indptr, self.paged_kv_indices,
                                        self.paged_kv_last_page_len)
        return FlashInferPageTable(self.paged_kv_indptr, self.paged_kv_indices[:n], self.paged_kv_last_page_len)

    def _ensure_capacity(self, required: int) -> None:
        if required <= self.paged_kv_indices.numel():
            return
        new_capacity = max(required, self.paged_kv_indices.numel() * 2)
        self.paged_kv_indices = torch.empty(new_capacity, device=self.device, dtype=torch.int32)


class FlashInferBatchPageTableBuffer:
    """Reusable batched page-table buffers (:68-134)."""

    def __init__(self, *, page_size: int, device: torch.device, initial_rows: int = 2,
                 initial_pages: int = 16) -> None:
        if page_size <= 0:
            raise ValueError("page_size must be positive")
        self.page_size = int(page_size)
        self.device = torch.device(device)
        rows = max(1, int(initial_rows))
        self.paged_kv_indptr = torch.empty(rows + 1, device=self.device, dtype=torch.int32)
        self.paged_kv_last_page_len = torch.empty(rows, device=self.device, dtype=torch.int32)
        self.paged_kv_indices = torch.empty(max(1, int(initial_pages)), device=self.device, dtype=torch.int32)

    def update_from_batch_spans(self, batch_spans) -> FlashInferPageTable:
        rows = len(batch_spans)
        self._ensure_row_capacity(rows)
        self._ensure_page_capacity(_span_count(batch_spans))
        n = _builder(self.device).build(batch_spans, self.page_size, self.paged_kv_indptr, self.paged_kv_indices,
                                        self.paged_kv_last_page_len)
        return FlashInferPageTable(self.paged_kv_indptr[: rows + 1], self.paged_kv_indices[:n],
                                   self.paged_kv_last_page_len[:rows])

    def _ensure_row_capacity(self, required_rows: int) -> None:
        if required_rows <= self.paged_kv_last_page_len.numel():
            return
        cap = max(required_rows, self.paged_kv_last_page_len.numel() * 2)
        self.paged_kv_indptr = torch.empty(cap + 1, device=self.device, dtype=torch.int32)
        self.paged_kv_last_page_len = torch.empty(cap, device=self.device, dtype=torch.int32)

    def _ensure_page_capacity(self, required_pages: int) -> None:
        if required_pages <= self.paged_kv_indices.numel():
            return
        cap = max(required_pages, self.paged_kv_indices.numel() * 2)
        self.paged_kv_indices = torch.empty(cap, device=self.device, dtype=torch.int32)


def build_flashinfer_page_table(spans, *, page_size: int, device: torch.device,
                                pin_memory: bool = False) -> FlashInferPageTable:
    """Single-row table from aligned page spans (:137-157)."""

    del pin_memory  # the table is built on the device
    buf = FlashInferPageTableBuffer(page_size=page_size, device=device, initial_capacity=max(1, len(spans)))
    return buf.update_from_spans(spans)


def build_flashinfer_batch_page_table(batch_spans, *, page_size: int, device: torch.device) -> FlashInferPageTable:
    """Batched table from per-request page spans (:160-181)."""

    buf = FlashInferBatchPageTableBuffer(page_size=page_size, device=device, initial_rows=max(1, len(batch_spans)),
                                         initial_pages=max(1, _span_count(batch_spans)))
    return buf.update_from_batch_spans(batch_spans)
