"""Drop-in replacement of the reference's FlashInfer attention backend.

``B200AttentionBackend`` keeps the constructor, attributes and plan/run
surface of model/flashinfer/attention_backend.py:18-292
(FlashInferAttentionBackend) so it can be injected where the reference
creates its backend (model/flashinfer/generation.py:105-121, _make_backend):

  * plan_decode(paged_kv_indptr=, paged_kv_indices=, paged_kv_last_page_len=,
    q_data_type=, kv_data_type=)                                   (:63-118)
  * run_decode(q, paged_kv_cache_layer) -> [B, Hq, 1, D]           (:120-131)
  * plan_prefill / run_prefill                                     (:133-190)
  * decode_graph_signature()                                       (:223-227)
  * decode_use_tensor_cores, query_rescale, use_flashinfer_qk_norm,
    workspace_buffer attributes                                    (:37-61)

Decode runs the sm_100a paged decode kernel through the C ABI; the page
table is copied into persistent, power-of-two sized device buffers at plan
time (the reference's graph-safe buffers, :198-221), so a captured decode
graph keeps valid pointers across replans.  Prefill runs the sm_100a
tcgen05 paged prefill kernel (ragged, causal) over the same page layout.
There is no FlashInfer and no CPU path: a non-CUDA device raises.
"""

from __future__ import annotations

import math
from collections import deque

import torch

from pagelora_b200 import kernels as K


class B200AttentionBackend:
    """Own the decode workspace and the plan/run calls of paged attention."""

    def __init__(self, *, device: torch.device, workspace_mb: int, num_qo_heads: int, num_kv_heads: int,
                 head_dim: int, page_size: int) -> None:
        self.device = torch.device(device)
        self.workspace_mb = max(1, int(workspace_mb))
        self.num_qo_heads = int(num_qo_heads)
        self.num_kv_heads = int(num_kv_heads)
        self.head_dim = int(head_dim)
        self.page_size = int(page_size)
        # Kept for interface parity: q / 16 with sm_scale * 16 is the same
        # softmax; the kernel applies sm_scale = 1/sqrt(D) in fp32 with a
        # true -inf mask, so no rescaling is needed.
        self.query_rescale = 16.0
        if self.num_kv_heads <= 0 or self.num_qo_heads % self.num_kv_heads:
            raise ValueError("Q head count must be divisible by KV head count")
        if self.device.type != "cuda":
            raise RuntimeError("B200AttentionBackend needs a CUDA device (no CPU path)")
        group = self.num_qo_heads // self.num_kv_heads
        # The reference picks FlashInfer's tensor-core wrapper for groups it
        # cannot specialise (:46-49); the value is kept for callers that read
        # it.  The B200 kernel always runs Q.K^T and P.V on the tensor cores.
        self.decode_use_tensor_cores = group not in (1, 2, 4, 8)
        self.use_flashinfer_qk_norm = False
        # Zeroed: the first bytes are the split-merge arrival counters.
        self.workspace_buffer = torch.zeros(self.workspace_mb * 1024 * 1024, dtype=torch.uint8, device=self.device)
        self.status = torch.zeros(1, dtype=torch.int32, device=self.device)
        self._decode_graph_buffers: tuple[torch.Tensor, torch.Tensor, torch.Tensor] | None = None
        self._decode_rows = 0
        self._decode_pages = 0
        self._num_splits = 1
        self._decode_host_uploads: deque = deque()
        self._prefill_plan: dict | None = None

    # ---------------------------------------------------------------- decode
    def plan_decode(self, *, paged_kv_indptr: torch.Tensor, paged_kv_indices: torch.Tensor,
                    paged_kv_last_page_len: torch.Tensor, q_data_type: torch.dtype | None = None,
                    kv_data_type: torch.dtype | None = None) -> None:
        """Plan one decode step (shared by all layers of the step)."""

        for dt in (q_data_type, kv_data_type):
            if dt is not None and dt != torch.bfloat16:
                raise NotImplementedError(f"B200 decode kernels are bf16 only (got {dt})")
        self._ensure_graph_safe_decode_buffers(paged_kv_indptr, paged_kv_indices, paged_kv_last_page_len)
        indptr_buf, indices_buf, last_buf = self._decode_graph_buffers
        host = (paged_kv_indptr, paged_kv_indices, paged_kv_last_page_len)
        async_host = all(t.device.type == "cpu" and t.is_pinned() for t in host)
        if async_host:
            # An async H2D source must stay alive until its copy completes (:80-88).
            while self._decode_host_uploads and self._decode_host_uploads[0][0].query():
                self._decode_host_uploads.popleft()
            if len(self._decode_host_uploads) >= 8:
                self._decode_host_uploads[0][0].synchronize()
                self._decode_host_uploads.popleft()
        nnz = paged_kv_indices.numel()
        indptr_buf.copy_(paged_kv_indptr.to(torch.int32), non_blocking=async_host)
        if nnz:
            indices_buf[:nnz].copy_(paged_kv_indices.to(torch.int32), non_blocking=async_host)
        last_buf.copy_(paged_kv_last_page_len.to(torch.int32), non_blocking=async_host)
        if async_host:
            ev = torch.cuda.Event()
            ev.record(torch.cuda.current_stream(self.device))
            self._decode_host_uploads.append((ev, host))
        batch = paged_kv_last_page_len.numel()
        plan = K.decode_plan(batch, self.num_qo_heads, self.num_kv_heads, self.head_dim, self.page_size, nnz)
        if plan.workspace_bytes > self.workspace_buffer.numel():
            raise RuntimeError(f"decode workspace of {self.workspace_mb} MiB is too small "
                               f"({plan.workspace_bytes} bytes needed)")
        self._num_splits = int(plan.num_splits)
        self._decode_rows = batch

    def run_decode(self, q: torch.Tensor, paged_kv_cache_layer: torch.Tensor) -> torch.Tensor:
        """One layer of paged decode attention; returns [B, Hq, 1, D]."""

        if self._decode_graph_buffers is None:
            raise RuntimeError("plan_decode must be called before run_decode")
        q_nhd = q.squeeze(2) if q.dim() == 4 and q.size(2) == 1 else q
        if q_nhd.stride(-1) != 1 or q_nhd.stride(-2) % 8 or q_nhd.stride(0) % 8:
            q_nhd = q_nhd.contiguous()
        indptr, indices, last = self._decode_graph_buffers
        out = K.paged_decode(q_nhd, paged_kv_cache_layer, indptr, indices, last, num_splits=self._num_splits,
                             workspace=self.workspace_buffer, status=self.status)
        return out.unsqueeze(2) if out.dim() == 3 else out

    def _ensure_graph_safe_decode_buffers(self, indptr: torch.Tensor, indices: torch.Tensor,
                                          last_page_len: torch.Tensor) -> None:
        buffers = self._decode_graph_buffers
        if buffers is not None and buffers[0].numel() == indptr.numel() and buffers[1].numel() >= indices.numel():
            return
        capacity = max(16, 1 << max(0, indices.numel() - 1).bit_length())
        self._decode_graph_buffers = (
            torch.empty(indptr.numel(), dtype=torch.int32, device=self.device),
            torch.zeros(capacity, dtype=torch.int32, device=self.device),
            torch.empty(last_page_len.numel(), dtype=torch.int32, device=self.device),
        )

    def decode_graph_signature(self):
        """Host-side plan values baked into a captured launch (:223-227)."""

        bufs = self._decode_graph_buffers
        ptrs = tuple(int(b.data_ptr()) for b in bufs) if bufs is not None else ()
        return (id(self), (self._num_splits, self._decode_rows, *ptrs))

    # --------------------------------------------------------------- prefill
    def plan_prefill(self, *, qo_indptr: torch.Tensor, paged_kv_indptr: torch.Tensor,
                     paged_kv_indices: torch.Tensor, paged_kv_last_page_len: torch.Tensor, causal: bool = True,
                     q_data_type: torch.dtype | None = None, kv_data_type: torch.dtype | None = None) -> None:
        """Record the ragged prefill layout (:133-170).  Nothing is planned on
        the host: the kernel finds each CTA's request and query tile from
        qo_indptr, so only device copies of the four index arrays are kept."""

        for dt in (q_data_type, kv_data_type):
            if dt is not None and dt != torch.bfloat16:
                raise NotImplementedError(f"B200 prefill kernel is bf16 only (got {dt})")
        dev = dict(device=self.device, dtype=torch.int32)
        self._prefill_plan = {
            "qo_indptr": qo_indptr.to(**dev).contiguous(),
            "kv_indptr": paged_kv_indptr.to(**dev).contiguous(),
            "kv_indices": paged_kv_indices.to(**dev).contiguous(),
            "last": paged_kv_last_page_len.to(**dev).contiguous(),
            "causal": bool(causal),
        }

    def run_prefill(self, q: torch.Tensor, paged_kv_cache_layer: torch.Tensor) -> torch.Tensor:
        """Paged prefill: q NHD [sum(qo), Hq, D] or BHSD [B, Hq, S, D] (:172-190).

        The reference runs q / query_rescale with sm_scale = query_rescale /
        sqrt(D); for the power-of-two rescale both scalings are exact, so the
        kernel applies 1 / sqrt(D) to q itself."""

        if q.dim() == 4:
            bsz, num_heads, seqlen, head_dim = q.shape
            q_nhd = q.transpose(1, 2).reshape(bsz * seqlen, num_heads, head_dim)
            out = self._prefill_nhd(q_nhd, paged_kv_cache_layer)
            return out.reshape(bsz, seqlen, num_heads, head_dim).transpose(1, 2).contiguous()
        return self._prefill_nhd(q, paged_kv_cache_layer)

    def _prefill_nhd(self, q: torch.Tensor, cache: torch.Tensor) -> torch.Tensor:
        plan = self._prefill_plan
        if plan is None:
            raise RuntimeError("plan_prefill must be called before run_prefill")
        if q.stride(-1) != 1 or q.stride(0) % 8 or q.stride(1) % 8 or q.data_ptr() % 16:
            q = q.contiguous()
        return K.paged_prefill(q, cache, plan["qo_indptr"], plan["kv_indptr"], plan["kv_indices"], plan["last"],
                               causal=plan["causal"], sm_scale=1.0 / math.sqrt(self.head_dim), status=self.status)


# Name of the reference class, for injection by name.
FlashInferAttentionBackend = B200AttentionBackend
