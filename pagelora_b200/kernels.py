"""Torch-tensor wrappers over the C ABI (``include/pagelora_b200.h``).

Each function validates dtype / device / layout on the host, passes raw
device pointers and the current CUDA stream to the library and raises on a
non-zero status.  None of them allocates unless it creates its own output
(``out=None``), and none synchronises, so every call is capturable in a
CUDA graph when its outputs are preallocated.
"""

from __future__ import annotations

import math

import torch

from pagelora_b200 import _capi
from pagelora_b200._capi import DecodePlan, call, ptr, stream_handle


def _need_cuda(*tensors: torch.Tensor | None) -> None:
    for t in tensors:
        if t is not None and t.device.type != "cuda":
            raise RuntimeError("pagelora_b200 kernels run on CUDA tensors only (no CPU path)")


def _need(t: torch.Tensor, dtype: torch.dtype, name: str) -> None:
    if t.dtype != dtype:
        raise TypeError(f"{name} must be {dtype}, got {t.dtype}")


def _row_stride(t: torch.Tensor, name: str) -> int:
    if t.dim() < 2:
        return t.shape[-1] if t.dim() == 1 else 0
    if t.stride(-1) != 1:
        raise ValueError(f"{name} must be contiguous in its last dimension")
    return t.stride(-2)


# ------------------------------------------------------------ page tables
def page_table_build(
    span_block_id: torch.Tensor,
    span_start: torch.Tensor,
    span_length: torch.Tensor,
    row_indptr: torch.Tensor,
    page_size: int,
    out_indptr: torch.Tensor,
    out_indices: torch.Tensor,
    out_last_page_len: torch.Tensor,
    status: torch.Tensor,
    err_row: torch.Tensor | None = None,
) -> None:
    """Device CSR page-table build from spans (see pl_page_table_build)."""

    _need_cuda(span_block_id, out_indptr, status)
    for name, t in (("span_block_id", span_block_id), ("span_start", span_start), ("span_length", span_length),
                    ("row_indptr", row_indptr), ("out_indptr", out_indptr), ("out_indices", out_indices),
                    ("out_last_page_len", out_last_page_len), ("status", status)):
        _need(t, torch.int32, name)
    num_rows = row_indptr.numel() - 1
    call("pl_page_table_build", ptr(span_block_id), ptr(span_start), ptr(span_length), ptr(row_indptr),
         num_rows, int(page_size), ptr(out_indptr), ptr(out_indices), ptr(out_last_page_len), ptr(status),
         ptr(err_row), stream_handle())


def page_table_advance(
    row_num_pages: torch.Tensor,
    last_page_len: torch.Tensor,
    row_pages: torch.Tensor,
    new_page_ids: torch.Tensor,
    page_size: int,
    out_indptr: torch.Tensor,
    out_indices: torch.Tensor,
    slot_page_id: torch.Tensor,
    slot_offset: torch.Tensor,
    positions: torch.Tensor | None,
    status: torch.Tensor,
) -> None:
    """Advance a device page table by one token per row (pl_page_table_advance)."""

    _need_cuda(row_pages, status)
    num_rows, cap = row_pages.shape
    call("pl_page_table_advance", ptr(row_num_pages), ptr(last_page_len), ptr(row_pages), ptr(new_page_ids),
         int(num_rows), int(cap), int(page_size), ptr(out_indptr), ptr(out_indices), ptr(slot_page_id),
         ptr(slot_offset), ptr(positions), ptr(status), stream_handle())


# ------------------------------------------------------- decode attention
def decode_plan(batch: int, num_qo_heads: int, num_kv_heads: int, head_dim: int, page_size: int,
                total_pages: int, max_splits: int = 0) -> DecodePlan:
    plan = DecodePlan()
    lib = _capi.load_library()
    _capi.check("pl_decode_plan", lib.pl_decode_plan(int(batch), int(num_qo_heads), int(num_kv_heads),
                                                     int(head_dim), int(page_size), int(total_pages),
                                                     int(max_splits), plan))
    return plan


def paged_decode(
    q: torch.Tensor,
    kv_cache: torch.Tensor,
    indptr: torch.Tensor,
    indices: torch.Tensor,
    last_page_len: torch.Tensor,
    *,
    num_splits: int,
    workspace: torch.Tensor | None,
    status: torch.Tensor | None = None,
    sm_scale: float | None = None,
    out: torch.Tensor | None = None,
    out_lse: torch.Tensor | None = None,
    prior: tuple[torch.Tensor, torch.Tensor] | None = None,
) -> torch.Tensor:
    """Paged decode attention: q [B, Hq, D] bf16, kv_cache [P, 2, PS, Hkv, D] bf16;
    ``out`` bf16, or fp32 for a split-KV shard's partial state.  ``prior`` =
    (O fp32 [B, Hq, D], LSE [B, Hq] natural log): a state merged into the
    bf16 output (pl_paged_decode_merge_prior)."""

    _need_cuda(q, kv_cache, indptr, indices, last_page_len)
    _need(q, torch.bfloat16, "q")
    _need(kv_cache, torch.bfloat16, "kv_cache")
    if kv_cache.dim() != 5 or kv_cache.size(1) != 2 or not kv_cache.is_contiguous():
        raise ValueError("kv_cache must be a contiguous [pages, 2, page_size, kv_heads, head_dim] tensor")
    if q.dim() != 3 or q.stride(-1) != 1:
        raise ValueError("q must be [batch, qo_heads, head_dim] with unit last stride")
    for name, t in (("indptr", indptr), ("indices", indices), ("last_page_len", last_page_len)):
        _need(t, torch.int32, name)
    batch, hq, d = q.shape
    num_pages, _, page_size, hkv, d2 = kv_cache.shape
    if d2 != d:
        raise ValueError("q and kv_cache head_dim differ")
    if out is None:
        out = torch.empty_like(q)
    scale = (1.0 / math.sqrt(d)) if sm_scale is None else float(sm_scale)
    ws_bytes = 0 if workspace is None else workspace.numel() * workspace.element_size()
    if prior is not None:
        po, pl = prior
        if (out.dtype != torch.bfloat16 or out_lse is not None or po.dtype != torch.float32 or
                pl.dtype != torch.float32 or not po.is_contiguous() or not pl.is_contiguous() or
                po.numel() < batch * hq * d or pl.numel() < batch * hq):
            raise ValueError("prior needs contiguous fp32 [B, Hq, D] / [B, Hq] states and a bf16 out without out_lse")
        call("pl_paged_decode_merge_prior", ptr(q), q.stride(0), q.stride(1), ptr(kv_cache), int(num_pages),
             ptr(indptr), ptr(indices), ptr(last_page_len), int(batch), int(hq), int(hkv), int(d), int(page_size),
             scale, int(num_splits), ptr(out), out.stride(0), out.stride(1), ptr(po), ptr(pl), ptr(workspace),
             int(ws_bytes), ptr(status), stream_handle())
        return out
    fn = "pl_paged_decode_f32" if out.dtype == torch.float32 else "pl_paged_decode"
    call(fn, ptr(q), q.stride(0), q.stride(1), ptr(kv_cache), int(num_pages), ptr(indptr),
         ptr(indices), ptr(last_page_len), int(batch), int(hq), int(hkv), int(d), int(page_size), scale,
         int(num_splits), ptr(out), out.stride(0), out.stride(1), ptr(out_lse), ptr(workspace), int(ws_bytes),
         ptr(status), stream_handle())
    return out


def paged_decode_shared(
    q: torch.Tensor,
    kv_cache: torch.Tensor,
    indptr: torch.Tensor,
    indices: torch.Tensor,
    last_page_len: torch.Tensor,
    *,
    fold: int,
    num_splits: int,
    workspace: torch.Tensor | None,
    out: torch.Tensor,
    out_lse: torch.Tensor | None = None,
    status: torch.Tensor | None = None,
    sm_scale: float | None = None,
) -> torch.Tensor:
    """Paged decode where query row b uses page-table row b // fold (rows
    that share a page list read it once per `fold` rows); ``out`` bf16 or
    fp32 [B, Hq, D]."""

    _need_cuda(q, kv_cache, indptr, indices, last_page_len, out)
    _need(q, torch.bfloat16, "q")
    _need(kv_cache, torch.bfloat16, "kv_cache")
    if kv_cache.dim() != 5 or kv_cache.size(1) != 2 or not kv_cache.is_contiguous():
        raise ValueError("kv_cache must be a contiguous [pages, 2, page_size, kv_heads, head_dim] tensor")
    batch, hq, d = q.shape
    num_pages, _, page_size, hkv, _ = kv_cache.shape
    scale = (1.0 / math.sqrt(d)) if sm_scale is None else float(sm_scale)
    ws_bytes = 0 if workspace is None else workspace.numel() * workspace.element_size()
    flags = _capi.PL_DECODE_OUT_F32 if out.dtype == torch.float32 else 0
    call("pl_paged_decode_shared", ptr(q), q.stride(0), q.stride(1), ptr(kv_cache), int(num_pages), ptr(indptr),
         ptr(indices), ptr(last_page_len), int(batch), int(fold), int(hq), int(hkv), int(d), int(page_size), scale,
         int(num_splits), ptr(out), out.stride(0), out.stride(1), ptr(out_lse), int(flags), ptr(workspace),
         int(ws_bytes), ptr(status), stream_handle())
    return out


def paged_decode_qkv(
    qkv: torch.Tensor,
    kv_cache: torch.Tensor,
    indptr: torch.Tensor,
    indices: torch.Tensor,
    last_page_len: torch.Tensor,
    *,
    num_qo_heads: int,
    num_kv_heads: int,
    positions: torch.Tensor,
    rope_theta: float,
    slot_page: torch.Tensor,
    slot_offset: torch.Tensor,
    num_splits: int,
    workspace: torch.Tensor | None,
    lora_down: torch.Tensor | None = None,
    lora_b: torch.Tensor | None = None,
    lora_scale: float = 1.0,
    tok_adapter: torch.Tensor | None = None,
    q_norm_weight: torch.Tensor | None = None,
    k_norm_weight: torch.Tensor | None = None,
    norm_eps: float = 1e-6,
    out: torch.Tensor | None = None,
    out_lse: torch.Tensor | None = None,
    q_out: torch.Tensor | None = None,
    status: torch.Tensor | None = None,
    sm_scale: float | None = None,
    rope_cos_sin: torch.Tensor | None = None,
) -> torch.Tensor:
    """q/k head norm + RoPE + paged append + paged decode in one launch, from
    the packed projection rows ``qkv`` [B, (Hq + 2 Hkv) * D] bf16; ``out`` is
    [B, Hq, D] bf16, or fp32 for a split-KV partial.  ``rope_cos_sin``: the
    step's table from :func:`rope_cos_sin` (else the angles are evaluated in
    the launch)."""

    _need_cuda(qkv, kv_cache, indptr, indices, last_page_len, positions, slot_page, slot_offset)
    _need(qkv, torch.bfloat16, "qkv")
    _need(kv_cache, torch.bfloat16, "kv_cache")
    if kv_cache.dim() != 5 or kv_cache.size(1) != 2 or not kv_cache.is_contiguous():
        raise ValueError("kv_cache must be a contiguous [pages, 2, page_size, kv_heads, head_dim] tensor")
    batch = qkv.shape[0]
    num_pages, _, page_size, hkv, d = kv_cache.shape
    if hkv != num_kv_heads or qkv.shape[1] != (num_qo_heads + 2 * num_kv_heads) * d:
        raise ValueError("qkv / kv_cache shapes do not match the head counts")
    if out is None:
        out = torch.empty(batch, num_qo_heads, d, dtype=torch.bfloat16, device=qkv.device)
    rank = 0
    if lora_b is not None:
        if lora_b.dim() == 2:
            lora_b = lora_b.unsqueeze(0)
        rank = lora_b.shape[-1]
    scale = (1.0 / math.sqrt(d)) if sm_scale is None else float(sm_scale)
    ws_bytes = 0 if workspace is None else workspace.numel() * workspace.element_size()
    flags = _capi.PL_DECODE_OUT_F32 if out.dtype == torch.float32 else 0
    call("pl_paged_decode_qkv", ptr(qkv), _row_stride(qkv, "qkv"), ptr(lora_down),
         0 if lora_down is None else _row_stride(lora_down, "lora_down"), ptr(lora_b), int(rank), float(lora_scale),
         ptr(tok_adapter), ptr(q_norm_weight), ptr(k_norm_weight), float(norm_eps), ptr(positions),
         float(rope_theta), ptr(rope_cos_sin), ptr(slot_page), ptr(slot_offset), ptr(q_out), ptr(kv_cache),
         int(num_pages), ptr(indptr),
         ptr(indices), ptr(last_page_len), int(batch), int(num_qo_heads), int(num_kv_heads), int(d),
         int(page_size), scale, int(num_splits), ptr(out), out.stride(0), out.stride(1), ptr(out_lse), int(flags),
         ptr(workspace), int(ws_bytes), ptr(status), stream_handle())
    return out


def rope_cos_sin(positions: torch.Tensor, head_dim: int, rope_theta: float,
                 out: torch.Tensor | None = None) -> torch.Tensor:
    """(cos, sin) of every RoPE angle of each row's position: [rows, D/2, 2] fp32."""

    _need_cuda(positions)
    _need(positions, torch.int32, "positions")
    rows = positions.numel()
    if out is None:
        out = torch.empty(rows, head_dim // 2, 2, dtype=torch.float32, device=positions.device)
    call("pl_rope_cos_sin", ptr(positions), int(rows), int(head_dim), float(rope_theta), ptr(out), stream_handle())
    return out


def merge_states(v_partial: torch.Tensor, lse_partial: torch.Tensor, out: torch.Tensor | None = None,
                 out_lse: torch.Tensor | None = None) -> torch.Tensor:
    """Merge [rows, S, D] fp32 partial states with natural-log LSE [rows, S]."""

    _need_cuda(v_partial, lse_partial)
    _need(v_partial, torch.float32, "v_partial")
    _need(lse_partial, torch.float32, "lse_partial")
    rows, states, d = v_partial.shape
    if not v_partial.is_contiguous() or not lse_partial.is_contiguous():
        raise ValueError("partial states must be contiguous")
    if out is None:
        out = torch.empty(rows, d, dtype=torch.bfloat16, device=v_partial.device)
    call("pl_merge_states", ptr(v_partial), ptr(lse_partial), int(rows), int(states), int(d), ptr(out),
         _row_stride(out, "out"), ptr(out_lse), stream_handle())
    return out


def merge_states_strided(v_partial: torch.Tensor, lse_partial: torch.Tensor, out: torch.Tensor,
                         out_lse: torch.Tensor | None = None) -> torch.Tensor:
    """Merge partial states given as views ``v_partial`` [rows, S, D] and
    ``lse_partial`` [rows, S] with any strides (D unit-stride), e.g. a
    permuted [S, rows, D] all-gather result."""

    _need_cuda(v_partial, lse_partial, out)
    _need(v_partial, torch.float32, "v_partial")
    _need(lse_partial, torch.float32, "lse_partial")
    rows, states, d = v_partial.shape
    if v_partial.stride(2) != 1:
        raise ValueError("partial states need unit stride along head_dim")
    call("pl_merge_states_strided", ptr(v_partial), v_partial.stride(0), v_partial.stride(1), ptr(lse_partial),
         lse_partial.stride(0), lse_partial.stride(1), int(rows), int(states), int(d), ptr(out),
         _row_stride(out, "out"), ptr(out_lse), stream_handle())
    return out


# ------------------------------------------------------- prefill attention
def paged_prefill(
    q: torch.Tensor,
    kv_cache: torch.Tensor,
    qo_indptr: torch.Tensor,
    kv_indptr: torch.Tensor,
    kv_indices: torch.Tensor,
    kv_last_page_len: torch.Tensor,
    *,
    causal: bool = True,
    sm_scale: float | None = None,
    out: torch.Tensor | None = None,
    out_lse: torch.Tensor | None = None,
    status: torch.Tensor | None = None,
) -> torch.Tensor:
    """Ragged paged prefill attention: q [total_q, Hq, D] bf16 (NHD), request b
    owns tokens qo_indptr[b]:qo_indptr[b+1], which are the last positions of
    its kv_len keys; ``out`` bf16 like q, ``out_lse`` fp32 [total_q, Hq]."""

    _need_cuda(q, kv_cache, qo_indptr, kv_indptr, kv_indices, kv_last_page_len)
    _need(q, torch.bfloat16, "q")
    _need(kv_cache, torch.bfloat16, "kv_cache")
    if kv_cache.dim() != 5 or kv_cache.size(1) != 2 or not kv_cache.is_contiguous():
        raise ValueError("kv_cache must be a contiguous [pages, 2, page_size, kv_heads, head_dim] tensor")
    if q.dim() != 3 or q.stride(-1) != 1:
        raise ValueError("q must be [tokens, qo_heads, head_dim] with unit last stride")
    for name, t in (("qo_indptr", qo_indptr), ("kv_indptr", kv_indptr), ("kv_indices", kv_indices),
                    ("kv_last_page_len", kv_last_page_len)):
        _need(t, torch.int32, name)
    total_q, hq, d = q.shape
    num_pages, _, page_size, hkv, d2 = kv_cache.shape
    if d2 != d:
        raise ValueError("q and kv_cache head_dim differ")
    if out is None:
        out = torch.empty_like(q)
    scale = (1.0 / math.sqrt(d)) if sm_scale is None else float(sm_scale)
    call("pl_paged_prefill", ptr(q), q.stride(0), q.stride(1), ptr(kv_cache), int(num_pages), ptr(qo_indptr),
         ptr(kv_indptr), ptr(kv_indices), ptr(kv_last_page_len), int(qo_indptr.numel() - 1), int(total_q), int(hq),
         int(hkv), int(d), int(page_size), scale, 1 if causal else 0, ptr(out), out.stride(0), out.stride(1),
         ptr(out_lse), ptr(status), stream_handle())
    return out


# --------------------------------------------------------------- LoRA path
def lora_shrink_seg(x: torch.Tensor, a_stack: torch.Tensor, seg_indptr: torch.Tensor,
                    seg_adapter: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """down[t] = x[t] . A[adapter(seg(t))]^T (fp32), a_stack [n_adapters, rank, in]."""

    _need_cuda(x, a_stack, seg_indptr, seg_adapter)
    _need(x, torch.bfloat16, "x")
    _need(a_stack, torch.bfloat16, "a_stack")
    _need(seg_indptr, torch.int32, "seg_indptr")
    _need(seg_adapter, torch.int32, "seg_adapter")
    n_ad, rank, k = a_stack.shape
    t = x.shape[0]
    if out is None:
        out = torch.empty(t, rank, dtype=torch.float32, device=x.device)
    call("pl_lora_shrink_seg", ptr(x), _row_stride(x, "x"), ptr(a_stack), int(n_ad), int(rank), int(k),
         ptr(seg_indptr), ptr(seg_adapter), int(seg_adapter.numel()), int(t), ptr(out), _row_stride(out, "down"),
         stream_handle())
    return out


SHRINK_ROWS_MAX_K = 8192


def lora_shrink_rows(x: torch.Tensor, a_stack: torch.Tensor, *, tok_adapter: torch.Tensor | None = None,
                     out: torch.Tensor | None = None, norm_weight: torch.Tensor | None = None,
                     norm_eps: float = 1e-6, xn_out: torch.Tensor | None = None) -> torch.Tensor:
    """down[t] = x[t] . A[tok_adapter[t]]^T (fp32, a_stack [n_adapters, rank,
    in]); with ``norm_weight`` the rows are RMS-normalised first (bit-identical
    to :func:`rmsnorm`) and written to ``xn_out`` when given.  ``in`` <= 8192."""

    _need_cuda(x, a_stack)
    _need(x, torch.bfloat16, "x")
    _need(a_stack, torch.bfloat16, "a_stack")
    if a_stack.dim() == 2:
        a_stack = a_stack.unsqueeze(0)
    if not a_stack.is_contiguous():
        raise ValueError("a_stack must be a contiguous [n_adapters, rank, in] stack")
    n_ad, rank, k = a_stack.shape
    t = x.shape[0]
    if x.shape[1] != k:
        raise ValueError("x and a_stack disagree on the input features")
    if out is None:
        out = torch.empty(t, rank, dtype=torch.float32, device=x.device)
    if tok_adapter is not None:
        _need(tok_adapter, torch.int32, "tok_adapter")
    call("pl_lora_shrink_rows", ptr(x), _row_stride(x, "x"), int(t), int(k), ptr(norm_weight), float(norm_eps),
         ptr(xn_out), 0 if xn_out is None else _row_stride(xn_out, "xn_out"), ptr(a_stack), int(n_ad), int(rank),
         ptr(tok_adapter), ptr(out), _row_stride(out, "down"), stream_handle())
    return out


def _gemv_phase(
    x: torch.Tensor,
    weight: torch.Tensor,
    *,
    bias: torch.Tensor | None = None,
    prologue: int = _capi.PL_PROLOGUE_NONE,
    norm_weight: torch.Tensor | None = None,
    norm_eps: float = 1e-6,
    lora_down: torch.Tensor | None = None,
    lora_b: torch.Tensor | None = None,
    lora_scale: float = 1.0,
    slice_ends: tuple[int, ...] = (),
    tok_adapter: torch.Tensor | None = None,
    residual: torch.Tensor | None = None,
    out: torch.Tensor | None = None,
    shrink_a: torch.Tensor | None = None,
    shrink_out: torch.Tensor | None = None,
    lora_a: torch.Tensor | None = None,
    weights_static: bool = False,
) -> tuple[_capi.GemvPhase, torch.Tensor | None, list]:
    """Checks one fused projection and packs it as a PlGemvPhase; returns the
    phase, the output tensor and the tensors it created (kept alive by the
    caller until the launch is enqueued)."""

    _need_cuda(x, weight)
    _need(x, torch.bfloat16, "x")
    _need(weight, torch.bfloat16, "weight")
    if not weight.is_contiguous():
        raise ValueError("weight must be contiguous [out, in]")
    t = x.shape[0]
    n, k = weight.shape
    keep = []
    if out is None and n > 0:
        out = torch.empty(t, n, dtype=torch.bfloat16, device=x.device)
    rank = 0
    num_slices = 1
    if lora_b is not None:
        if lora_b.dim() == 2:
            lora_b = lora_b.unsqueeze(0)
        rank = lora_b.shape[-1]
        num_slices = len(slice_ends) + 1 if slice_ends else 1
        if num_slices > 4:
            raise ValueError("at most 4 LoRA slices")
    flags = _capi.PL_FLAG_WEIGHTS_STATIC if weights_static else 0
    if lora_a is not None:
        if shrink_a is not None or lora_down is not None or lora_b is None or slice_ends:
            raise ValueError("lora_a replaces lora_down / shrink_a and needs lora_b with one slice")
        if lora_a.dim() == 2:
            lora_a = lora_a.unsqueeze(0)
        if not lora_a.is_contiguous() or lora_a.shape[1] != rank or lora_a.shape[2] != k:
            raise ValueError("lora_a must be a contiguous [n_adapters, rank, in] stack")
        shrink_a, flags = lora_a, flags | _capi.PL_FLAG_DOWN_FROM_X
    n_shrink = 0 if shrink_a is None else shrink_a.shape[0]
    if shrink_a is not None and shrink_out is None and lora_a is None:
        shrink_out = torch.empty(t, n_shrink, dtype=torch.float32, device=x.device)
    keep += [out, shrink_out, lora_b, lora_a]
    ph = _capi.GemvPhase()
    ph.x, ph.x_stride, ph.num_tokens, ph.k_in, ph.prologue = ptr(x), _row_stride(x, "x"), int(t), int(k), int(prologue)
    ph.norm_w, ph.norm_eps, ph.w, ph.n_out, ph.bias = ptr(norm_weight), float(norm_eps), ptr(weight), int(n), ptr(bias)
    ph.lora_down = ptr(lora_down)
    ph.down_stride = 0 if lora_down is None else _row_stride(lora_down, "lora_down")
    ph.lora_b, ph.lora_rank, ph.lora_scale = ptr(lora_b), int(rank), float(lora_scale)
    for i, e in enumerate(slice_ends if lora_b is not None else ()):
        ph.slice_end[i] = int(e)
    ph.num_slices = int(num_slices)
    ph.tok_adapter, ph.residual = ptr(tok_adapter), ptr(residual)
    ph.res_stride = 0 if residual is None else _row_stride(residual, "residual")
    ph.y, ph.y_stride = ptr(out), 0 if out is None else _row_stride(out, "out")
    ph.shrink_a, ph.n_shrink, ph.shrink_out = ptr(shrink_a), int(n_shrink), ptr(shrink_out)
    ph.shrink_stride = 0 if shrink_out is None else _row_stride(shrink_out, "shrink_out")
    ph.flags = int(flags)
    return ph, out, keep


def linear_lora_fused(
    x: torch.Tensor,
    weight: torch.Tensor,
    *,
    status: torch.Tensor | None = None,
    prefetch_next: tuple | None = None,
    prefetch_units: int = 1,
    **kw,
) -> torch.Tensor:
    """y = x . W^T (+bias) (+ LoRA expand) (+ residual) for <= 8 tokens.

    ``x`` is [T, K] (or [T, 2K] for the SiLU-and-mul prologue), ``weight``
    [N, K], ``lora_b`` [n_adapters, N, rank] with scale folded in,
    ``lora_down`` [T, >= num_slices*rank] fp32, ``shrink_a`` [n_shrink, K]
    whose fp32 products go to ``shrink_out`` [T, n_shrink].  With ``lora_a``
    [n_adapters, rank, K] instead of ``lora_down`` the kernel computes the
    down values x . A^T itself (PL_FLAG_DOWN_FROM_X; one LoRA slice).
    Keywords: bias, prologue, norm_weight, norm_eps, lora_down, lora_b,
    lora_scale, slice_ends, tok_adapter, residual, out, shrink_a, shrink_out,
    lora_a, weights_static.
    ``prefetch_next`` = (x, weight, keywords) of the projection launched next
    on the stream: once a CTA has issued its own weight copies it pulls the
    first ``prefetch_units`` ring stages of that launch's rows into L2
    (pl_linear_lora_phase); the results are unchanged.
    """

    ph, out, keep = _gemv_phase(x, weight, **kw)
    if prefetch_next is not None and prefetch_units > 0:
        import ctypes

        nx, nw, nkw = prefetch_next
        _need_cuda(nw)
        n_shrink_a = nkw.get("shrink_a") if nkw.get("lora_a") is None else None
        pf = _capi.GemvPrefetch()
        pf.w, pf.n_out, pf.k_in = ptr(nw), int(nw.shape[0]), int(nw.shape[1])
        pf.shrink_a = ptr(n_shrink_a)
        pf.n_shrink = 0 if n_shrink_a is None else int(n_shrink_a.shape[0])
        pf.num_tokens, pf.units = int(nx.shape[0]), int(prefetch_units)
        call("pl_linear_lora_phase", ctypes.byref(ph), ctypes.byref(pf), ptr(status), stream_handle())
        del keep
        return out
    slice_ptr, slice_keepalive = None, None
    if ph.num_slices > 1:
        slice_ptr, slice_keepalive = ctypes_int32_array(list(ph.slice_end)[: ph.num_slices - 1])
    call("pl_linear_lora_expand_fused", ph.x, ph.x_stride, ph.num_tokens, ph.k_in, ph.prologue, ph.norm_w,
         ph.norm_eps, ph.w, ph.n_out, ph.bias, ph.lora_down, ph.down_stride, ph.lora_b, ph.lora_rank,
         ph.lora_scale, slice_ptr, ph.num_slices, ph.tok_adapter, ph.residual, ph.res_stride, ph.y, ph.y_stride,
         ph.shrink_a, ph.n_shrink, ph.shrink_out, ph.shrink_stride, ph.flags, ptr(status), stream_handle())
    del slice_keepalive, keep
    return out


CHAIN_MAX_PHASES = 6


def linear_lora_chain(phases: list[tuple[torch.Tensor, torch.Tensor, dict]], *, grid_barrier: torch.Tensor | None,
                      status: torch.Tensor | None = None) -> list[torch.Tensor | None]:
    """Consecutive fused projections in one persistent launch
    (pl_linear_lora_chain).  ``phases`` holds (x, weight, keywords of
    linear_lora_fused) per projection; a later phase may read an earlier
    phase's output as its x or residual.  ``grid_barrier``: device int32,
    zero before the first call (left zero by every call that completes).
    Returns each phase's output."""

    if not 1 <= len(phases) <= CHAIN_MAX_PHASES:
        raise ValueError(f"1 to {CHAIN_MAX_PHASES} phases")
    if grid_barrier is not None:
        _need_cuda(grid_barrier)
        _need(grid_barrier, torch.int32, "grid_barrier")
    elif len(phases) > 1:
        raise ValueError("grid_barrier is required for more than one phase")
    arr = (_capi.GemvPhase * len(phases))()
    outs, keep = [], []
    for i, (x, w, kw) in enumerate(phases):
        ph, out, kp = _gemv_phase(x, w, **kw)
        arr[i] = ph
        outs.append(out)
        keep += kp
    call("pl_linear_lora_chain", arr, len(phases), ptr(grid_barrier), ptr(status), stream_handle())
    del keep
    return outs


GEMV_MAX_ROWS = 8
GEMV_MAX_STAGED_BYTES = 96 * 1024  # activations the decode GEMV keeps in shared memory
GEMM_MAX_ROWS = 128


def gemv_fits(rows: int, k_in: int) -> bool:
    """Whether :func:`linear_lora_fused` takes ``rows`` tokens of ``k_in``
    inputs: every row's activations are staged in shared memory."""

    return rows <= GEMV_MAX_ROWS and rows * (2 * k_in + 16) <= GEMV_MAX_STAGED_BYTES


def gemm_plan(num_tokens: int, k_in: int, n_out: int, num_ctas: int = 0) -> _capi.GemmPlan:
    """Work split of :func:`linear_lora_gemm` (``num_ctas`` 0: one CTA per SM)."""

    plan = _capi.GemmPlan()
    call("pl_linear_gemm_plan", int(num_tokens), int(k_in), int(n_out), int(num_ctas), _capi.ctypes.byref(plan))
    return plan


def linear_lora_gemm(
    x: torch.Tensor,
    weight: torch.Tensor,
    *,
    bias: torch.Tensor | None = None,
    lora_down: torch.Tensor | None = None,
    lora_b: torch.Tensor | None = None,
    lora_scale: float = 1.0,
    slice_ends: tuple[int, ...] = (),
    tok_adapter: torch.Tensor | None = None,
    residual: torch.Tensor | None = None,
    out: torch.Tensor | None = None,
    workspace: torch.Tensor | None = None,
    num_ctas: int = 0,
    weights_static: bool = False,
    silu_pairs: bool = False,
    status: torch.Tensor | None = None,
) -> torch.Tensor:
    """y = x . W^T (+bias) (+ per-token LoRA expand) (+ residual) for 1..128
    tokens on the tcgen05 tensor cores.  ``x`` [T, K] is used as given (apply
    :func:`rmsnorm` / :func:`silu_mul` first); the epilogue arguments are those
    of :func:`linear_lora_fused`.  ``workspace`` (uint8, zeroed once) is sized
    by :func:`gemm_plan` for the same ``num_ctas``; one is allocated when
    omitted.  ``silu_pairs``: ``weight`` is a gate/up stack interleaved by
    :func:`interleave_gate_up` and the output [T, N/2] is the SiLU-and-mul of
    the gate and up projections (PL_FLAG_SILU_PAIRS)."""

    _need_cuda(x, weight)
    _need(x, torch.bfloat16, "x")
    _need(weight, torch.bfloat16, "weight")
    if not weight.is_contiguous():
        raise ValueError("weight must be contiguous [out, in]")
    t = x.shape[0]
    n, k = weight.shape
    if out is None:
        out = torch.empty(t, n // 2 if silu_pairs else n, dtype=torch.bfloat16, device=x.device)
    if workspace is None:
        need = int(gemm_plan(t, k, n, num_ctas).workspace_bytes)
        workspace = torch.zeros(need, dtype=torch.uint8, device=x.device)
    rank = 0
    num_slices = 1
    slice_ptr, slice_keepalive = None, None
    if lora_b is not None:
        if lora_b.dim() == 2:
            lora_b = lora_b.unsqueeze(0)
        rank = lora_b.shape[-1]
        num_slices = len(slice_ends) + 1 if slice_ends else 1
        if slice_ends:
            slice_ptr, slice_keepalive = ctypes_int32_array(slice_ends)
    flags = (_capi.PL_FLAG_WEIGHTS_STATIC if weights_static else 0) | (_capi.PL_FLAG_SILU_PAIRS if silu_pairs else 0)
    call("pl_linear_lora_gemm", ptr(x), _row_stride(x, "x"), int(t), int(k), ptr(weight), int(n), ptr(bias),
         ptr(lora_down), 0 if lora_down is None else _row_stride(lora_down, "lora_down"), ptr(lora_b), int(rank),
         float(lora_scale), slice_ptr, int(num_slices), ptr(tok_adapter), ptr(residual),
         0 if residual is None else _row_stride(residual, "residual"), ptr(out), _row_stride(out, "out"),
         int(num_ctas), ptr(workspace), int(workspace.numel()), int(flags), ptr(status), stream_handle())
    del slice_keepalive
    return out


def interleave_gate_up(w_gate_up: torch.Tensor) -> torch.Tensor:
    """[gate; up] rows ([2I, K], I % 64 == 0) reordered into the blocks of
    PL_FLAG_SILU_PAIRS: 64 gate rows, then the same 64 up rows, and so on."""

    n, k = w_gate_up.shape
    i = n // 2
    if n % 2 or i % 64:
        raise ValueError("the gate/up stack needs an even row count with I % 64 == 0")
    g, u = w_gate_up[:i].view(i // 64, 64, k), w_gate_up[i:].view(i // 64, 64, k)
    return torch.stack([g, u], dim=1).reshape(n, k).contiguous()


def rmsnorm(x: torch.Tensor, weight: torch.Tensor, eps: float, out: torch.Tensor | None = None) -> torch.Tensor:
    """FlashInfer-style RMSNorm (one bf16 rounding) over rows of ``x`` [T, K]."""

    _need_cuda(x, weight)
    _need(x, torch.bfloat16, "x")
    _need(weight, torch.bfloat16, "weight")
    if out is None:
        out = torch.empty_like(x)
    call("pl_rmsnorm", ptr(x), _row_stride(x, "x"), int(x.shape[0]), int(x.shape[1]), ptr(weight), float(eps),
         ptr(out), _row_stride(out, "out"), stream_handle())
    return out


def rmsnorm_hf(x: torch.Tensor, weight: torch.Tensor, eps: float, out: torch.Tensor | None = None) -> torch.Tensor:
    """Hugging Face RMSNorm (two bf16 roundings) over rows of ``x`` [R, K]."""

    _need_cuda(x, weight)
    _need(x, torch.bfloat16, "x")
    _need(weight, torch.bfloat16, "weight")
    if out is None:
        out = torch.empty_like(x)
    call("pl_rmsnorm_hf", ptr(x), _row_stride(x, "x"), int(x.shape[0]), int(x.shape[1]), ptr(weight), float(eps),
         ptr(out), _row_stride(out, "out"), stream_handle())
    return out


def silu_mul(x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """bf16(silu(gate) * up) over packed [T, 2K] rows -> [T, K]."""

    _need_cuda(x)
    _need(x, torch.bfloat16, "x")
    t, k2 = x.shape
    if out is None:
        out = torch.empty(t, k2 // 2, dtype=torch.bfloat16, device=x.device)
    call("pl_silu_mul", ptr(x), _row_stride(x, "x"), int(t), int(k2 // 2), ptr(out), _row_stride(out, "out"),
         stream_handle())
    return out


def ctypes_int32_array(values):
    """A host int32 array and its address (keep the array alive across the call)."""

    import ctypes

    arr = (ctypes.c_int32 * len(values))(*[int(v) for v in values])
    return ctypes.cast(arr, ctypes.c_void_p).value, arr


def lora_merge_weight(w_in: torch.Tensor, a: torch.Tensor, b: torch.Tensor, scale: float, *, sign: int = 1,
                      mode: int = 0, out: torch.Tensor | None = None) -> torch.Tensor:
    """w_out = w_in + sign * scale * (B @ A) with the reference's rounding (mode 0/1)."""

    _need_cuda(w_in, a, b)
    for name, t in (("w", w_in), ("a", a), ("b", b)):
        _need(t, torch.bfloat16, name)
        if not t.is_contiguous():
            raise ValueError(f"{name} must be contiguous")
    n, k = w_in.shape
    r = a.shape[0]
    if out is None:
        out = torch.empty_like(w_in)
    call("pl_lora_merge_weight", ptr(w_in), ptr(out), ptr(a), ptr(b), int(n), int(k), int(r), float(scale),
         int(sign), int(mode), stream_handle())
    return out


# ---------------------------------------------------- decode-step glue ops
def kv_append(k: torch.Tensor, v: torch.Tensor, kv_cache: torch.Tensor, page_id: torch.Tensor,
              page_offset: torch.Tensor, status: torch.Tensor | None = None) -> None:
    """Scatter k, v [T, Hkv, D] into the pool at (page_id[t], page_offset[t])."""

    _need_cuda(k, v, kv_cache, page_id, page_offset)
    _need(page_id, torch.int32, "page_id")
    _need(page_offset, torch.int32, "page_offset")
    t, hkv, d = k.shape
    if not (k.stride(-1) == 1 and k.stride(-2) == d and v.stride(-1) == 1 and v.stride(-2) == d):
        raise ValueError("k/v must be [T, Hkv, D] with contiguous heads")
    num_pages, _, page_size, _, _ = kv_cache.shape
    call("pl_kv_append", ptr(k), k.stride(0), ptr(v), v.stride(0), ptr(kv_cache), int(num_pages), ptr(page_id),
         ptr(page_offset), int(t), int(hkv), int(d), int(page_size), ptr(status), stream_handle())


def qkv_rope_append(
    qkv: torch.Tensor,
    *,
    num_qo_heads: int,
    num_kv_heads: int,
    head_dim: int,
    positions: torch.Tensor,
    rope_theta: float,
    kv_cache: torch.Tensor,
    page_id: torch.Tensor,
    page_offset: torch.Tensor,
    q_out: torch.Tensor,
    lora_down: torch.Tensor | None = None,
    lora_b: torch.Tensor | None = None,
    lora_scale: float = 1.0,
    tok_adapter: torch.Tensor | None = None,
    q_norm_weight: torch.Tensor | None = None,
    k_norm_weight: torch.Tensor | None = None,
    norm_eps: float = 1e-6,
    status: torch.Tensor | None = None,
) -> torch.Tensor:
    _need_cuda(qkv, positions, kv_cache, q_out)
    t = qkv.shape[0]
    num_pages, _, page_size, _, _ = kv_cache.shape
    rank = 0
    if lora_b is not None:
        if lora_b.dim() == 2:
            lora_b = lora_b.unsqueeze(0)
        rank = lora_b.shape[-1]
    call("pl_qkv_rope_append", ptr(qkv), _row_stride(qkv, "qkv"), ptr(lora_down),
         0 if lora_down is None else _row_stride(lora_down, "lora_down"), ptr(lora_b), int(rank),
         float(lora_scale), ptr(tok_adapter),
         ptr(q_norm_weight), ptr(k_norm_weight), float(norm_eps), ptr(positions), float(rope_theta), ptr(q_out),
         ptr(kv_cache), int(num_pages), ptr(page_id), ptr(page_offset), int(t), int(num_qo_heads),
         int(num_kv_heads), int(head_dim), int(page_size), ptr(status), stream_handle())
    return q_out


def embed(token_ids: torch.Tensor, table: torch.Tensor, out: torch.Tensor,
          status: torch.Tensor | None = None) -> torch.Tensor:
    _need_cuda(token_ids, table, out)
    _need(token_ids, torch.int64, "token_ids")
    vocab, dim = table.shape
    call("pl_embed", ptr(token_ids), ptr(table), int(vocab), int(dim), int(token_ids.numel()), ptr(out),
         ptr(status), stream_handle())
    return out


def argmax_workspace_bytes(num_tokens: int, max_chunks: int = 1024) -> int:
    return 4 * num_tokens + 8 * num_tokens * max_chunks


def argmax(logits: torch.Tensor, out: torch.Tensor, workspace: torch.Tensor | None = None) -> torch.Tensor:
    """First-index argmax per row (torch.argmax semantics) on up to one CTA per SM.

    ``workspace`` (uint8, zero-initialised once, reusable) holds the per-row
    candidates and arrival tickets; a fresh zeroed one is made if omitted.
    """

    _need_cuda(logits, out)
    _need(logits, torch.bfloat16, "logits")
    _need(out, torch.int64, "out")
    t, vocab = logits.shape
    if workspace is None:
        workspace = torch.zeros(argmax_workspace_bytes(t), dtype=torch.uint8, device=logits.device)
    call("pl_argmax", ptr(logits), _row_stride(logits, "logits"), int(vocab), int(t), ptr(out), ptr(workspace),
         int(workspace.numel()), stream_handle())
    return out
