"""Greedy paged-KV LoRA decode on B200 kernels (the benchmark's decode step).

``DecodeEngine`` runs the decode layer of the reference
(model/flashinfer/layer_runner.py:283-337, cuda_graph.py:245-263) with the
no-merge LoRA delta (packed_ops.py:105-165, multilora/linear.py:200-231) on
this package's kernels, five launches per layer:

  1. linear_lora_fused   RMSNorm -> [W_q;W_k;W_v] and the packed LoRA A rows
  2. paged_decode_qkv    + B.down (packed expand), q/k head norm, RoPE, KV append,
                         then split-KV paged attention with the split merge
                         (thread-block cluster or arrival ticket) in the kernel
  3. linear_lora_fused   attn . A_o^T in the prologue (every CTA), then W_o with
                         the LoRA expand and the residual in the epilogue
  4. linear_lora_fused   RMSNorm -> [W_gate;W_up]
  5. linear_lora_fused   SiLU-and-mul -> W_down with the residual in the epilogue

plus page-table advance + embedding in front and the final norm + lm_head +
argmax behind.  With ``chain_projections`` launches 3-5 and the next
layer's launch 1 (or lm_head) run as one persistent launch
(pl_linear_lora_chain: grid barriers between the projections).  The page table lives on the device and is advanced inside
the step, so one captured CUDA graph serves every context length (the
reference recaptures whenever the page count changes, cuda_graph.py:90).
Consecutive kernels use programmatic dependent launch, so each weight
stream starts while the previous kernel drains.

The prompt is prefilled with torch GEMMs around the sm_100a paged prefill
attention kernel (pl_paged_prefill over the pool pages just written).
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.nn.functional as F

from pagelora_b200 import kernels as K
from pagelora_b200._capi import PL_PROLOGUE_RMSNORM, PL_PROLOGUE_SILU_MUL
from pagelora_b200.synthetic import LoRASpec, ModelSpec


@dataclass
class LayerWeights:
    w_qkv: torch.Tensor          # [q+2kv, H]
    a_qkv: torch.Tensor | None   # [3r, H] packed LoRA A (zero rows for untargeted modules)
    b_qkv: torch.Tensor | None   # [1, q+2kv, r] packed LoRA B * scale
    w_o: torch.Tensor            # [H, q]
    a_o: torch.Tensor | None     # [1, r, q]
    b_o: torch.Tensor | None     # [1, H, r] (* scale)
    w_gate_up: torch.Tensor      # [2I, H]
    w_down: torch.Tensor         # [H, I]
    input_norm: torch.Tensor
    post_norm: torch.Tensor
    q_norm: torch.Tensor | None
    k_norm: torch.Tensor | None


def _rmsnorm_fused(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    xf = x.float()
    r = torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    return (xf * r * w.float()).to(torch.bfloat16)


def _rmsnorm_hf(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    xf = x.float()
    r = torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    return (w.float() * (xf * r).to(torch.bfloat16).float()).to(torch.bfloat16)


def _rope(x: torch.Tensor, pos: torch.Tensor, theta: float) -> torch.Tensor:
    d = x.shape[-1]
    inv = 1.0 / (theta ** (torch.arange(0, d, 2, device=x.device, dtype=torch.float32) / d))
    ang = pos.float()[:, None] * inv[None, :]
    cos, sin = ang.cos()[:, None, :], ang.sin()[:, None, :]
    xf = x.float()
    x1, x2 = xf[..., : d // 2], xf[..., d // 2:]
    return torch.cat([x1 * cos - x2 * sin, x2 * cos + x1 * sin], dim=-1).to(torch.bfloat16)


class DecodeEngine:
    """Single-sequence (batch 1) greedy decoder; weights in Hugging Face naming."""

    def __init__(self, spec: ModelSpec, weights: dict[str, torch.Tensor], *, lora: dict | None = None,
                 lora_spec: LoRASpec | None = None, page_size: int = 16, max_seq_len: int = 4096,
                 num_pages: int | None = None, device: torch.device | str = "cuda") -> None:
        self.spec = spec
        self.device = torch.device(device)
        self.page_size = page_size
        self.lora_rank = lora_spec.rank if (lora and lora_spec) else 0
        self.lora_scale = lora_spec.scale if (lora and lora_spec) else 1.0
        self.qkv_lora_scale = 1.0
        # o projection: the LoRA shrink runs inside the o GEMV's prologue
        # (PL_FLAG_DOWN_FROM_X); False keeps the separate pl_lora_shrink_seg launch
        self.fold_o_shrink = True
        # True: o -> gate_up -> down -> next q/k/v (or lm_head) as one
        # persistent launch (pl_linear_lora_chain, 2 launches per layer
        # instead of 5).  Off by default: inside the CUDA graph the chain's
        # grid barriers cost more than the programmatic launch boundaries
        # they replace (config 2: 3.57 vs 3.37 ms per step); it pays where
        # launches are issued one by one from the host.
        self.chain_projections = False
        # every projection launch pulls the first two ring stages of the next
        # projection's rows (same CTA) into L2 once its own copies are issued
        # (pl_linear_lora_phase); 0 turns the hand-over off
        self.l2_handover_units = 2
        dev, bf = self.device, torch.bfloat16
        H, D = spec.hidden, spec.head_dim

        def take(name: str) -> torch.Tensor:
            return weights.pop(name).to(device=dev, dtype=bf).contiguous()

        self.layers: list[LayerWeights] = []
        for i in range(spec.num_layers):
            p = f"model.layers.{i}."
            wq, wk, wv = take(p + "self_attn.q_proj.weight"), take(p + "self_attn.k_proj.weight"), take(
                p + "self_attn.v_proj.weight")
            w_qkv = torch.cat([wq, wk, wv], 0).contiguous()
            del wq, wk, wv
            a_qkv = b_qkv = a_o = b_o = None
            if self.lora_rank:
                r, sc = lora_spec.rank, lora_spec.scale
                # With LoRA on all of q/k/v the reference packs B * scale into one
                # block-diagonal matrix (packed_ops.py:363-375); otherwise each
                # module's delta is bf16(bf16(down . B^T) * scale) (:534-553).
                packed = all(f"layers.{i}.{t}" in lora for t in "qkv")
                self.qkv_lora_scale = 1.0 if packed else sc
                a_parts, b_parts = [], []
                for t, od in (("q", spec.q_dim), ("k", spec.kv_dim), ("v", spec.kv_dim)):
                    ab = lora.get(f"layers.{i}.{t}")
                    if ab is None:
                        a_parts.append(torch.zeros(r, H, device=dev, dtype=bf))
                        b_parts.append(torch.zeros(od, r, device=dev, dtype=bf))
                    else:
                        a_parts.append(ab[0].to(dev, bf))
                        b_parts.append((ab[1].to(dev, bf) * sc).to(bf) if packed else ab[1].to(dev, bf))
                a_qkv = torch.cat(a_parts, 0).contiguous()
                b_qkv = torch.cat(b_parts, 0).unsqueeze(0).contiguous()
                ab = lora.get(f"layers.{i}.o")
                if ab is not None:  # LoRALinear.forward: scale applied to the rounded product
                    a_o = ab[0].to(dev, bf).unsqueeze(0).contiguous()
                    b_o = ab[1].to(dev, bf).unsqueeze(0).contiguous()
            wg, wu = take(p + "mlp.gate_proj.weight"), take(p + "mlp.up_proj.weight")
            w_gu = torch.cat([wg, wu], 0).contiguous()
            del wg, wu
            self.layers.append(LayerWeights(
                w_qkv=w_qkv, a_qkv=a_qkv, b_qkv=b_qkv, w_o=take(p + "self_attn.o_proj.weight"), a_o=a_o, b_o=b_o,
                w_gate_up=w_gu, w_down=take(p + "mlp.down_proj.weight"),
                input_norm=take(p + "input_layernorm.weight"), post_norm=take(p + "post_attention_layernorm.weight"),
                q_norm=take(p + "self_attn.q_norm.weight") if spec.qk_norm else None,
                k_norm=take(p + "self_attn.k_norm.weight") if spec.qk_norm else None,
            ))
        self.embed = take("model.embed_tokens.weight")
        self.final_norm = take("model.norm.weight")
        self.lm_head = take("lm_head.weight") if "lm_head.weight" in weights else self.embed

        # Paged KV pool [L, P, 2, PS, Hkv, D] and a LIFO free list (paged_kv_allocator.py:42-61).
        self.max_pages_per_row = -(-max_seq_len // page_size)
        self.num_pages = num_pages or self.max_pages_per_row + 4
        self.kv = torch.zeros(spec.num_layers, self.num_pages, 2, page_size, spec.num_kv_heads, D, device=dev,
                              dtype=bf)
        self.free_pages = list(range(self.num_pages))
        # Device page table (one row) and per-step buffers.
        i32 = dict(device=dev, dtype=torch.int32)
        self.row_pages = torch.zeros(1, self.max_pages_per_row, **i32)
        self.row_num_pages = torch.zeros(1, **i32)
        self.last_page_len = torch.zeros(1, **i32)
        self.new_page_ids = torch.zeros(1, **i32)
        self.indptr = torch.zeros(2, **i32)
        self.indices = torch.zeros(self.max_pages_per_row, **i32)
        self.slot_page = torch.zeros(1, **i32)
        self.slot_off = torch.zeros(1, **i32)
        self.positions = torch.zeros(1, **i32)
        self.status = torch.zeros(1, **i32)
        self.chain_barrier = torch.zeros(1, **i32)  # grid barrier of the chained projections
        self.seg_indptr = torch.tensor([0, 1], **i32)
        self.seg_adapter = torch.zeros(1, **i32)
        self.token_buf = torch.zeros(1, device=dev, dtype=torch.int64)
        self.x = torch.zeros(1, H, device=dev, dtype=bf)
        self.qkv = torch.zeros(1, spec.qkv_dim, device=dev, dtype=bf)
        self.down_qkv = torch.zeros(1, 3 * max(self.lora_rank, 1), device=dev, dtype=torch.float32)
        self.q = torch.zeros(1, spec.num_qo_heads, D, device=dev, dtype=bf)
        self.attn = torch.zeros(1, spec.num_qo_heads, D, device=dev, dtype=bf)
        self.down_o = torch.zeros(1, max(self.lora_rank, 1), device=dev, dtype=torch.float32)
        self.gate_up = torch.zeros(1, 2 * spec.intermediate, device=dev, dtype=bf)
        self.logits = torch.zeros(1, spec.vocab, device=dev, dtype=bf)
        self.argmax_ws = torch.zeros(K.argmax_workspace_bytes(1), device=dev, dtype=torch.uint8)
        self.rope_cs = torch.zeros(1, D // 2, 2, device=dev, dtype=torch.float32)
        self.num_splits = 1
        self.workspace = torch.zeros(1 << 20, device=dev, dtype=torch.uint8)
        # Host mirror of the row state (decides when a new page is needed).
        self.host_pages: list[int] = []
        self.host_last = 0
        self.graph: torch.cuda.CUDAGraph | None = None
        self.pinned_page = torch.zeros(1, dtype=torch.int32, pin_memory=True)
        self.pinned_token = torch.zeros(1, dtype=torch.int64, pin_memory=True)

    # ------------------------------------------------------------ planning
    def plan(self, expected_pages: int) -> None:
        """Split-KV plan for this context length (fixed for the captured graph)."""

        s = self.spec
        p = K.decode_plan(1, s.num_qo_heads, s.num_kv_heads, s.head_dim, self.page_size, expected_pages)
        if p.workspace_bytes > self.workspace.numel():
            self.workspace = torch.zeros(int(p.workspace_bytes), device=self.device, dtype=torch.uint8)
            self.graph = None
        if int(p.num_splits) != self.num_splits:
            self.num_splits = int(p.num_splits)
            self.graph = None  # the split count is baked into the captured launches

    # ------------------------------------------------------------- prefill
    @torch.no_grad()
    def reset(self) -> None:
        self.free_pages = list(range(self.num_pages))
        self.host_pages, self.host_last = [], 0
        self.row_num_pages.zero_()
        self.last_page_len.zero_()
        self.status.zero_()

    def _alloc_page(self) -> int:
        if not self.free_pages:
            raise RuntimeError("paged KV pool exhausted")
        return self.free_pages.pop()

    @torch.no_grad()
    def prefill(self, prompt: list[int]) -> int:
        """Prefill the prompt into fresh pages (torch GEMMs, the paged prefill
        attention kernel over the pool); returns the first greedy token."""

        s = self.spec
        self.reset()
        n = len(prompt)
        pages = [self._alloc_page() for _ in range(-(-n // self.page_size))]
        self.host_pages, self.host_last = list(pages), n - (len(pages) - 1) * self.page_size
        ids = torch.tensor(prompt, device=self.device, dtype=torch.int64)
        pos = torch.arange(n, device=self.device)
        page_of = torch.tensor(pages, device=self.device, dtype=torch.int32)[pos // self.page_size]
        off_of = (pos % self.page_size).to(torch.int32)
        x = self.embed[ids]
        i32 = dict(device=self.device, dtype=torch.int32)
        pf_qo = torch.tensor([0, n], **i32)
        pf_kvp = torch.tensor([0, len(pages)], **i32)
        pf_idx = torch.tensor(pages, **i32)
        pf_last = torch.tensor([self.host_last], **i32)
        for li, L in enumerate(self.layers):
            h = _rmsnorm_fused(x, L.input_norm, s.rms_eps)
            qkv = F.linear(h, L.w_qkv)
            if L.a_qkv is not None:
                down = F.linear(h, L.a_qkv)
                r = self.lora_rank
                deltas = []
                off = 0
                for j, od in enumerate((s.q_dim, s.kv_dim, s.kv_dim)):
                    dj = F.linear(down[:, j * r:(j + 1) * r], L.b_qkv[0, off:off + od])
                    deltas.append(dj if self.qkv_lora_scale == 1.0 else dj * self.qkv_lora_scale)
                    off += od
                qkv = qkv + torch.cat(deltas, -1)
            q = qkv[:, : s.q_dim].view(n, s.num_qo_heads, s.head_dim)
            k = qkv[:, s.q_dim: s.q_dim + s.kv_dim].view(n, s.num_kv_heads, s.head_dim)
            v = qkv[:, s.q_dim + s.kv_dim:].reshape(n, s.num_kv_heads, s.head_dim).contiguous()
            if L.q_norm is not None:
                q = _rmsnorm_hf(q, L.q_norm, s.rms_eps)
                k = _rmsnorm_hf(k, L.k_norm, s.rms_eps)
            q = _rope(q, pos, s.rope_theta)
            k = _rope(k, pos, s.rope_theta).contiguous()
            K.kv_append(k, v, self.kv[li], page_of, off_of, status=self.status)
            # causal paged prefill over the pages just written (tcgen05 kernel)
            attn = K.paged_prefill(q, self.kv[li], pf_qo, pf_kvp, pf_idx, pf_last, status=self.status)
            attn = attn.reshape(n, s.q_dim)
            o = F.linear(attn, L.w_o)
            if L.a_o is not None:
                o = o + F.linear(F.linear(attn, L.a_o[0]), L.b_o[0]) * self.lora_scale
            x = x + o
            h2 = _rmsnorm_fused(x, L.post_norm, s.rms_eps)
            gu = F.linear(h2, L.w_gate_up)
            g, u = gu[:, : s.intermediate].float(), gu[:, s.intermediate:].float()
            act = (g / (1.0 + torch.exp(-g)) * u).to(torch.bfloat16)
            x = x + F.linear(act, L.w_down)
        logits = F.linear(_rmsnorm_fused(x[-1:], self.final_norm, s.rms_eps), self.lm_head)
        self.prefill_logits = logits[0]
        first = int(torch.argmax(logits[0]).item())
        # Device row state: pages of the prompt; the decode step appends after them.
        self.row_pages.zero_()
        self.row_pages[0, : len(pages)] = page_of.new_tensor(pages)
        self.row_num_pages.fill_(len(pages))
        self.last_page_len.fill_(self.host_last)
        self.token_buf.fill_(first)
        self.plan(len(pages) + 1)
        self._check_status()
        return first

    # --------------------------------------------------------- decode step
    def _host_reserve(self) -> int:
        """Host side of one token's slot reservation: a new page id when needed."""

        if not self.host_pages or self.host_last >= self.page_size:
            page = self._alloc_page()
            self.host_pages.append(page)
            self.host_last = 1
            return page
        self.host_last += 1
        return -1

    def _decode_body(self) -> None:
        """All launches of one decode step (captured into the graph)."""

        s = self.spec
        st = self.status
        K.page_table_advance(self.row_num_pages, self.last_page_len, self.row_pages, self.new_page_ids,
                             self.page_size, self.indptr, self.indices, self.slot_page, self.slot_off,
                             self.positions, st)
        # the step's RoPE angles, read by every layer's attention launch
        K.rope_cos_sin(self.positions, s.head_dim, s.rope_theta, out=self.rope_cs)
        K.embed(self.token_buf, self.embed, self.x, st)
        attn2d = self.attn.view(1, s.q_dim)

        def qkv_phase(L: LayerWeights) -> tuple:
            return (self.x, L.w_qkv, dict(prologue=PL_PROLOGUE_RMSNORM, norm_weight=L.input_norm,
                                          norm_eps=s.rms_eps, out=self.qkv, shrink_a=L.a_qkv,
                                          shrink_out=self.down_qkv if L.a_qkv is not None else None,
                                          weights_static=True))

        def o_phase(L: LayerWeights) -> tuple:
            if self.fold_o_shrink and L.a_o is not None:
                # the o GEMV computes attn . A_o^T in its prologue: no shrink launch
                return (attn2d, L.w_o, dict(lora_a=L.a_o, lora_b=L.b_o, lora_scale=self.lora_scale,
                                            residual=self.x, out=self.x, weights_static=True))
            return (attn2d, L.w_o, dict(lora_down=self.down_o if L.b_o is not None else None, lora_b=L.b_o,
                                        lora_scale=self.lora_scale, residual=self.x, out=self.x,
                                        weights_static=True))

        def mlp_phases(L: LayerWeights) -> list:
            return [(self.x, L.w_gate_up, dict(prologue=PL_PROLOGUE_RMSNORM, norm_weight=L.post_norm,
                                               norm_eps=s.rms_eps, out=self.gate_up, weights_static=True)),
                    (self.gate_up, L.w_down, dict(prologue=PL_PROLOGUE_SILU_MUL, residual=self.x, out=self.x,
                                                  weights_static=True))]

        head = (self.x, self.lm_head, dict(prologue=PL_PROLOGUE_RMSNORM, norm_weight=self.final_norm,
                                           norm_eps=s.rms_eps, out=self.logits, weights_static=True))
        # every projection of the step in launch order (attention in between)
        proj = [qkv_phase(self.layers[0])]
        for li, L in enumerate(self.layers):
            proj += [o_phase(L)] + mlp_phases(L) + [qkv_phase(self.layers[li + 1]) if li + 1 < len(self.layers)
                                                    else head]

        def launch(i: int) -> None:
            x_, w_, kw_ = proj[i]
            nxt = proj[i + 1] if i + 1 < len(proj) and self.l2_handover_units > 0 else None
            K.linear_lora_fused(x_, w_, status=st, prefetch_next=nxt, prefetch_units=self.l2_handover_units, **kw_)

        launch(0)
        for li, L in enumerate(self.layers):
            # q/k head norm + RoPE + KV append + paged decode: one launch
            K.paged_decode_qkv(self.qkv, self.kv[li], self.indptr, self.indices, self.last_page_len,
                               num_qo_heads=s.num_qo_heads, num_kv_heads=s.num_kv_heads, positions=self.positions,
                               rope_theta=s.rope_theta, slot_page=self.slot_page, slot_offset=self.slot_off,
                               num_splits=self.num_splits, workspace=self.workspace,
                               lora_down=self.down_qkv if L.b_qkv is not None else None, lora_b=L.b_qkv,
                               lora_scale=self.qkv_lora_scale, q_norm_weight=L.q_norm, k_norm_weight=L.k_norm,
                               norm_eps=s.rms_eps, out=self.attn, status=st, rope_cos_sin=self.rope_cs)
            if not (self.fold_o_shrink and L.a_o is not None) and L.a_o is not None:
                K.lora_shrink_seg(attn2d, L.a_o, self.seg_indptr, self.seg_adapter, out=self.down_o)
            base = 1 + 4 * li
            if self.chain_projections:
                K.linear_lora_chain(proj[base:base + 4], grid_barrier=self.chain_barrier, status=st)
            else:
                for i in range(base, base + 4):
                    launch(i)
        K.argmax(self.logits, self.token_buf, self.argmax_ws)

    def launches_per_step(self) -> int:
        shrink = sum(1 for L in self.layers[:1] if L.a_o is not None and not self.fold_o_shrink)
        per_layer = 1 + shrink + (1 if self.chain_projections else 4)
        return 3 + 1 + per_layer * len(self.layers) + 1

    def capture(self) -> None:
        """Capture one decode step into a CUDA graph (after an eager warm-up
        that also sets kernel attributes and caches tensor maps)."""

        stream = torch.cuda.Stream(device=self.device)
        stream.wait_stream(torch.cuda.current_stream(self.device))
        # Warm up on a scratch copy of the mutable row state so no token is consumed.
        saved = [t.clone() for t in (self.row_num_pages, self.last_page_len, self.row_pages, self.token_buf)]
        kv_backup_slot = None
        with torch.cuda.stream(stream):
            self.new_page_ids.fill_(self.free_pages[-1] if self.free_pages else 0)
            self._decode_body()
        torch.cuda.current_stream(self.device).wait_stream(stream)
        torch.cuda.synchronize(self.device)
        for dst, src in zip((self.row_num_pages, self.last_page_len, self.row_pages, self.token_buf), saved):
            dst.copy_(src)
        del kv_backup_slot
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            self._decode_body()
        torch.cuda.synchronize(self.device)
        self.graph = g

    def step_device(self) -> None:
        """One decode step with inputs already on the device (graph replay);
        the host only supplies the next page id through new_page_ids."""

        page = self._host_reserve()
        if page >= 0:
            self.new_page_ids.fill_(page)
        if self.graph is not None:
            self.graph.replay()
        else:
            self._decode_body()

    def step_host(self, token: int) -> int:
        """One decode step driven from host memory: H2D of the step inputs
        (token id, page id) from pinned buffers, replay, D2H of the next id."""

        page = self._host_reserve()
        self.pinned_page[0] = page if page >= 0 else 0
        self.pinned_token[0] = token
        self.new_page_ids.copy_(self.pinned_page, non_blocking=True)
        self.token_buf.copy_(self.pinned_token, non_blocking=True)
        if self.graph is not None:
            self.graph.replay()
        else:
            self._decode_body()
        self.pinned_token.copy_(self.token_buf, non_blocking=True)
        torch.cuda.current_stream(self.device).synchronize()
        return int(self.pinned_token[0])

    def _check_status(self) -> None:
        code = int(self.status.item())
        if code != 0:
            from pagelora_b200._capi import status_string

            raise RuntimeError(f"device status {code}: {status_string(code)}")

    @torch.no_grad()
    def generate(self, prompt: list[int], max_new_tokens: int, *, use_graph: bool = True) -> list[int]:
        """Greedy generation (ignore_eos): prefill, then decode steps."""

        first = self.prefill(prompt)
        out = [first]
        if max_new_tokens > 1 and use_graph:
            self.capture()
        while len(out) < max_new_tokens:
            out.append(self.step_host(out[-1]))
        self._check_status()
        return out
