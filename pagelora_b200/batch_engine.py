"""Batched multi-adapter decode on the B200 kernels (many sequences, one step).

The batched counterpart of :class:`pagelora_b200.engine.DecodeEngine`: B rows
decode one token each per step, every row with its own context length, pages
anywhere in the pool, and its own LoRA adapter.  It is the shape of the
reference's batched graph runner (model/flashinfer/cuda_graph.py:118-543,
``FlashInferBatchDecodeCudaGraphRunner``) over the batched layer
(model/flashinfer/layer_runner.py:338-396) with the multi-adapter serving
path of multilora (one adapter per row, segment-grouped shrink).

One decode step (captured once into a CUDA graph, every launch PDL-chained):

    page_table_advance (all rows) -> embed
    per layer:  rmsnorm -> LoRA-A shrink (segments by adapter) -> q/k/v projection
                -> q/k norm + RoPE + paged KV append (+ per-row LoRA-B expand)
                -> paged decode -> o shrink -> o projection (+ per-row LoRA-B, residual)
                -> rmsnorm -> gate_up projection -> SiLU-mul -> down projection (+ residual)
    rmsnorm -> lm_head -> argmax (per row)

Projections go to the tcgen05 GEMM (:func:`kernels.linear_lora_gemm`) for
more than 8 rows and to the fused decode GEMV (norm / SiLU-mul prologue in
the kernel) for up to 8.  Rows must be ordered by adapter so the shrink sees
one segment per adapter.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

from pagelora_b200 import kernels as K
from pagelora_b200._capi import PL_PROLOGUE_RMSNORM, PL_PROLOGUE_SILU_MUL
from pagelora_b200.engine import _rmsnorm_fused, _rmsnorm_hf, _rope
from pagelora_b200.split_kv import shard_row
from pagelora_b200.synthetic import LoRASpec, ModelSpec

GEMV_MAX_ROWS = K.GEMV_MAX_ROWS


def uses_gemv(rows: int, k_in: int) -> bool:
    """Whether a projection of `rows` tokens and K = k_in runs on the fused
    decode GEMV (all rows' activations staged in shared memory) rather than
    the tcgen05 GEMM."""

    return K.gemv_fits(rows, k_in)


class BatchDecodeEngine:
    """Greedy decoder for B rows with per-row adapters; weights in Hugging Face naming.

    ``adapters`` is a list of LoRA weight dicts ({"layers.{i}.{q|k|v|o}": (A, B)}),
    ``row_adapter[r]`` the adapter of row r (-1: base model only); rows are
    grouped by adapter (non-decreasing ids, base rows first).
    """

    def __init__(self, spec: ModelSpec, weights: dict[str, torch.Tensor], *, adapters: list[dict] | None,
                 lora_spec: LoRASpec | None, row_adapter: list[int], page_size: int = 16, max_context: int = 4096,
                 num_pages: int | None = None, device: torch.device | str = "cuda",
                 kv_shard: tuple[int, int] = (0, 1), group=None, exchange: str = "nccl") -> None:
        self.spec = spec
        # Split-KV: shard `rank` of `world` holds a contiguous page range of
        # every row's context; the last shard owns the growing tail.
        self.shard, self.world = int(kv_shard[0]), int(kv_shard[1])
        if not 0 <= self.shard < self.world:
            raise ValueError("kv_shard must be (rank, world) with 0 <= rank < world")
        self.group = group
        self.owner = self.shard == self.world - 1
        # Split-KV partial exchange: "nccl" (all-gather + merge launch), "p2p"
        # (pl_splitkv_exchange_merge over NVLink peer memory) or "auto" (p2p,
        # and nccl on every rank when the peer mappings fail on any rank)
        if exchange not in ("nccl", "p2p", "auto"):
            raise ValueError("exchange must be 'nccl', 'p2p' or 'auto'")
        self.exchange = exchange
        self.peer = None
        self.device = torch.device(device)
        self.page_size = page_size
        self.rows = len(row_adapter)
        # gate_up and down both on the tcgen05 GEMM: the gate/up weights are
        # stored interleaved in blocks of 64 rows and the gate_up launch writes
        # the SiLU-and-mul directly (PL_FLAG_SILU_PAIRS), one launch fewer
        self.silu_pairs = (not uses_gemv(self.rows, spec.hidden) and not uses_gemv(self.rows, spec.intermediate)
                           and spec.intermediate % 64 == 0)
        if any(b < a for a, b in zip(row_adapter, row_adapter[1:])):
            raise ValueError("rows must be grouped by adapter (non-decreasing adapter ids)")
        n_ad = len(adapters) if adapters else 0
        if any(a >= n_ad for a in row_adapter):
            raise ValueError("row_adapter names an adapter that was not given")
        self.row_adapter = list(row_adapter)
        self.lora_rank = lora_spec.rank if (adapters and lora_spec) else 0
        self.lora_scale = lora_spec.scale if (adapters and lora_spec) else 1.0
        self.qkv_lora_scale = 1.0
        dev, bf = self.device, torch.bfloat16
        H, D, B = spec.hidden, spec.head_dim, self.rows

        def take(name: str) -> torch.Tensor:
            return weights.pop(name).to(device=dev, dtype=bf).contiguous()

        self.layers = []
        for i in range(spec.num_layers):
            p = f"model.layers.{i}."
            w_qkv = torch.cat([take(p + f"self_attn.{m}_proj.weight") for m in "qkv"], 0).contiguous()
            L = dict(w_qkv=w_qkv, w_o=take(p + "self_attn.o_proj.weight"),
                     w_gate_up=self._gate_up(torch.cat([take(p + "mlp.gate_proj.weight"),
                                                        take(p + "mlp.up_proj.weight")], 0)),
                     w_down=take(p + "mlp.down_proj.weight"), input_norm=take(p + "input_layernorm.weight"),
                     post_norm=take(p + "post_attention_layernorm.weight"),
                     q_norm=take(p + "self_attn.q_norm.weight") if spec.qk_norm else None,
                     k_norm=take(p + "self_attn.k_norm.weight") if spec.qk_norm else None,
                     a_qkv=None, b_qkv=None, a_o=None, b_o=None)
            if self.lora_rank:
                r, sc = lora_spec.rank, lora_spec.scale
                packed = all(f"layers.{i}.{t}" in adapters[0] for t in "qkv")
                self.qkv_lora_scale = 1.0 if packed else sc
                a_st, b_st, ao_st, bo_st = [], [], [], []
                for ad in adapters:
                    a_parts, b_parts = [], []
                    for t, od in (("q", spec.q_dim), ("k", spec.kv_dim), ("v", spec.kv_dim)):
                        ab = ad.get(f"layers.{i}.{t}")
                        if ab is None:
                            a_parts.append(torch.zeros(r, H, device=dev, dtype=bf))
                            b_parts.append(torch.zeros(od, r, device=dev, dtype=bf))
                        else:
                            a_parts.append(ab[0].to(dev, bf))
                            b_parts.append((ab[1].to(dev, bf) * sc).to(bf) if packed else ab[1].to(dev, bf))
                    a_st.append(torch.cat(a_parts, 0))
                    b_st.append(torch.cat(b_parts, 0))
                    ab = ad.get(f"layers.{i}.o")
                    ao_st.append(ab[0].to(dev, bf) if ab is not None else torch.zeros(r, spec.q_dim, device=dev,
                                                                                     dtype=bf))
                    bo_st.append(ab[1].to(dev, bf) if ab is not None else torch.zeros(H, r, device=dev, dtype=bf))
                L["a_qkv"] = torch.stack(a_st).contiguous()    # [n_ad, 3r, H]
                L["b_qkv"] = torch.stack(b_st).contiguous()    # [n_ad, qkv_dim, r]
                L["a_o"] = torch.stack(ao_st).contiguous()     # [n_ad, r, q_dim]
                L["b_o"] = torch.stack(bo_st).contiguous()     # [n_ad, H, r]
            self.layers.append(L)
        self.embed = take("model.embed_tokens.weight")
        self.final_norm = take("model.norm.weight")
        self.lm_head = take("lm_head.weight") if "lm_head.weight" in weights else self.embed

        # Paged KV pool [L, P, 2, PS, Hkv, D] and per-row device page tables.
        self.max_pages_per_row = -(-max_context // page_size) + 1
        self.num_pages = num_pages or B * self.max_pages_per_row + 4
        self.kv = torch.zeros(spec.num_layers, self.num_pages, 2, page_size, spec.num_kv_heads, D, device=dev,
                              dtype=bf)
        self.free_pages = list(range(self.num_pages))
        i32 = dict(device=dev, dtype=torch.int32)
        self.row_pages = torch.zeros(B, self.max_pages_per_row, **i32)
        self.row_num_pages = torch.zeros(B, **i32)
        self.last_page_len = torch.zeros(B, **i32)
        self.new_page_ids = torch.zeros(B, **i32)
        self.indptr = torch.zeros(B + 1, **i32)
        self.indices = torch.zeros(B * self.max_pages_per_row, **i32)
        self.slot_page = torch.zeros(B, **i32)
        self.slot_off = torch.zeros(B, **i32)
        self.positions = torch.zeros(B, **i32)
        self.status = torch.zeros(1, **i32)
        self.tok_adapter = torch.tensor(self.row_adapter, **i32)
        segs = [0]
        seg_ad = []
        for r in range(B):
            if r == 0 or self.row_adapter[r] != self.row_adapter[r - 1]:
                if r:
                    segs.append(r)
                seg_ad.append(self.row_adapter[r])
        segs.append(B)
        self.seg_indptr = torch.tensor(segs, **i32)
        self.seg_adapter = torch.tensor(seg_ad, **i32)
        self.token_buf = torch.zeros(B, device=dev, dtype=torch.int64)
        r = max(self.lora_rank, 1)
        self.x = torch.zeros(B, H, device=dev, dtype=bf)
        self.xn = torch.zeros(B, H, device=dev, dtype=bf)
        self.qkv = torch.zeros(B, spec.qkv_dim, device=dev, dtype=bf)
        self.down_qkv = torch.zeros(B, 3 * r, device=dev, dtype=torch.float32)
        self.q = torch.zeros(B, spec.num_qo_heads, D, device=dev, dtype=bf)
        self.attn = torch.zeros(B, spec.num_qo_heads, D, device=dev, dtype=bf)
        self.down_o = torch.zeros(B, r, device=dev, dtype=torch.float32)
        self.gate_up = torch.zeros(B, 2 * spec.intermediate, device=dev, dtype=bf)
        self.act = torch.zeros(B, spec.intermediate, device=dev, dtype=bf)
        self.logits = torch.zeros(B, spec.vocab, device=dev, dtype=bf)
        self.argmax_ws = torch.zeros(K.argmax_workspace_bytes(B), device=dev, dtype=torch.uint8)
        ws = 256
        for n, k in ((spec.qkv_dim, H), (H, spec.q_dim), (2 * spec.intermediate, H), (H, spec.intermediate),
                     (spec.vocab, H)):
            if not uses_gemv(B, k):
                ws = max(ws, int(K.gemm_plan(B, k, n).workspace_bytes))
        self.gemm_ws = torch.zeros(ws, device=dev, dtype=torch.uint8)
        self.rope_cs = torch.zeros(B, spec.head_dim // 2, 2, device=dev, dtype=torch.float32)
        self.num_splits = 1
        self.workspace = torch.zeros(1 << 20, device=dev, dtype=torch.uint8)
        if self.world > 1:
            # One packed [O fp32 | LSE] partial per shard, all-gathered each layer.
            rows_h = B * spec.num_qo_heads
            self.part = torch.zeros(rows_h * (D + 1), device=dev, dtype=torch.float32)
            self.gathered = torch.zeros(self.world, rows_h * (D + 1), device=dev, dtype=torch.float32)
            self.dummy_page = self._alloc_page()  # append target of the shards that do not own the tail
            if exchange in ("p2p", "auto"):
                from pagelora_b200.peer_exchange import PeerExchange, PeerExchangeUnavailable

                try:
                    self.peer = PeerExchange(rows_h, D, group=group, device=dev)
                    self.exchange = "p2p"
                except PeerExchangeUnavailable:
                    if exchange == "p2p":
                        raise
                    self.exchange = "nccl"
        self.host_pages: list[list[int]] = [[] for _ in range(B)]
        self.host_last = [0] * B
        self.context_len = [0] * B
        self.cascade = None  # shared-prefix decode (branch batches)
        self.prefix_len = 0
        self.graph: torch.cuda.CUDAGraph | None = None
        self.pinned_pages = torch.zeros(B, dtype=torch.int32, pin_memory=True)
        self.pinned_tokens = torch.zeros(B, dtype=torch.int64, pin_memory=True)

    # ------------------------------------------------------------ planning
    def plan(self) -> None:
        """Split-KV plan for the current contexts (fixed in the captured graph)."""

        s = self.spec
        total = sum(len(p) for p in self.host_pages) + self.rows
        p = K.decode_plan(self.rows, s.num_qo_heads, s.num_kv_heads, s.head_dim, self.page_size, total)
        if p.workspace_bytes > self.workspace.numel():
            self.workspace = torch.zeros(int(p.workspace_bytes), device=self.device, dtype=torch.uint8)
            self.graph = None
        if int(p.num_splits) != self.num_splits:
            self.num_splits = int(p.num_splits)
            self.graph = None

    def _alloc_page(self) -> int:
        if not self.free_pages:
            raise RuntimeError("paged KV pool exhausted")
        return self.free_pages.pop()

    def shuffle_free_pages(self, seed: int) -> None:
        """Randomly permute the free list (pages land anywhere in the pool)."""

        g = torch.Generator().manual_seed(seed)
        perm = torch.randperm(len(self.free_pages), generator=g).tolist()
        self.free_pages = [self.free_pages[i] for i in perm]

    # ------------------------------------------------------------- prefill
    def _sync_rows(self) -> None:
        self.row_pages.zero_()
        for r in range(self.rows):
            if self.host_pages[r]:
                self.row_pages[r, : len(self.host_pages[r])] = torch.tensor(self.host_pages[r], dtype=torch.int32)
        self.row_num_pages.copy_(torch.tensor([len(p) for p in self.host_pages], dtype=torch.int32))
        self.last_page_len.copy_(torch.tensor(self.host_last, dtype=torch.int32))
        if self.world > 1:
            # Global position of each row's next token (every shard applies RoPE to it).
            self.positions.copy_(torch.tensor([n - 1 for n in self.context_len], dtype=torch.int32))
            if not self.owner:
                # Static page table of this shard; the new token's K/V go to the dummy page.
                indptr = [0]
                for pgs in self.host_pages:
                    indptr.append(indptr[-1] + len(pgs))
                self.indptr.copy_(torch.tensor(indptr, dtype=torch.int32))
                flat = [p for pgs in self.host_pages for p in pgs]
                if flat:
                    self.indices[: len(flat)] = torch.tensor(flat, dtype=torch.int32)
                self.slot_page.fill_(self.dummy_page)
                self.slot_off.zero_()

    def _own_pages(self, pages: list[int], n_tokens: int) -> tuple[list[int], list[int], int]:
        """Split a row's pages between shards: (kept, released, tokens in the
        kept last page)."""

        p0, p1, last = shard_row(n_tokens, self.page_size, self.shard, self.world)
        return pages[p0:p1], pages[:p0] + pages[p1:], last

    @torch.no_grad()
    def _forward_prompt(self, prompt: list[int], ad: int, page_of: torch.Tensor, off_of: torch.Tensor,
                        keep: torch.Tensor | None = None) -> torch.Tensor:
        """Forward of one row's whole prompt with adapter `ad` (torch GEMMs,
        the paged prefill attention kernel); writes
        the K/V of position i to (page_of[i], off_of[i]) for the positions in
        `keep` (all when None) and returns the last position's logits."""

        s = self.spec
        n = len(prompt)
        ids = torch.tensor(prompt, device=self.device, dtype=torch.int64)
        pos = torch.arange(n, device=self.device)
        x = self.embed[ids]
        # The row's K/V are not always one page list of this pool (a split-KV
        # shard keeps its range only; a shared prefix may end mid-page), so
        # each layer's K/V also go to a scratch pool of the row's own pages,
        # over which the paged prefill kernel attends.
        ps = self.page_size
        npg = -(-n // ps)
        i32 = dict(device=self.device, dtype=torch.int32)
        scratch = torch.empty((npg, 2, ps) + tuple(self.kv.shape[-2:]), device=self.device, dtype=torch.bfloat16)
        s_page, s_off = (pos // ps).to(torch.int32), (pos % ps).to(torch.int32)
        pf_qo = torch.tensor([0, n], **i32)
        pf_kvp = torch.tensor([0, npg], **i32)
        pf_idx = torch.arange(npg, **i32)
        pf_last = torch.tensor([n - (npg - 1) * ps], **i32)
        for li, L in enumerate(self.layers):
            h = _rmsnorm_fused(x, L["input_norm"], s.rms_eps)
            qkv = F.linear(h, L["w_qkv"])
            if ad >= 0 and L["a_qkv"] is not None:
                down = F.linear(h, L["a_qkv"][ad])
                rk = self.lora_rank
                deltas, off = [], 0
                for j, od in enumerate((s.q_dim, s.kv_dim, s.kv_dim)):
                    dj = F.linear(down[:, j * rk:(j + 1) * rk], L["b_qkv"][ad, off:off + od])
                    deltas.append(dj if self.qkv_lora_scale == 1.0 else dj * self.qkv_lora_scale)
                    off += od
                qkv = qkv + torch.cat(deltas, -1)
            q = qkv[:, : s.q_dim].view(n, s.num_qo_heads, s.head_dim)
            k = qkv[:, s.q_dim: s.q_dim + s.kv_dim].view(n, s.num_kv_heads, s.head_dim)
            v = qkv[:, s.q_dim + s.kv_dim:].reshape(n, s.num_kv_heads, s.head_dim).contiguous()
            if L["q_norm"] is not None:
                q = _rmsnorm_hf(q, L["q_norm"], s.rms_eps)
                k = _rmsnorm_hf(k, L["k_norm"], s.rms_eps)
            q = _rope(q, pos, s.rope_theta)
            k = _rope(k, pos, s.rope_theta).contiguous()
            if keep is None:
                K.kv_append(k, v, self.kv[li], page_of, off_of, status=self.status)
            elif keep.numel():
                K.kv_append(k[keep].contiguous(), v[keep].contiguous(), self.kv[li], page_of[keep].contiguous(),
                            off_of[keep].contiguous(), status=self.status)
            K.kv_append(k, v, scratch, s_page, s_off, status=self.status)
            attn = K.paged_prefill(q, scratch, pf_qo, pf_kvp, pf_idx, pf_last, status=self.status)
            attn = attn.reshape(n, s.q_dim)
            o = F.linear(attn, L["w_o"])
            if ad >= 0 and L["a_o"] is not None:
                o = o + F.linear(F.linear(attn, L["a_o"][ad]), L["b_o"][ad]) * self.lora_scale
            x = x + o
            h2 = _rmsnorm_fused(x, L["post_norm"], s.rms_eps)
            gu = F.linear(h2, L["w_gate_up"])
            if self.silu_pairs:  # interleaved rows: blocks of 64 gate outputs, then 64 up outputs
                gu = gu.view(n, s.intermediate // 64, 2, 64)
                g, u = gu[:, :, 0].reshape(n, -1).float(), gu[:, :, 1].reshape(n, -1).float()
            else:
                g, u = gu[:, : s.intermediate].float(), gu[:, s.intermediate:].float()
            x = x + F.linear((g / (1.0 + torch.exp(-g)) * u).to(torch.bfloat16), L["w_down"])
        return F.linear(_rmsnorm_fused(x[-1:], self.final_norm, s.rms_eps), self.lm_head)[0]

    @torch.no_grad()
    def prefill(self, prompts: list[list[int]]) -> list[int]:
        """Prefill every row's prompt (torch ops, each row with its adapter);
        returns each row's first greedy token."""

        if len(prompts) != self.rows:
            raise ValueError("one prompt per row")
        firsts = []
        self.prefill_logits = []
        for r, prompt in enumerate(prompts):
            n = len(prompt)
            pages = [self._alloc_page() for _ in range(-(-n // self.page_size))]
            self.host_pages[r], self.host_last[r] = list(pages), n - (len(pages) - 1) * self.page_size
            pos = torch.arange(n, device=self.device)
            page_of = torch.tensor(pages, device=self.device, dtype=torch.int32)[pos // self.page_size]
            off_of = (pos % self.page_size).to(torch.int32)
            logits = self._forward_prompt(prompt, self.row_adapter[r], page_of, off_of)
            self.prefill_logits.append(logits)
            firsts.append(int(torch.argmax(logits).item()))
        self.context_len = [len(p) for p in prompts]
        if self.world > 1:
            for r, n in enumerate(self.context_len):
                kept, released, last = self._own_pages(self.host_pages[r], n)
                self.host_pages[r], self.host_last[r] = kept, last
                self.free_pages.extend(released)
        self._sync_rows()
        self.token_buf.copy_(torch.tensor(firsts, dtype=torch.int64))
        self.plan()
        self._check_status()
        return firsts

    @torch.no_grad()
    def fill_random_context(self, lengths: list[int], *, seed: int = 0) -> None:
        """Give row r a context of lengths[r] tokens whose K/V are random
        N(0, 1) values (a stand-in for prefill when only the decode step is
        measured); the first decode token of each row is random too."""

        if len(lengths) != self.rows:
            raise ValueError("one length per row")
        g = torch.Generator(device=self.device).manual_seed(seed)
        self.context_len = list(lengths)
        for r, n in enumerate(lengths):
            p0, p1, last = shard_row(n, self.page_size, self.shard, self.world)
            pages = [self._alloc_page() for _ in range(p1 - p0)]
            self.host_pages[r], self.host_last[r] = list(pages), last
            if not pages:
                continue
            idx = torch.tensor(pages, device=self.device, dtype=torch.int64)
            for li in range(self.spec.num_layers):
                vals = torch.randn((len(pages),) + tuple(self.kv.shape[2:]), generator=g, device=self.device)
                self.kv[li].index_copy_(0, idx, vals.to(torch.bfloat16))
        self._sync_rows()
        self.token_buf.copy_(torch.randint(0, self.spec.vocab, (self.rows,), generator=g, device=self.device))
        self.plan()

    # ------------------------------------------------------ shared prefix
    def _set_shared_prefix(self, prefix_pages: list[int], prefix_len: int) -> None:
        from pagelora_b200.cascade import SharedPrefixDecode

        if self.world != 1:
            raise ValueError("a shared prefix is not combined with split-KV")
        s = self.spec
        self.prefix_pages = list(prefix_pages)
        self.prefix_len = int(prefix_len)
        self.cascade = SharedPrefixDecode(num_rows=self.rows, num_qo_heads=s.num_qo_heads,
                                          num_kv_heads=s.num_kv_heads, head_dim=s.head_dim,
                                          page_size=self.page_size, prefix_pages=self.prefix_pages,
                                          prefix_last_len=prefix_len - (len(prefix_pages) - 1) * self.page_size,
                                          device=self.device, max_suffix_pages=self.max_pages_per_row)
        self.graph = None

    @torch.no_grad()
    def prefill_shared(self, prefix: list[int], suffixes: list[list[int]]) -> list[int]:
        """Branch batch (the reference's generation.py:872-1132 shape): every
        row continues the same `prefix` with its own suffix.  The prefix K/V
        are stored once in shared pages; each row's page table holds only its
        own tokens, and decode attends to the shared pages through the
        shared-prefix pass.  As in the reference's KV manager
        (pagelora_b200.prefix_plan.plan_prefix), only whole pages of the
        prefix are shared: a partial last page is recomputed into each row's
        own pages.  All rows must use the same adapter (the prefix K/V depend
        on it).  Returns each row's first token."""

        from pagelora_b200.page_table import KVBlockSpan
        from pagelora_b200.prefix_plan import plan_prefix

        if len(suffixes) != self.rows:
            raise ValueError("one suffix per row")
        if len(set(self.row_adapter)) != 1:
            raise ValueError("rows sharing a prefix must use the same adapter")
        ps = self.page_size
        n_pre = len(prefix)
        prefix_pages = [self._alloc_page() for _ in range(-(-n_pre // ps))]
        # what each branch would reuse after the prefix was cached: its radix
        # match is the prefix, its spans the prefix pages
        spans = [KVBlockSpan(p, 0, min(ps, n_pre - i * ps)) for i, p in enumerate(prefix_pages)]
        n_shared = min(plan_prefix(n_pre + len(suf), n_pre, spans, ps).prefill_from for suf in suffixes)
        shared_pages = prefix_pages[: n_shared // ps]
        for p in prefix_pages[n_shared // ps:]:
            self.free_pages.append(p)
        firsts = []
        self.prefill_logits = []
        for r, suf in enumerate(suffixes):
            n = n_pre + len(suf)
            pages = [self._alloc_page() for _ in range(-(-(n - n_shared) // ps))]
            self.host_pages[r], self.host_last[r] = list(pages), (n - n_shared) - (len(pages) - 1) * ps
            pos = torch.arange(n)
            page_of = torch.tensor([shared_pages[p // ps] if p < n_shared else pages[(p - n_shared) // ps]
                                    for p in pos.tolist()], dtype=torch.int32, device=self.device)
            off_of = torch.tensor([p % ps if p < n_shared else (p - n_shared) % ps for p in pos.tolist()],
                                  dtype=torch.int32, device=self.device)
            keep = torch.arange(0 if r == 0 else n_shared, n, device=self.device)  # the shared K/V once
            logits = self._forward_prompt(prefix + suf, self.row_adapter[r], page_of, off_of, keep)
            self.prefill_logits.append(logits)
            firsts.append(int(torch.argmax(logits).item()))
        self.context_len = [n_pre + len(suf) for suf in suffixes]
        if n_shared > 0:
            self._set_shared_prefix(shared_pages, n_shared)
        else:
            self.cascade, self.prefix_pages, self.prefix_len = None, [], 0
        self._sync_rows()
        self.token_buf.copy_(torch.tensor(firsts, dtype=torch.int64))
        self.plan()
        self._check_status()
        return firsts

    @torch.no_grad()
    def fill_random_shared(self, prefix_len: int, suffix_lens: list[int], *, seed: int = 0) -> None:
        """fill_random_context for a branch batch: one shared prefix of random
        K/V plus a random suffix per row."""

        g = torch.Generator(device=self.device).manual_seed(seed)
        ps = self.page_size
        prefix_pages = [self._alloc_page() for _ in range(-(-prefix_len // ps))]
        groups = [prefix_pages] + [[self._alloc_page() for _ in range(-(-n // ps))] for n in suffix_lens]
        for r, n in enumerate(suffix_lens):
            self.host_pages[r], self.host_last[r] = groups[r + 1], n - (len(groups[r + 1]) - 1) * ps
        for pages in groups:
            idx = torch.tensor(pages, device=self.device, dtype=torch.int64)
            for li in range(self.spec.num_layers):
                vals = torch.randn((len(pages),) + tuple(self.kv.shape[2:]), generator=g, device=self.device)
                self.kv[li].index_copy_(0, idx, vals.to(torch.bfloat16))
        self.context_len = [prefix_len + n for n in suffix_lens]
        self._set_shared_prefix(prefix_pages, prefix_len)
        self._sync_rows()
        self.token_buf.copy_(torch.randint(0, self.spec.vocab, (self.rows,), generator=g, device=self.device))
        self.plan()

    # --------------------------------------------------------- decode step
    def _linear(self, x, w, *, prologue=0, norm_weight=None, **kw):
        """Projection of all rows: fused GEMV (prologue inside) when the rows'
        activations fit in shared memory (uses_gemv), else tcgen05 GEMM after
        an explicit norm / SiLU-mul launch."""

        s = self.spec
        if uses_gemv(self.rows, w.shape[1]):
            return K.linear_lora_fused(x, w, prologue=prologue, norm_weight=norm_weight, norm_eps=s.rms_eps,
                                       weights_static=True, status=self.status, **kw)
        if prologue == PL_PROLOGUE_RMSNORM:
            x = K.rmsnorm(x, norm_weight, s.rms_eps, out=self.xn)
        elif prologue == PL_PROLOGUE_SILU_MUL:
            x = K.silu_mul(x, out=self.act)
        return K.linear_lora_gemm(x, w, workspace=self.gemm_ws, weights_static=True, status=self.status, **kw)

    def _decode_body(self) -> None:
        s = self.spec
        st = self.status
        if self.world == 1:
            K.page_table_advance(self.row_num_pages, self.last_page_len, self.row_pages, self.new_page_ids,
                                 self.page_size, self.indptr, self.indices, self.slot_page, self.slot_off,
                                 self.positions, st)
            if self.cascade is not None:
                self.positions.add_(self.prefix_len)  # the rows' tables hold only their suffixes
        else:
            self.positions.add_(1)
            if self.owner:
                K.page_table_advance(self.row_num_pages, self.last_page_len, self.row_pages, self.new_page_ids,
                                     self.page_size, self.indptr, self.indices, self.slot_page, self.slot_off,
                                     None, st)
        # the step's RoPE angles, read by every layer's attention launch
        K.rope_cos_sin(self.positions, s.head_dim, s.rope_theta, out=self.rope_cs)
        K.embed(self.token_buf, self.embed, self.x, st)
        attn2d = self.attn.view(self.rows, s.q_dim)
        lora = self.lora_rank > 0
        for li, L in enumerate(self.layers):
            if lora:
                # The shrink reads the normalised rows: one launch normalises
                # them (written to xn for the projection) and shrinks them.
                if s.hidden <= K.SHRINK_ROWS_MAX_K:
                    K.lora_shrink_rows(self.x, L["a_qkv"], tok_adapter=self.tok_adapter, out=self.down_qkv,
                                       norm_weight=L["input_norm"], norm_eps=s.rms_eps, xn_out=self.xn)
                else:
                    K.rmsnorm(self.x, L["input_norm"], s.rms_eps, out=self.xn)
                    K.lora_shrink_seg(self.xn, L["a_qkv"], self.seg_indptr, self.seg_adapter, out=self.down_qkv)
                self._linear(self.xn, L["w_qkv"], out=self.qkv)
            else:
                self._linear(self.x, L["w_qkv"], prologue=PL_PROLOGUE_RMSNORM, norm_weight=L["input_norm"],
                             out=self.qkv)
            # q/k head norm + RoPE + KV append + paged decode in one launch
            # (on split-KV shards without the tail the slot is not in their
            # page table, so they append nothing and return a partial state).
            qkv_args = dict(num_qo_heads=s.num_qo_heads, num_kv_heads=s.num_kv_heads, positions=self.positions,
                            rope_theta=s.rope_theta, slot_page=self.slot_page, slot_offset=self.slot_off,
                            num_splits=self.num_splits, workspace=self.workspace,
                            lora_down=self.down_qkv if lora else None, lora_b=L["b_qkv"] if lora else None,
                            lora_scale=self.qkv_lora_scale, tok_adapter=self.tok_adapter if lora else None,
                            q_norm_weight=L["q_norm"], k_norm_weight=L["k_norm"], norm_eps=s.rms_eps, status=st,
                            rope_cos_sin=self.rope_cs)
            if self.cascade is not None:
                # shared prefix: append + rotate, then prefix pass + suffix pass + merge
                K.qkv_rope_append(self.qkv, num_qo_heads=s.num_qo_heads, num_kv_heads=s.num_kv_heads,
                                  head_dim=s.head_dim, positions=self.positions, rope_theta=s.rope_theta,
                                  kv_cache=self.kv[li], page_id=self.slot_page, page_offset=self.slot_off,
                                  q_out=self.q, lora_down=qkv_args["lora_down"], lora_b=qkv_args["lora_b"],
                                  lora_scale=self.qkv_lora_scale, tok_adapter=qkv_args["tok_adapter"],
                                  q_norm_weight=L["q_norm"], k_norm_weight=L["k_norm"], norm_eps=s.rms_eps,
                                  status=st)  # (no table argument: evaluates its angles)
                self.cascade.run(self.q, self.kv[li], self.indptr, self.indices, self.last_page_len, self.attn, st)
            elif self.world == 1:
                K.paged_decode_qkv(self.qkv, self.kv[li], self.indptr, self.indices, self.last_page_len,
                                   out=self.attn, **qkv_args)
            else:
                self._split_kv_attention(li, qkv_args)
            if lora:
                if s.q_dim <= K.SHRINK_ROWS_MAX_K:
                    K.lora_shrink_rows(attn2d, L["a_o"], tok_adapter=self.tok_adapter, out=self.down_o)
                else:
                    K.lora_shrink_seg(attn2d, L["a_o"], self.seg_indptr, self.seg_adapter, out=self.down_o)
            self._linear(attn2d, L["w_o"], lora_down=self.down_o if lora else None, lora_b=L["b_o"] if lora else None,
                         lora_scale=self.lora_scale, tok_adapter=self.tok_adapter if lora else None,
                         residual=self.x, out=self.x)
            if self.silu_pairs:
                xn = K.rmsnorm(self.x, L["post_norm"], s.rms_eps, out=self.xn)
                K.linear_lora_gemm(xn, L["w_gate_up"], silu_pairs=True, out=self.act, workspace=self.gemm_ws,
                                   weights_static=True, status=st)
                K.linear_lora_gemm(self.act, L["w_down"], residual=self.x, out=self.x, workspace=self.gemm_ws,
                                   weights_static=True, status=st)
            else:
                self._linear(self.x, L["w_gate_up"], prologue=PL_PROLOGUE_RMSNORM, norm_weight=L["post_norm"],
                             out=self.gate_up)
                self._linear(self.gate_up, L["w_down"], prologue=PL_PROLOGUE_SILU_MUL, residual=self.x,
                             out=self.x)
        self._linear(self.x, self.lm_head, prologue=PL_PROLOGUE_RMSNORM, norm_weight=self.final_norm,
                     out=self.logits)
        K.argmax(self.logits, self.token_buf, self.argmax_ws)

    def _split_kv_attention(self, li: int, qkv_args: dict) -> None:
        """This shard's partial (O fp32, LSE) over its pages, one all-gather of
        the packed partials over NCCL, then the LSE merge (same result on
        every shard)."""

        import torch.distributed as dist

        s = self.spec
        rows_h = self.rows * s.num_qo_heads
        nd = rows_h * s.head_dim
        o_part = self.part[:nd].view(self.rows, s.num_qo_heads, s.head_dim)
        lse_part = self.part[nd:].view(self.rows, s.num_qo_heads)
        K.paged_decode_qkv(self.qkv, self.kv[li], self.indptr, self.indices, self.last_page_len, out=o_part,
                           out_lse=lse_part, **qkv_args)
        if self.peer is not None:
            self.peer.merge(self.part, self.attn.view(rows_h, s.head_dim), self.status)
            return
        dist.all_gather_into_tensor(self.gathered, self.part, group=self.group)
        v = self.gathered[:, :nd].view(self.world, rows_h, s.head_dim).permute(1, 0, 2)
        lse = self.gathered[:, nd:].permute(1, 0)
        K.merge_states_strided(v, lse, self.attn.view(rows_h, s.head_dim))

    def _gate_up(self, w: torch.Tensor) -> torch.Tensor:
        """The [gate; up] stack as the decode projection reads it."""

        return K.interleave_gate_up(w) if self.silu_pairs else w.contiguous()

    def close(self) -> None:
        """Release the graph and unmap the peers' exchange buffers (call on
        every rank once no step is in flight anywhere, before the process
        group goes)."""

        self.graph = None
        if self.peer is not None:
            import torch.distributed as dist

            torch.cuda.synchronize(self.device)
            dist.barrier(group=self.group)
            self.peer.close()
            self.peer = None

    def launches_per_step(self) -> int:
        """Kernel launches of one step (all of them this library's kernels;
        the split-KV position increment and all-gather are not counted)."""

        s, B = self.spec, self.rows
        lora = self.lora_rank > 0
        # q/k norm + RoPE + append + paged decode; with a shared prefix:
        # RoPE + append, prefix pass, suffix pass (merging the prefix state)
        per_layer = 3 if self.cascade is not None else 1
        if self.world > 1:
            per_layer += 1  # partial-state merge
        # q/k/v: with LoRA the norm and the shrink are one launch (up to 8192
        # features), then the projection
        if lora:
            per_layer += 2 if s.hidden <= K.SHRINK_ROWS_MAX_K else 3
        else:
            per_layer += 1 if uses_gemv(B, s.hidden) else 2
        per_layer += 2 if lora else 1  # (o shrink +) o projection
        per_layer += 1 if uses_gemv(B, s.hidden) else 2  # (norm +) gate_up
        # (SiLU-mul +) down; with silu_pairs the gate_up launch writes the SiLU-mul
        per_layer += 1 if (uses_gemv(B, s.intermediate) or self.silu_pairs) else 2
        head = 1 if uses_gemv(B, s.hidden) else 2  # (norm +) lm_head
        advance = 1 if (self.world == 1 or self.owner) else 0
        return advance + 2 + per_layer * s.num_layers + head + 1  # + RoPE table, embed; argmax

    def capture(self) -> None:
        """Capture one decode step into a CUDA graph (after an eager warm-up
        on a copy of the row state)."""

        stream = torch.cuda.Stream(device=self.device)
        stream.wait_stream(torch.cuda.current_stream(self.device))
        state = (self.row_num_pages, self.last_page_len, self.row_pages, self.token_buf, self.positions)
        saved = [t.clone() for t in state]
        with torch.cuda.stream(stream):
            # Rows that need a page in the warm-up get a free one, so no live page is written.
            self.new_page_ids.fill_(self.free_pages[-1] if self.free_pages else 0)
            self._decode_body()
        torch.cuda.current_stream(self.device).wait_stream(stream)
        torch.cuda.synchronize(self.device)
        for dst, src in zip(state, saved):
            dst.copy_(src)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            self._decode_body()
        torch.cuda.synchronize(self.device)
        self.graph = g

    def _host_reserve(self) -> list[int]:
        """Host side of one token's slot reservation per row: a new page id
        where the row's last page is full (0 elsewhere, unused)."""

        out = []
        if self.world > 1 and not self.owner:
            return [0] * self.rows  # the tail lives on the last shard
        for r in range(self.rows):
            if not self.host_pages[r] or self.host_last[r] >= self.page_size:
                page = self._alloc_page()
                self.host_pages[r].append(page)
                self.host_last[r] = 1
                out.append(page)
            else:
                self.host_last[r] += 1
                out.append(0)
        return out

    def step_device(self) -> None:
        """One decode step of all rows with inputs on the device (graph replay)."""

        pages = self._host_reserve()
        self.pinned_pages.copy_(torch.tensor(pages, dtype=torch.int32))
        self.new_page_ids.copy_(self.pinned_pages, non_blocking=True)
        if self.graph is not None:
            self.graph.replay()
        else:
            self._decode_body()

    def step_host(self, tokens: list[int]) -> list[int]:
        """One decode step driven from host memory: H2D of the rows' tokens and
        page ids (pinned), replay, D2H of the next ids."""

        pages = self._host_reserve()
        self.pinned_pages.copy_(torch.tensor(pages, dtype=torch.int32))
        self.pinned_tokens.copy_(torch.tensor(tokens, dtype=torch.int64))
        self.new_page_ids.copy_(self.pinned_pages, non_blocking=True)
        self.token_buf.copy_(self.pinned_tokens, non_blocking=True)
        if self.graph is not None:
            self.graph.replay()
        else:
            self._decode_body()
        self.pinned_tokens.copy_(self.token_buf, non_blocking=True)
        torch.cuda.current_stream(self.device).synchronize()
        return self.pinned_tokens.tolist()

    def _check_status(self) -> None:
        code = int(self.status.item())
        if code != 0:
            from pagelora_b200._capi import status_string

            raise RuntimeError(f"device status {code}: {status_string(code)}")
