"""Numpy restatement of one paged decode step of a Llama / Qwen3 decoder
with LoRA on the attention projections (test oracle and CPU baseline).

The layer follows the reference's decode layer
(model/flashinfer/layer_runner.py:283-337, 399-421): RMSNorm -> packed
q/k/v projection + LoRA delta (packed_ops.py:105-165) -> Qwen3 q/k head
norms (projection.py:90-103) -> RoPE (projection.py:155-190) -> paged KV
append (layer_runner.py:399-412) -> paged decode attention
(attention_backend.py:120-131) -> o_proj + LoRA (linear.py:200-231) ->
residual + RMSNorm (norm.py:27-57) -> SwiGLU MLP -> residual, then the
final norm and lm_head (cuda_graph.py:262-263) and greedy argmax
(sampling.py:8-15).  Pages come from a LIFO free list
(paged_kv_allocator.py:42-61) and the page table from oracle.page_table.

``bf16=True`` rounds where the reference's bf16 FlashInfer path rounds;
``bf16=False`` is the reference's fp32 eager (HF) arithmetic.
"""

from __future__ import annotations

import numpy as np

from oracle import lora as olora
from oracle import page_table as opt
from oracle.numerics import apply_rope, bf16 as _bf16, rmsnorm_fused, rmsnorm_hf, silu
from oracle.paged_decode import paged_decode


def _np(t) -> np.ndarray:
    import torch

    if isinstance(t, torch.Tensor):
        return t.detach().float().cpu().numpy()
    return np.asarray(t, dtype=np.float32)


class OracleDecoder:
    """Single-sequence greedy decoder over a paged KV pool."""

    def __init__(self, spec, weights: dict, loras: dict | None, lora_scale: float, *, page_size: int = 16,
                 num_pages: int = 64, bf16: bool = True) -> None:
        self.spec = spec
        self.bf = bf16
        self.w = {k: _np(v) for k, v in weights.items()}
        self.loras = {k: (_np(a), _np(b)) for k, (a, b) in (loras or {}).items()}
        self.scale = float(lora_scale)
        self.ps = page_size
        self.cache = np.zeros((spec.num_layers, num_pages, 2, page_size, spec.num_kv_heads, spec.head_dim),
                              dtype=np.float32)
        self.free = list(range(num_pages))  # popped from the end: LIFO reuse
        self.pages: list[int] = []
        self.last = 0
        self.pos = 0

    # -------------------------------------------------------------- helpers
    def _r(self, x):
        return _bf16(x) if self.bf else np.asarray(x, dtype=np.float32)

    def _norm(self, x, w):
        if self.bf:
            return rmsnorm_fused(x, w, self.spec.rms_eps)
        xf = x.astype(np.float64)
        r = 1.0 / np.sqrt(np.mean(xf * xf, axis=-1, keepdims=True) + self.spec.rms_eps)
        return (xf * r * w).astype(np.float32)

    def _head_norm(self, x, w):
        if self.bf:
            return rmsnorm_hf(x, w, self.spec.rms_eps)
        xf = x.astype(np.float64)
        r = 1.0 / np.sqrt(np.mean(xf * xf, axis=-1, keepdims=True) + self.spec.rms_eps)
        return (xf * r * w).astype(np.float32)

    def _lora(self, layer: int, target: str):
        key = f"layers.{layer}.{target}"
        if key not in self.loras:
            return None
        a, b = self.loras[key]
        return (a, b, self.scale)

    def _reserve_slot(self) -> tuple[int, int]:
        """paged_kv_store.reserve_spans for a one-token chunk."""

        if not self.pages or self.last >= self.ps:
            self.pages.append(self.free.pop())
            self.last = 0
        page, off = self.pages[-1], self.last
        self.last += 1
        return page, off

    def page_table(self):
        spans = [(p, 0, self.ps) for p in self.pages[:-1]] + ([(self.pages[-1], 0, self.last)] if self.pages else [])
        return opt.build_batch([spans], self.ps)

    # ----------------------------------------------------------------- step
    def step(self, token: int) -> tuple[int, np.ndarray]:
        """Feed one token at the next position; return (greedy next id, logits)."""

        s = self.spec
        p = "model.layers.{}."
        h = self.w["model.embed_tokens.weight"][token][None, :].astype(np.float32)
        page, off = self._reserve_slot()
        pos = self.pos
        for i in range(s.num_layers):
            pre = p.format(i)
            x = self._norm(h, self.w[pre + "input_layernorm.weight"])
            qkv_loras = [self._lora(i, "q"), self._lora(i, "k"), self._lora(i, "v")]
            if self.bf:
                q, k, v = olora.packed_qkv(
                    x,
                    [self.w[pre + "self_attn.q_proj.weight"], self.w[pre + "self_attn.k_proj.weight"],
                     self.w[pre + "self_attn.v_proj.weight"]],
                    [None, None, None], qkv_loras, bf16=True)
            else:  # fp32: the three projections plus per-module deltas (same math, no packing copies)
                q, k, v = (olora.linear(x, self.w[pre + f"self_attn.{m}_proj.weight"], bf16=False)
                           + (0.0 if l is None else olora.lora_delta(x, l[0], l[1], l[2], bf16=False))
                           for m, l in zip("qkv", qkv_loras))
            q = np.asarray(q, dtype=np.float32).reshape(1, s.num_qo_heads, s.head_dim)
            k = np.asarray(k, dtype=np.float32).reshape(1, s.num_kv_heads, s.head_dim)
            v = np.asarray(v, dtype=np.float32).reshape(1, s.num_kv_heads, s.head_dim)
            if s.qk_norm:
                q = self._head_norm(q, self.w[pre + "self_attn.q_norm.weight"])
                k = self._head_norm(k, self.w[pre + "self_attn.k_norm.weight"])
            q = self._r(apply_rope(q, np.array([pos]), s.rope_theta))
            k = self._r(apply_rope(k, np.array([pos]), s.rope_theta))
            self.cache[i, page, 0, off] = k[0]
            self.cache[i, page, 1, off] = v[0]
            indptr, indices, last = self.page_table()
            o, _ = paged_decode(q, self.cache[i], indptr, indices, last)
            attn = self._r(o.reshape(1, s.q_dim))
            lo = self._lora(i, "o")
            y = olora.lora_linear(attn, self.w[pre + "self_attn.o_proj.weight"], None,
                                  None if lo is None else lo[0], None if lo is None else lo[1], self.scale,
                                  bf16=self.bf)
            h = self._r(h + y)
            x2 = self._norm(h, self.w[pre + "post_attention_layernorm.weight"])
            gate = olora.linear(x2, self.w[pre + "mlp.gate_proj.weight"], bf16=self.bf)
            up = olora.linear(x2, self.w[pre + "mlp.up_proj.weight"], bf16=self.bf)
            act = self._r(silu(gate) * up)
            mlp = olora.linear(act, self.w[pre + "mlp.down_proj.weight"], bf16=self.bf)
            h = self._r(h + mlp)
        xf = self._norm(h, self.w["model.norm.weight"])
        head = self.w.get("lm_head.weight", self.w["model.embed_tokens.weight"])
        logits = olora.linear(xf, head, bf16=self.bf)[0]
        self.pos += 1
        return int(np.argmax(logits)), logits

    def generate(self, prompt: list[int], max_new_tokens: int) -> tuple[list[int], np.ndarray]:
        """Prefill token by token, then greedy decode; returns (new ids, first-step logits)."""

        nxt, logits = 0, None
        for t in prompt:
            nxt, logits = self.step(int(t))
        first_logits = logits
        out = [nxt]
        while len(out) < max_new_tokens:
            nxt, _ = self.step(out[-1])
            out.append(nxt)
        return out, first_logits
