"""The reference's Hugging Face / PyTorch eager decode path on the host CPU.

Test infrastructure and CPU baseline only: ``bench.py --impl reference`` and
its ``cpu_baseline`` leg time this module; no product code imports it.

The reference's CPU path is ``model.generate`` of a transformers causal LM
whose q/k/v/o projections are ``LoRALinear`` modules
(model/generation.py:312-375), with the prefill / decode split of
test/inference/common.py:363-474: one prefill forward, then per decode token
``model(input_ids=[[tok]], past_key_values=cache, attention_mask=...,
cache_position=...)`` followed by a greedy ``argmax`` of the last logits.
This module builds that model from the transformers library itself (the
same third-party code the reference runs), with the Qwen3 / Llama
configuration of a benchmark workload, random-init weights from
``pagelora_b200.synthetic`` and the serve-role LoRA forward of
multilora/linear.py:200-231 restated:

    y = F.linear(x, W, b) + F.linear(F.linear(dropout(x), A), B) * (alpha / rank)

The prompt's KV cache is filled with seeded random K/V of the workload's
context length instead of a CPU prefill (a decode step's cost does not depend
on where its cached K/V came from, and a 2048-token bf16 prefill of an 8B
model takes minutes on a few host cores).
"""

from __future__ import annotations

import os
import time

import torch
import torch.nn as nn
import torch.nn.functional as F


class EagerLoRALinear(nn.Module):
    """Serve-role forward of the reference's LoRALinear (multilora/linear.py:200-231)."""

    def __init__(self, weight: torch.Tensor, a: torch.Tensor, b: torch.Tensor, scale: float) -> None:
        super().__init__()
        self.weight = nn.Parameter(weight, requires_grad=False)
        self.bias = None
        self.serve_a = nn.Parameter(a, requires_grad=False)
        self.serve_b = nn.Parameter(b, requires_grad=False)
        self.scale = float(scale)
        self.dropout = nn.Identity()

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        base = F.linear(x, self.weight, self.bias)
        lora_down = F.linear(self.dropout(x), self.serve_a, None)
        lora_up = F.linear(lora_down, self.serve_b, None)
        return base + lora_up * self.scale


def hf_config(spec):
    """transformers config of a benchmark ModelSpec (Qwen3 when it has q/k norm, else Llama)."""

    common = dict(vocab_size=spec.vocab, hidden_size=spec.hidden, intermediate_size=spec.intermediate,
                  num_hidden_layers=spec.num_layers, num_attention_heads=spec.num_qo_heads,
                  num_key_value_heads=spec.num_kv_heads, head_dim=spec.head_dim, rms_norm_eps=spec.rms_eps,
                  rope_theta=spec.rope_theta, max_position_embeddings=65536,
                  tie_word_embeddings=spec.tie_embeddings, attention_bias=False, use_cache=True)
    if spec.qk_norm:
        from transformers import Qwen3Config

        cfg = Qwen3Config(**common)
    else:
        from transformers import LlamaConfig

        cfg = LlamaConfig(**common)
    cfg._attn_implementation = "sdpa"
    return cfg


def _fill_normal_parallel(params: list[torch.Tensor], std: float, seed: int, threads: int,
                          chunk: int = 1 << 24) -> None:
    """Fill tensors with N(0, std) from seeded per-chunk generators, chunks in parallel.

    torch's CPU normal_ with an explicit generator is single-threaded (~60 M
    samples/s here), so drawing 8 G weights one tensor at a time takes
    minutes; the chunks release the GIL and spread over the host threads."""

    from concurrent.futures import ThreadPoolExecutor

    jobs = []
    for ti, t in enumerate(params):
        flat = t.detach().view(-1)
        for ci, start in enumerate(range(0, flat.numel(), chunk)):
            jobs.append((flat, start, min(flat.numel(), start + chunk), seed * 1_000_003 + ti * 4099 + ci))

    @torch.no_grad()
    def run(job):
        flat, a, b, s = job
        g = torch.Generator().manual_seed(s)
        flat[a:b].copy_(torch.empty(b - a, dtype=torch.float32).normal_(0.0, std, generator=g))

    prev = torch.get_num_threads()
    torch.set_num_threads(1)
    try:
        with ThreadPoolExecutor(max_workers=threads) as pool:
            list(pool.map(run, jobs))
    finally:
        torch.set_num_threads(prev)


def build_model(spec, weights: dict[str, torch.Tensor] | None, loras: dict | None, lora_scale: float,
                dtype=torch.bfloat16, *, seed: int = 0, threads: int = 1):
    """A transformers causal LM holding ``weights`` (HF names), with LoRA on the targeted projections.

    With ``weights=None`` the linear and embedding weights are drawn in place
    as N(0, 0.02) (the Hugging Face initialisation; seeded, parallel chunks)
    and the RMSNorm weights are ones."""

    from transformers import AutoModelForCausalLM

    cfg = hf_config(spec)
    with torch.device("meta"):
        model = AutoModelForCausalLM.from_config(cfg, dtype=dtype)
    model.to_empty(device="cpu")
    if weights is None:
        with torch.no_grad():
            mats = [p for n, p in model.named_parameters() if p.dim() == 2]
            for n, p in model.named_parameters():
                if p.dim() == 1:
                    p.fill_(1.0)
            _fill_normal_parallel(mats, 0.02, seed, threads)
    else:
        state = {k: v.to(dtype) for k, v in weights.items()}
        if spec.tie_embeddings:
            state["lm_head.weight"] = state["model.embed_tokens.weight"]
        missing, unexpected = model.load_state_dict(state, strict=False, assign=True)
        missing = [m for m in missing if "rotary_emb" not in m]
        if missing or unexpected:
            raise RuntimeError(f"weights do not match the model: missing {missing[:4]}, unexpected {unexpected[:4]}")
    # The rotary tables were allocated on the meta device: rebuild them on the CPU.
    rope_cls = type(model.model.rotary_emb)
    model.model.rotary_emb = rope_cls(config=cfg)
    for key, (a, b) in (loras or {}).items():
        _, li, target = key.split(".")
        attn = model.model.layers[int(li)].self_attn
        name = f"{target}_proj"
        base = getattr(attn, name)
        setattr(attn, name, EagerLoRALinear(base.weight.data, a.to(dtype), b.to(dtype), lora_scale))
    model.eval()
    return model


class HFEagerDecoder:
    """Greedy decode of one sequence through the transformers eager forward."""

    def __init__(self, spec, weights: dict | None, loras: dict | None, lora_scale: float, *,
                 dtype=torch.bfloat16, seed: int = 0, threads: int = 1) -> None:
        from transformers import DynamicCache

        self.spec = spec
        self.dtype = dtype
        self.model = build_model(spec, weights, loras, lora_scale, dtype=dtype, seed=seed, threads=threads)
        self.cache = DynamicCache(config=self.model.config)
        self.pos = 0
        self.attention_mask = torch.ones((1, 0), dtype=torch.long)
        self.logits: torch.Tensor | None = None

    @torch.no_grad()
    def fill_random_context(self, context: int, *, seed: int = 0) -> None:
        """Put ``context`` tokens of seeded random K/V into every layer's cache."""

        gen = torch.Generator().manual_seed(seed)
        shape = (1, self.spec.num_kv_heads, context, self.spec.head_dim)
        for li in range(self.spec.num_layers):
            k = torch.randn(shape, generator=gen, dtype=torch.float32).to(self.dtype)
            v = torch.randn(shape, generator=gen, dtype=torch.float32).to(self.dtype)
            self.cache.update(k, v, li)
        self.pos = context
        self.attention_mask = torch.ones((1, context), dtype=torch.long)

    @torch.no_grad()
    def prefill(self, prompt: list[int]) -> int:
        """The prompt forward of test/inference/common.py:394-404; returns the greedy next token."""

        ids = torch.tensor([prompt], dtype=torch.long)
        self.attention_mask = torch.ones_like(ids)
        out = self.model(input_ids=ids, attention_mask=self.attention_mask, past_key_values=self.cache,
                         use_cache=True, return_dict=True)
        self.cache = out.past_key_values
        self.pos = len(prompt)
        self.logits = out.logits[:, -1, :]
        return int(torch.argmax(self.logits, dim=-1)[0])

    @torch.no_grad()
    def step(self, token: int) -> int:
        """One decode token (test/inference/common.py:445-465): forward, argmax."""

        self.attention_mask = torch.cat([self.attention_mask, torch.ones((1, 1), dtype=torch.long)], dim=1)
        out = self.model(input_ids=torch.tensor([[token]], dtype=torch.long), past_key_values=self.cache,
                         attention_mask=self.attention_mask, use_cache=True,
                         cache_position=torch.tensor([self.pos], dtype=torch.long), return_dict=True)
        self.cache = out.past_key_values
        self.pos += 1
        self.logits = out.logits[:, -1, :]
        return int(torch.argmax(self.logits, dim=-1)[0])

    def generate(self, prompt: list[int], max_new_tokens: int) -> list[int]:
        toks = [self.prefill(prompt)]
        while len(toks) < max_new_tokens:
            toks.append(self.step(toks[-1]))
        return toks


def time_decode(workload: str = "config2", *, steps: int, warmup: int, threads: int | None = None) -> dict:
    """Time ``steps`` decode tokens of a benchmark workload's single sequence
    on the host CPU (after ``warmup`` untimed tokens)."""

    from pagelora_b200.synthetic import WORKLOADS, make_lora_weights

    threads = threads or os.cpu_count() or 1
    torch.set_num_threads(threads)
    wl = WORKLOADS[workload]
    t0 = time.perf_counter()
    loras = make_lora_weights(wl.model, wl.lora, dtype=torch.bfloat16)
    dec = HFEagerDecoder(wl.model, None, loras, wl.lora.scale, seed=0, threads=threads)
    del loras
    dec.fill_random_context(wl.prompt_len, seed=0)
    build_s = time.perf_counter() - t0
    tok = 1
    for _ in range(warmup):
        tok = dec.step(tok)
    t0 = time.perf_counter()
    for _ in range(steps):
        tok = dec.step(tok)
    s_per_token = (time.perf_counter() - t0) / max(1, steps)
    return {"value": 1.0 / s_per_token, "unit": "tok/s", "cores": threads, "kind": "port",
            "s_per_token": s_per_token, "build_s": build_s, "cpu": _cpu_model(),
            "sample": (f"{workload}: transformers {wl.model.name} eager forward ({wl.model.num_layers} full-size "
                       f"layers + lm_head, bf16, N(0, 0.02) weights, {threads} threads) with the reference "
                       f"LoRALinear serve forward on {'/'.join(wl.lora.targets)}, KV cache of {wl.prompt_len} "
                       f"random tokens, {steps} timed greedy decode tokens after {warmup} untimed")}


def _cpu_model() -> str:
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"
