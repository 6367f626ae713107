"""Synthetic workloads of the benchmark configurations.

There are no checkpoints or datasets on the benchmark hosts, so every model
is the named architecture with random-init weights (N(0, 0.02) linear and
embedding weights, unit RMSNorm weights: the Hugging Face initialisation)
drawn from a seeded generator in a fixed tensor order, and every prompt is
uniform-random token ids.  LoRA A and B are N(0, 0.02) with seed
1 + adapter index (the reference initialises B to zero, which would make the
delta vanish).
"""

from __future__ import annotations

from dataclasses import dataclass, field

import torch


@dataclass(frozen=True)
class ModelSpec:
    """Decoder-only Llama / Qwen3 architecture (the fields the decode path reads)."""

    name: str
    num_layers: int
    hidden: int
    num_qo_heads: int
    num_kv_heads: int
    head_dim: int
    intermediate: int
    vocab: int
    rope_theta: float
    rms_eps: float
    qk_norm: bool = False
    tie_embeddings: bool = False

    @property
    def q_dim(self) -> int:
        return self.num_qo_heads * self.head_dim

    @property
    def kv_dim(self) -> int:
        return self.num_kv_heads * self.head_dim

    @property
    def qkv_dim(self) -> int:
        return self.q_dim + 2 * self.kv_dim

    def weight_bytes(self, itemsize: int = 2) -> int:
        """Bytes of weights one decode step streams (embedding row excluded)."""

        per_layer = (self.qkv_dim * self.hidden + self.hidden * self.q_dim + 2 * self.intermediate * self.hidden
                     + self.hidden * self.intermediate + 2 * self.hidden)
        if self.qk_norm:
            per_layer += 2 * self.head_dim
        return itemsize * (self.num_layers * per_layer + self.vocab * self.hidden + self.hidden)


@dataclass(frozen=True)
class LoRASpec:
    rank: int
    alpha: float
    targets: tuple[str, ...]  # subset of ("q", "k", "v", "o")
    num_adapters: int = 1

    @property
    def scale(self) -> float:
        return self.alpha / self.rank


@dataclass(frozen=True)
class Workload:
    name: str
    model: ModelSpec
    lora: LoRASpec
    batch: int
    prompt_len: int
    decode_tokens: int
    page_size: int = 16
    notes: str = ""
    extra: dict = field(default_factory=dict)


TINY_LLAMA = ModelSpec("tiny-llama", 2, 512, 8, 2, 64, 1408, 32000, 10000.0, 1e-6)
QWEN3_8B = ModelSpec("qwen3-8b", 36, 4096, 32, 8, 128, 12288, 151936, 1.0e6, 1e-6, qk_norm=True)
LLAMA2_7B = ModelSpec("llama2-7b", 32, 4096, 32, 32, 128, 11008, 32000, 10000.0, 1e-5)
LLAMA3_8B = ModelSpec("llama3-8b", 32, 4096, 32, 8, 128, 14336, 128256, 500000.0, 1e-5)

WORKLOADS = {
    "config1": Workload("config1", TINY_LLAMA, LoRASpec(8, 16.0, ("q", "v")), 1, 128, 32),
    "config2": Workload("config2", QWEN3_8B, LoRASpec(16, 32.0, ("q", "k", "v", "o")), 1, 2048, 128),
    "config3": Workload("config3", LLAMA2_7B, LoRASpec(16, 32.0, ("q", "k", "v", "o"), num_adapters=8), 64, 0, 0,
                        notes="64 rows, context U[512, 4096], pages randomly permuted"),
    "config4": Workload("config4", QWEN3_8B, LoRASpec(16, 32.0, ("q", "k", "v", "o")), 16, 2048 + 64, 128,
                        notes="2048 shared prefix + 16 x 64 suffix"),
    "config5": Workload("config5", LLAMA3_8B, LoRASpec(16, 32.0, ("q", "v")), 8, 32768, 64),
}


def _normal(gen: torch.Generator, shape, std: float, device, dtype) -> torch.Tensor:
    return torch.empty(shape, device=device, dtype=torch.float32).normal_(0.0, std, generator=gen).to(dtype)


def make_model_weights(spec: ModelSpec, *, seed: int = 0, device="cpu", dtype=torch.bfloat16,
                       norm_jitter: float = 0.0) -> dict[str, torch.Tensor]:
    """Random-init weights in Hugging Face naming (``model.layers.{i}.self_attn.q_proj.weight`` ...).

    ``norm_jitter`` > 0 draws RMSNorm weights as 1 + N(0, jitter) so tests
    exercise the norm weights; the benchmark uses the HF default of ones.
    """

    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    std = 0.02
    w: dict[str, torch.Tensor] = {}

    def norm(n: int) -> torch.Tensor:
        if norm_jitter > 0:
            return (1.0 + _normal(gen, (n,), norm_jitter, device, torch.float32)).to(dtype)
        return torch.ones(n, device=device, dtype=dtype)

    w["model.embed_tokens.weight"] = _normal(gen, (spec.vocab, spec.hidden), std, device, dtype)
    for i in range(spec.num_layers):
        p = f"model.layers.{i}."
        w[p + "self_attn.q_proj.weight"] = _normal(gen, (spec.q_dim, spec.hidden), std, device, dtype)
        w[p + "self_attn.k_proj.weight"] = _normal(gen, (spec.kv_dim, spec.hidden), std, device, dtype)
        w[p + "self_attn.v_proj.weight"] = _normal(gen, (spec.kv_dim, spec.hidden), std, device, dtype)
        w[p + "self_attn.o_proj.weight"] = _normal(gen, (spec.hidden, spec.q_dim), std, device, dtype)
        w[p + "mlp.gate_proj.weight"] = _normal(gen, (spec.intermediate, spec.hidden), std, device, dtype)
        w[p + "mlp.up_proj.weight"] = _normal(gen, (spec.intermediate, spec.hidden), std, device, dtype)
        w[p + "mlp.down_proj.weight"] = _normal(gen, (spec.hidden, spec.intermediate), std, device, dtype)
        w[p + "input_layernorm.weight"] = norm(spec.hidden)
        w[p + "post_attention_layernorm.weight"] = norm(spec.hidden)
        if spec.qk_norm:
            w[p + "self_attn.q_norm.weight"] = norm(spec.head_dim)
            w[p + "self_attn.k_norm.weight"] = norm(spec.head_dim)
    w["model.norm.weight"] = norm(spec.hidden)
    if not spec.tie_embeddings:
        w["lm_head.weight"] = _normal(gen, (spec.vocab, spec.hidden), std, device, dtype)
    return w


def module_dims(spec: ModelSpec, target: str) -> tuple[int, int]:
    """(out_features, in_features) of q/k/v/o."""

    return {
        "q": (spec.q_dim, spec.hidden),
        "k": (spec.kv_dim, spec.hidden),
        "v": (spec.kv_dim, spec.hidden),
        "o": (spec.hidden, spec.q_dim),
    }[target]


def make_lora_weights(spec: ModelSpec, lora: LoRASpec, *, adapter: int = 0, device="cpu",
                      dtype=torch.bfloat16) -> dict[str, tuple[torch.Tensor, torch.Tensor]]:
    """{"layers.{i}.{target}": (A [r, in], B [out, r])} with N(0, 0.02) entries."""

    gen = torch.Generator(device=device)
    gen.manual_seed(1 + adapter)
    out = {}
    for i in range(spec.num_layers):
        for t in lora.targets:
            o, k = module_dims(spec, t)
            a = _normal(gen, (lora.rank, k), 0.02, device, dtype)
            b = _normal(gen, (o, lora.rank), 0.02, device, dtype)
            out[f"layers.{i}.{t}"] = (a, b)
    return out


def random_prompt(vocab: int, length: int, *, seed: int = 0) -> list[int]:
    gen = torch.Generator().manual_seed(seed)
    return torch.randint(0, vocab, (length,), generator=gen).tolist()
