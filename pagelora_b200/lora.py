"""Drop-in LoRA linear path on the B200 kernels.

Mirrors the reference's LoRA-linear interface:
  * LoRAModuleWeights, LoRALinear               multilora/linear.py:30-231
  * project_qkv_packed, project_gate_up_packed,
    get_base_gate_up_packed_linear,
    apply_gate_up_activation, project_down,
    project_linear                              model/flashinfer/packed_ops.py:105-265
  * project_qkv_with_optional_norm, ProjectedQKV
                                                model/flashinfer/projection.py:15-110, 248-262
  * effective_linear, effective_packed_linear,
    clear_flashinfer_effective_weight_cache     model/flashinfer/effective_weights.py:53-137
with the same names, arguments, roles (base / serve / train), environment
switches (MINI_OPENCLAW_FLASHINFER_*) and return values.

A projection of T bf16 tokens runs on one kernel with the LoRA expand fused
into its epilogue, after the segment shrink x.A^T:
  * T <= 8 whose activations fit in shared memory: the decode GEMV
    (pl_linear_lora_expand_fused);
  * otherwise T <= 128 (batched decode, branch batches, prefill chunks): the
    tcgen05 GEMM (pl_linear_lora_gemm), with one zeroed workspace per device
    that every call leaves zeroed again.
LoRALinear scales the rounded B product (linear.py:230-231) while the packed
paths fold the scale into B (packed_ops.py:371-373); the kernels reproduce
both roundings.  Merged ("effective") weights are built by the on-device
merge kernel.  More than 128 tokens in one call (a whole prompt) and the
train role use torch ops on the GPU, as the reference does; neither is on
the decode path.  CPU inputs raise: there is no CPU path.
"""

from __future__ import annotations

import itertools
import math
import os
from dataclasses import dataclass
from typing import Iterable

import torch
import torch.nn as nn
import torch.nn.functional as F

from pagelora_b200 import kernels as K

MAX_KERNEL_TOKENS = K.GEMM_MAX_ROWS  # tokens one kernel call projects (GEMV up to 8, tcgen05 GEMM above)


def _env_enabled(name: str, *, default: bool) -> bool:
    value = os.getenv(name)
    if value is None:
        return default
    return value.lower() in {"1", "true", "yes", "on"}


def _need_cuda(x: torch.Tensor) -> None:
    if x.device.type != "cuda":
        raise RuntimeError("pagelora_b200 LoRA path runs on CUDA tensors only (no CPU path)")


_seg_cache: dict[torch.device, tuple[torch.Tensor, torch.Tensor]] = {}


def _single_segment(device: torch.device, tokens: int) -> tuple[torch.Tensor, torch.Tensor]:
    key = (device, tokens)
    seg = _seg_cache.get(key)
    if seg is None:
        seg = (torch.tensor([0, tokens], dtype=torch.int32, device=device),
               torch.zeros(1, dtype=torch.int32, device=device))
        _seg_cache[key] = seg
    return seg


def _tensor_key(t: torch.Tensor) -> tuple:
    return (t.data_ptr(), tuple(t.shape), t.dtype, t.device, int(getattr(t, "_version", 0)))


_gemm_ws: dict[torch.device, torch.Tensor] = {}


def _gemm_workspace(device: torch.device, tokens: int, k_in: int, n_out: int) -> torch.Tensor:
    """The device's shared GEMM workspace (zeroed once; each completed call leaves it zeroed)."""

    need = int(K.gemm_plan(tokens, k_in, n_out).workspace_bytes)
    ws = _gemm_ws.get(device)
    if ws is None or ws.numel() < need:
        ws = torch.zeros(max(need, 1 << 16), dtype=torch.uint8, device=device)
        _gemm_ws[device] = ws
    return ws


def _shrink(x2: torch.Tensor, a_stack: torch.Tensor) -> torch.Tensor:
    """x2 . A^T (fp32) for one adapter: the row kernel (one CTA per token and
    4 rank rows) up to 8192 input features, the segment kernel beyond."""

    if x2.shape[1] <= K.SHRINK_ROWS_MAX_K and x2.shape[1] % 8 == 0:
        return K.lora_shrink_rows(x2, a_stack)
    seg_indptr, seg_adapter = _single_segment(x2.device, x2.shape[0])
    return K.lora_shrink_seg(x2, a_stack, seg_indptr, seg_adapter)


def _kernel_kind(x2: torch.Tensor, k_in: int) -> str | None:
    """Which kernel projects the rows of ``x2`` [T, K]: "gemv", "gemm" or None (torch)."""

    if x2.dtype != torch.bfloat16 or torch.is_grad_enabled() or k_in % 16:
        return None
    t = x2.shape[0]
    if K.gemv_fits(t, k_in):
        return "gemv"
    if t <= K.GEMM_MAX_ROWS:
        return "gemm"
    return None


def _project(kind: str, x2: torch.Tensor, w: torch.Tensor, **epilogue) -> torch.Tensor:
    """x2 . W^T with the fused epilogue (bias, LoRA expand) on the chosen kernel."""

    if kind == "gemv":
        return K.linear_lora_fused(x2, w, **epilogue)
    ws = _gemm_workspace(x2.device, x2.shape[0], w.shape[1], w.shape[0])
    return K.linear_lora_gemm(x2, w, workspace=ws, **epilogue)


@dataclass
class LoRAModuleWeights:
    """Metadata and parameter handles for one LoRA-instrumented linear layer (linear.py:30-41)."""

    a: nn.Parameter
    b: nn.Parameter
    alpha: float
    rank: int

    @property
    def scale(self) -> float:
        return self.alpha / self.rank


class LoRALinear(nn.Module):
    """Single-layer LoRA execution unit (linear.py:44-231)."""

    def __init__(self, linear: nn.Linear, *, rank: int, alpha: float, dropout: float) -> None:
        super().__init__()
        self.in_features = linear.in_features
        self.out_features = linear.out_features
        self.weight = linear.weight
        self.bias = linear.bias
        self.rank = rank
        self.alpha = alpha
        self.scale = alpha / rank
        self.dropout = nn.Dropout(dropout) if dropout > 0 else nn.Identity()
        self.serve_a: nn.Parameter | None = None
        self.serve_b: nn.Parameter | None = None
        self.train_a: nn.Parameter | None = None
        self.train_b: nn.Parameter | None = None
        self.active_role: str = "base"

    # ----------------------------------------------------------- binding
    def bind_serve(self, a: nn.Parameter, b: nn.Parameter) -> None:
        self.serve_a = a
        self.serve_b = b

    def has_train_workspace(self) -> bool:
        return self.train_a is not None and self.train_b is not None

    def materialize_train(self, a: nn.Parameter, b: nn.Parameter) -> None:
        with torch.no_grad():
            self.train_a = nn.Parameter(a.detach().clone(), requires_grad=True)
            self.train_b = nn.Parameter(b.detach().clone(), requires_grad=True)

    def release_train(self) -> None:
        self.train_a = None
        self.train_b = None
        if self.active_role == "train":
            self.active_role = "base"

    def commit_train_to_serve(self, target_a: nn.Parameter, target_b: nn.Parameter) -> None:
        if self.train_a is None or self.train_b is None:
            raise RuntimeError("train workspace is not materialized")
        with torch.no_grad():
            target_a.data.copy_(self.train_a.data.to(target_a.device))
            target_b.data.copy_(self.train_b.data.to(target_b.device))

    # ----------------------------------------------------- merge / unmerge
    def is_lora_merged(self) -> bool:
        return bool(getattr(self, "_merged_lora_adapter", None))

    def merge_serve_lora(self, adapter_name: str) -> bool:
        """Fold the serve LoRA into ``weight`` with the merge kernel (linear.py:130-147)."""

        if self.active_role != "serve" or self.serve_a is None or self.serve_b is None:
            return False
        if not self._dropout_mergeable():
            return False
        merged = getattr(self, "_merged_lora_adapter", None)
        if merged == adapter_name:
            return False
        if merged is not None:
            self.unmerge_serve_lora()
        self._merge(sign=1)
        self._merged_lora_adapter = adapter_name
        return True

    def unmerge_serve_lora(self) -> bool:
        if not self.is_lora_merged():
            return False
        if self.serve_a is None or self.serve_b is None:
            raise RuntimeError("cannot unmerge serve LoRA without bound serve parameters")
        self._merge(sign=-1)
        try:
            delattr(self, "_merged_lora_adapter")
        except AttributeError:
            pass
        return True

    def _merge(self, *, sign: int) -> None:
        w = self.weight.data
        _need_cuda(w)
        a = self.serve_a.detach().to(device=w.device, dtype=w.dtype).contiguous()
        b = self.serve_b.detach().to(device=w.device, dtype=w.dtype).contiguous()
        with torch.no_grad():
            K.lora_merge_weight(w, a, b, float(self.scale), sign=sign, mode=0, out=w)

    def _serve_lora_weight_delta(self) -> torch.Tensor:
        if self.serve_a is None or self.serve_b is None:
            raise RuntimeError("serve LoRA parameters are not bound")
        w = self.weight
        zero = torch.zeros_like(w)
        a = self.serve_a.detach().to(device=w.device, dtype=w.dtype).contiguous()
        b = self.serve_b.detach().to(device=w.device, dtype=w.dtype).contiguous()
        return K.lora_merge_weight(zero, a, b, float(self.scale), mode=0, out=zero)

    def _dropout_mergeable(self) -> bool:
        if isinstance(self.dropout, nn.Identity):
            return True
        if isinstance(self.dropout, nn.Dropout):
            return float(self.dropout.p) == 0.0 or not self.dropout.training
        return False

    # ------------------------------------------------------------ roles
    def set_active_base(self) -> None:
        self.active_role = "base"

    def set_active_serve(self) -> None:
        if self.serve_a is None or self.serve_b is None:
            raise RuntimeError("serve mode requested without a bound serve adapter")
        self.active_role = "serve"

    def set_active_train(self) -> None:
        if self.train_a is None or self.train_b is None:
            raise RuntimeError("train mode requested without materialized train workspace")
        self.active_role = "train"

    # ---------------------------------------------------------- forward
    def forward(self, x: torch.Tensor, *, return_lora_down: bool = False):
        _need_cuda(x)
        lora_on = self.active_role != "base" and not self.is_lora_merged()
        shape = x.shape
        x2 = x.reshape(-1, self.in_features)
        kind = None if self.weight.dtype != torch.bfloat16 else _kernel_kind(x2, self.in_features)
        if kind is None or lora_on and (self.active_role == "train" or not self._dropout_mergeable()):
            return self._forward_torch(x, return_lora_down=return_lora_down)
        x2 = x2.contiguous()
        w = self.weight.contiguous()
        if not lora_on:
            y = _project(kind, x2, w, bias=self.bias).view(*shape[:-1], self.out_features)
            return (y, None) if return_lora_down else y
        if self.serve_a is None or self.serve_b is None:
            raise RuntimeError("serve mode active without bound serve parameters")
        a = self.serve_a.detach().contiguous()
        down = _shrink(x2, a.unsqueeze(0))
        if return_lora_down:
            base = _project(kind, x2, w, bias=self.bias).view(*shape[:-1], self.out_features)
            return base, down.to(x.dtype).view(*shape[:-1], -1)
        b = self.serve_b.detach().to(w.dtype).contiguous()
        y = _project(kind, x2, w, bias=self.bias, lora_down=down, lora_b=b.unsqueeze(0), lora_scale=float(self.scale))
        return y.view(*shape[:-1], self.out_features)

    def _forward_torch(self, x: torch.Tensor, *, return_lora_down: bool):
        base = F.linear(x, self.weight, self.bias)
        if self.active_role == "base" or self.is_lora_merged():
            return (base, None) if return_lora_down else base
        if self.active_role == "serve":
            a, b = self.serve_a, self.serve_b
        else:
            a, b = self.train_a, self.train_b
        if a is None or b is None:
            raise RuntimeError(f"{self.active_role} mode active without bound parameters")
        down = F.linear(self.dropout(x), a, None)
        if return_lora_down:
            return base, down
        return base + F.linear(down, b, None) * self.scale


def init_lora_pair(*, rank: int, in_features: int, out_features: int, device=None, dtype=None):
    """Freshly initialised LoRA A/B (A kaiming-uniform, B zeros; linear.py:234-254)."""

    a = nn.Parameter(torch.empty(rank, in_features, device=device, dtype=dtype), requires_grad=False)
    b = nn.Parameter(torch.empty(out_features, rank, device=device, dtype=dtype), requires_grad=False)
    nn.init.kaiming_uniform_(a, a=math.sqrt(5))
    nn.init.zeros_(b)
    return a, b


# ------------------------------------------------------------- packed / effective
def effective_weights_enabled() -> bool:
    """Same switches as effective_weights.py:32-50."""

    memory_mode = os.getenv("MINI_OPENCLAW_FLASHINFER_MEMORY_MODE", "throughput").lower()
    storage = os.getenv("MINI_OPENCLAW_FLASHINFER_PACKED_WEIGHT_STORAGE", "").lower()
    single = _env_enabled("MINI_OPENCLAW_FLASHINFER_SINGLE_LORA_MERGE", default=False)
    low_vram = memory_mode in {"balanced", "low_vram"} or storage in {"shared", "share", "alias",
                                                                        "shared_storage"} or single
    return _env_enabled("MINI_OPENCLAW_FLASHINFER_EFFECTIVE_WEIGHTS", default=not low_vram)


@dataclass(frozen=True)
class EffectiveLinear:
    weight: torch.Tensor
    bias: torch.Tensor | None
    cache_key: tuple


@dataclass(frozen=True)
class EffectivePackedLinear:
    weight: torch.Tensor
    bias: torch.Tensor | None
    out_features: tuple[int, ...]
    cache_key: tuple


def _serve_lora(module) -> tuple[torch.Tensor, torch.Tensor, float] | None:
    checker = getattr(module, "is_lora_merged", None)
    if callable(checker) and checker():
        return None
    if getattr(module, "active_role", "base") != "serve":
        return None
    a, b = getattr(module, "serve_a", None), getattr(module, "serve_b", None)
    if not isinstance(a, torch.Tensor) or not isinstance(b, torch.Tensor):
        return None
    dropout = getattr(module, "dropout", None)
    if module.training and not isinstance(dropout, nn.Identity) and dropout is not None:
        return None
    return a, b, float(getattr(module, "scale", 1.0))


def _module_key(module) -> tuple:
    a, b = module.serve_a, module.serve_b
    bias = getattr(module, "bias", None)
    return (id(module), "serve", _tensor_key(module.weight), _tensor_key(a), _tensor_key(b),
            float(getattr(module, "scale", 1.0)), None if bias is None else _tensor_key(bias))


def effective_linear(module) -> EffectiveLinear | None:
    """Cached W + scale * B @ A built on the device (effective_weights.py:53-75)."""

    if not effective_weights_enabled():
        return None
    lo = _serve_lora(module)
    if lo is None:
        return None
    key = _module_key(module)
    cached = getattr(module, "_flashinfer_effective_linear", None)
    if isinstance(cached, EffectiveLinear) and cached.cache_key == key:
        return cached
    w = module.weight.detach().contiguous()
    _need_cuda(w)
    a, b, sc = lo
    merged = K.lora_merge_weight(w, a.detach().to(w.dtype).contiguous(), b.detach().to(w.dtype).contiguous(), sc,
                                 mode=0)
    eff = EffectiveLinear(weight=merged, bias=getattr(module, "bias", None), cache_key=key)
    setattr(module, "_flashinfer_effective_linear", eff)
    return eff


def effective_packed_linear(*, owner: object, attr: str, modules: tuple) -> EffectivePackedLinear | None:
    """Packed effective weights of a group (effective_weights.py:78-129): each
    slice is bf16(W + scale * bf16(B @ A)) (add_ with alpha)."""

    if not effective_weights_enabled():
        return None
    los = [_serve_lora(m) for m in modules]
    if any(l is None for l in los):
        return None
    first = modules[0].weight
    if any(m.weight.size(1) != first.size(1) or m.weight.dtype != first.dtype for m in modules):
        return None
    key = tuple(_module_key(m) for m in modules)
    cached = getattr(owner, attr, None)
    if isinstance(cached, EffectivePackedLinear) and cached.cache_key == key:
        return cached
    outs = tuple(m.weight.size(0) for m in modules)
    weight = torch.empty(sum(outs), first.size(1), device=first.device, dtype=first.dtype)
    off = 0
    for m, (a, b, sc), od in zip(modules, los, outs):
        K.lora_merge_weight(m.weight.detach().contiguous(), a.detach().to(first.dtype).contiguous(),
                            b.detach().to(first.dtype).contiguous(), sc, mode=1, out=weight[off: off + od])
        off += od
    biases = [getattr(m, "bias", None) for m in modules]
    bias = None
    if any(bb is not None for bb in biases):
        bias = torch.cat([torch.zeros(od, device=first.device, dtype=first.dtype) if bb is None else bb.detach()
                          for bb, od in zip(biases, outs)])
    packed = EffectivePackedLinear(weight=weight, bias=bias, out_features=outs, cache_key=key)
    setattr(owner, attr, packed)
    return packed


def clear_flashinfer_effective_weight_cache(*roots: object) -> None:
    """Drop cached effective weights below the given objects (effective_weights.py:132-137)."""

    seen: set[int] = set()

    def visit(obj: object) -> None:
        if obj is None or id(obj) in seen:
            return
        seen.add(id(obj))
        if hasattr(obj, "__dict__"):
            for name in list(vars(obj).keys()):
                if name.startswith("_flashinfer_effective_"):
                    try:
                        delattr(obj, name)
                    except AttributeError:
                        pass
        if isinstance(obj, nn.Module):
            for child in obj.children():
                visit(child)
            return
        values: Iterable = obj.values() if isinstance(obj, dict) else (obj if isinstance(obj, (list, tuple, set))
                                                                         else ())
        for v in values:
            visit(v)

    for root in roots:
        visit(root)


@dataclass(frozen=True)
class PackedGroup:
    """Packed base weights of a module group and, when every module serves a
    LoRA of one rank, the packed A rows and B * scale (packed_ops.py:314-384)."""

    weight: torch.Tensor
    bias: torch.Tensor | None
    out_features: tuple[int, ...]
    a_cat: torch.Tensor | None
    b_cat: torch.Tensor | None


def _lora_pack_info(module) -> tuple[torch.Tensor, torch.Tensor, float] | None:
    """A serve LoRA that may be packed: not merged, identity dropout (packed_ops.py:475-502)."""

    checker = getattr(module, "is_lora_merged", None)
    if callable(checker) and checker():
        return None
    if getattr(module, "active_role", "base") != "serve":
        return None
    dropout = getattr(module, "dropout", None)
    if dropout is not None and not isinstance(dropout, nn.Identity) and not (
            isinstance(dropout, nn.Dropout) and float(dropout.p) == 0.0):
        return None
    a, b = getattr(module, "serve_a", None), getattr(module, "serve_b", None)
    if not isinstance(a, torch.Tensor) or not isinstance(b, torch.Tensor) or a.ndim != 2 or b.ndim != 2:
        return None
    return a, b, float(getattr(module, "scale", 1.0))


def _packed_group(owner: object, attr: str, modules: tuple) -> PackedGroup:
    key = tuple((_tensor_key(m.weight), *(_tensor_key(t) for t in (getattr(m, "serve_a", None),
                                                                   getattr(m, "serve_b", None)) if t is not None),
                 getattr(m, "active_role", "base"), float(getattr(m, "scale", 1.0))) for m in modules)
    cached = getattr(owner, attr, None)
    if cached is not None and cached[0] == key:
        return cached[1]
    w = torch.cat([m.weight.detach() for m in modules], 0).contiguous()
    outs = tuple(m.weight.size(0) for m in modules)
    biases = [getattr(m, "bias", None) for m in modules]
    bias = None
    if any(bb is not None for bb in biases):
        bias = torch.cat([torch.zeros(od, device=w.device, dtype=w.dtype) if bb is None else bb.detach().to(w.dtype)
                          for bb, od in zip(biases, outs)]).contiguous()
    infos = [_lora_pack_info(m) for m in modules]
    a_cat = b_cat = None
    if all(i is not None for i in infos) and len({i[0].shape[0] for i in infos}) == 1:
        a_cat = torch.cat([i[0].detach().to(w.dtype) for i in infos], 0).contiguous()
        b_cat = torch.cat([(i[1].detach().to(w.dtype) * i[2]).to(w.dtype) for i in infos], 0).unsqueeze(0).contiguous()
    val = PackedGroup(weight=w, bias=bias, out_features=outs, a_cat=a_cat, b_cat=b_cat)
    setattr(owner, attr, (key, val))
    return val


def _project_group(group: PackedGroup, modules: tuple, hidden: torch.Tensor) -> tuple[torch.Tensor, ...] | None:
    """One packed projection of a module group plus its LoRA deltas, split per
    module (packed_ops.py:140-165, 184-203); None when no kernel takes the input."""

    shape = hidden.shape
    x2 = hidden.reshape(-1, shape[-1])
    kind = _kernel_kind(x2, shape[-1])
    if kind is None:
        return None
    x2 = x2.contiguous()
    dims = list(group.out_features)
    ends = tuple(itertools.accumulate(dims[:-1]))
    packed_delta = _env_enabled("MINI_OPENCLAW_FLASHINFER_PACKED_LORA_DELTA", default=True)
    if group.a_cat is not None and packed_delta and len(dims) <= 4:
        down = _shrink(x2, group.a_cat.unsqueeze(0))
        out = _project(kind, x2, group.weight, bias=group.bias, lora_down=down, lora_b=group.b_cat,
                       slice_ends=ends)
        return tuple(torch.split(out.view(*shape[:-1], -1), dims, dim=-1))
    if not any(getattr(m, "active_role", "base") != "base" and not getattr(m, "is_lora_merged", lambda: False)()
               for m in modules):
        out = _project(kind, x2, group.weight, bias=group.bias)
        return tuple(torch.split(out.view(*shape[:-1], -1), dims, dim=-1))
    # Per-module deltas (packed delta off, or ranks differ): each module's own
    # projection carries its delta, bf16(base) + bf16(bf16(down.B^T) * scale).
    return tuple(m(hidden) if getattr(m, "active_role", "base") != "base" else
                 _project(kind, x2, m.weight.contiguous(), bias=getattr(m, "bias", None)).view(*shape[:-1], -1)
                 for m in modules)


def project_qkv_packed(layer, plan, hidden: torch.Tensor):
    """Q/K/V from one packed projection plus the packed LoRA delta (packed_ops.py:105-165)."""

    if not _env_enabled("MINI_OPENCLAW_FLASHINFER_PACKED_QKV", default=True):
        return None
    attn = layer.self_attn
    mods = tuple(plan.modules.get(f"self_attn.{n}_proj") or getattr(attn, f"{n}_proj") for n in "qkv")
    _need_cuda(hidden)
    if not any(getattr(m, "is_lora_merged", lambda: False)() for m in mods):
        eff = effective_packed_linear(owner=plan, attr="_flashinfer_effective_qkv", modules=mods)
        if eff is not None:
            qkv = project_dense(hidden, eff.weight, eff.bias)
            return torch.split(qkv, list(eff.out_features), dim=-1)
    group = _packed_group(plan, "_b200_packed_qkv", mods)
    out = _project_group(group, mods, hidden)
    if out is not None:
        return out
    return tuple(m(hidden) for m in mods)


def get_base_gate_up_packed_linear(mlp):
    """Packed gate/up parameters (packed_ops.py:206-228): effective weights when
    enabled, else the packed base weights; None when packing is off."""

    if not _env_enabled("MINI_OPENCLAW_FLASHINFER_PACKED_MLP", default=True):
        return None
    gate, up = getattr(mlp, "gate_proj", None), getattr(mlp, "up_proj", None)
    if gate is None or up is None:
        return None
    if not any(getattr(m, "is_lora_merged", lambda: False)() for m in (gate, up)):
        eff = effective_packed_linear(owner=mlp, attr="_flashinfer_effective_gate_up", modules=(gate, up))
        if eff is not None:
            return eff
    return _packed_group(mlp, "_b200_packed_gate_up", (gate, up))


def project_gate_up_packed(mlp, hidden: torch.Tensor):
    """MLP gate/up from one packed projection plus LoRA deltas (packed_ops.py:168-203)."""

    packed = get_base_gate_up_packed_linear(mlp)
    if packed is None:
        return None
    _need_cuda(hidden)
    if isinstance(packed, EffectivePackedLinear):
        return project_dense(hidden, packed.weight, packed.bias)
    mods = (mlp.gate_proj, mlp.up_proj)
    out = _project_group(packed, mods, hidden)
    if out is None:
        return torch.cat([m(hidden) for m in mods], dim=-1)
    return torch.cat(out, dim=-1) if len(out) > 1 else out[0]


def apply_gate_up_activation(gate_up: torch.Tensor, act_fn) -> torch.Tensor:
    """SwiGLU over packed [gate | up] (packed_ops.py:231-240) on the SiLU-and-mul kernel."""

    name = act_fn.__class__.__name__.lower()
    silu = (name in {"silu", "siluactivation", "swishactivation"}
            or getattr(act_fn, "__name__", "").lower() in {"silu", "swish"})
    fused = _env_enabled("MINI_OPENCLAW_FLASHINFER_FUSED_ACT", default=True)
    if (fused and silu and gate_up.dtype == torch.bfloat16 and gate_up.device.type == "cuda"
            and gate_up.size(-1) % 16 == 0):
        shape = gate_up.shape
        return K.silu_mul(gate_up.reshape(-1, shape[-1]).contiguous()).view(*shape[:-1], shape[-1] // 2)
    gate, up = gate_up.chunk(2, dim=-1)
    return act_fn(gate) * up


def project_down(mlp, hidden: torch.Tensor) -> torch.Tensor:
    """The MLP down projection with its optional LoRA wrapper (packed_ops.py:243-248)."""

    down = getattr(mlp, "down_proj", None)
    if down is None:
        raise RuntimeError("MLP module does not expose down_proj")
    return project_linear(down, hidden)


def project_dense(hidden: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None) -> torch.Tensor:
    """F.linear on the GEMV / tcgen05 GEMM for up to 128 bf16 tokens."""

    _need_cuda(hidden)
    shape = hidden.shape
    x2 = hidden.reshape(-1, shape[-1])
    kind = _kernel_kind(x2, shape[-1]) if weight.dtype == torch.bfloat16 else None
    if kind is not None:
        return _project(kind, x2.contiguous(), weight.contiguous(), bias=bias).view(*shape[:-1], -1)
    return F.linear(hidden, weight, bias)


def project_linear(module, hidden: torch.Tensor) -> torch.Tensor:
    """One linear module with serve effective weights when enabled (packed_ops.py:251-265)."""

    checker = getattr(module, "is_lora_merged", None)
    if callable(checker) and checker():
        return project_dense(hidden, module.weight, getattr(module, "bias", None))
    eff = effective_linear(module)
    if eff is not None:
        return project_dense(hidden, eff.weight, eff.bias)
    if getattr(module, "active_role", "base") != "base":
        return module(hidden)
    weight = getattr(module, "weight", None)
    if isinstance(weight, torch.Tensor) and weight.ndim == 2:
        return project_dense(hidden, weight, getattr(module, "bias", None))
    return module(hidden)


# ------------------------------------------------------- q/k/v + head norm
@dataclass(frozen=True)
class ProjectedQKV:
    """Q/K/V after projection and optional per-head Q/K normalisation (projection.py:15-22)."""

    q_bshd: torch.Tensor
    k_bshd: torch.Tensor
    v_bshd: torch.Tensor
    v_bhsd: torch.Tensor | None


def _head_norm(states: torch.Tensor, norm, *, use_flashinfer_norm: bool) -> torch.Tensor:
    """Per-head RMSNorm of [B, S, H, D] states (projection.py:248-262): the
    FlashInfer rounding (once) when enabled, else the Hugging Face module's
    (normalise, round, scale, round)."""

    weight = getattr(norm, "weight", None)
    eps = float(getattr(norm, "variance_epsilon", getattr(norm, "eps", 1e-6)))
    if (not isinstance(weight, torch.Tensor) or states.dtype != torch.bfloat16 or weight.dtype != torch.bfloat16
            or states.device.type != "cuda" or states.size(-1) % 8):
        return norm(states)
    flat = states.reshape(-1, states.size(-1)).contiguous()
    fn = K.rmsnorm if use_flashinfer_norm else K.rmsnorm_hf
    return fn(flat, weight.contiguous(), eps).view_as(states)


def project_qkv_with_optional_norm(layer, plan, normed_hidden: torch.Tensor, *,
                                   use_flashinfer_norm: bool | None = None) -> ProjectedQKV:
    """Project Q/K/V (packed, with LoRA) and apply the model's optional q/k
    head norms (projection.py:34-110)."""

    attn = layer.self_attn
    if use_flashinfer_norm is None:
        use_flashinfer_norm = _env_enabled("MINI_OPENCLAW_FLASHINFER_QK_NORM", default=False)
    config = attn.config
    num_qo_heads = int(config.num_attention_heads)
    num_kv_heads = int(getattr(config, "num_key_value_heads", num_qo_heads))
    head_dim = int(attn.head_dim)
    bsz, seqlen, _ = normed_hidden.shape
    packed = project_qkv_packed(layer, plan, normed_hidden)
    if packed is None:
        mods = tuple(plan.modules.get(f"self_attn.{n}_proj") or getattr(attn, f"{n}_proj") for n in "qkv")
        packed = tuple(project_linear(m, normed_hidden) for m in mods)
    q_flat, k_flat, v_flat = packed
    q_bshd = q_flat.reshape(bsz, seqlen, num_qo_heads, head_dim)
    k_bshd = k_flat.reshape(bsz, seqlen, num_kv_heads, head_dim)
    q_norm, k_norm = getattr(attn, "q_norm", None), getattr(attn, "k_norm", None)
    if q_norm is not None:
        q_bshd = _head_norm(q_bshd, q_norm, use_flashinfer_norm=use_flashinfer_norm)
    if k_norm is not None:
        k_bshd = _head_norm(k_bshd, k_norm, use_flashinfer_norm=use_flashinfer_norm)
    v_bshd = v_flat.reshape(bsz, seqlen, num_kv_heads, head_dim)
    return ProjectedQKV(q_bshd=q_bshd, k_bshd=k_bshd, v_bshd=v_bshd,
                        v_bhsd=None if bsz == 1 else v_bshd.transpose(1, 2).contiguous())
