"""bf16 rounding and small numeric helpers for the numpy oracle.

``bf16`` reproduces a torch bfloat16 store (round-to-nearest-even of the
fp32 value), so the oracle can place rounding at the same points as the
reference's torch / FlashInfer ops.
"""

from __future__ import annotations

import numpy as np


def bf16(x) -> np.ndarray:
    """Round to the nearest bf16 (ties to even); returns float32."""

    a = np.ascontiguousarray(np.asarray(x, dtype=np.float32))
    u = a.view(np.uint32).astype(np.uint64)
    u = (u + (((u >> 16) & 1) + 0x7FFF)) & 0xFFFF0000
    out = u.astype(np.uint32).view(np.float32)
    nan = np.isnan(a)
    if nan.any():
        out = np.where(nan, np.float32(np.nan), out)
    return out.reshape(a.shape)


def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    return (np.asarray(bits, dtype=np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    return (bf16(x).view(np.uint32) >> 16).astype(np.uint16)


def rmsnorm_fused(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    """FlashInfer rmsnorm as called by model/flashinfer/norm.py:60-65: fp32
    math, one bf16 rounding: bf16(x * rsqrt(mean(x^2) + eps) * w)."""

    xf = np.asarray(x, dtype=np.float32)
    r = 1.0 / np.sqrt(np.mean(xf.astype(np.float64) ** 2, axis=-1, keepdims=True) + eps)
    return bf16(xf * r.astype(np.float32) * np.asarray(w, dtype=np.float32))


def rmsnorm_hf(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    """HF LlamaRMSNorm / Qwen3RMSNorm module (used for Qwen3 q_norm/k_norm,
    model/flashinfer/projection.py:248-260): normalise in fp32, round to
    bf16, multiply by the weight, round again."""

    xf = np.asarray(x, dtype=np.float32)
    r = 1.0 / np.sqrt(np.mean(xf.astype(np.float64) ** 2, axis=-1, keepdims=True) + eps)
    return bf16(np.asarray(w, dtype=np.float32) * bf16(xf * r.astype(np.float32)))


def rope_inv_freq(head_dim: int, theta: float) -> np.ndarray:
    """inv_freq[i] = 1 / theta^(2i / D) in fp32 (HF rotary embedding)."""

    i = np.arange(0, head_dim, 2, dtype=np.float32)
    return (1.0 / (np.float32(theta) ** (i / np.float32(head_dim)))).astype(np.float32)


def apply_rope(x: np.ndarray, positions: np.ndarray, theta: float) -> np.ndarray:
    """Non-interleaved RoPE in fp32 (FlashInfer apply_rope_pos_ids with
    interleave=False, model/flashinfer/projection.py:181-189):
    out[i] = x[i] cos - x[i+D/2] sin ; out[i+D/2] = x[i+D/2] cos + x[i] sin.
    x [..., T, H, D] with positions [T]."""

    d = x.shape[-1]
    inv = rope_inv_freq(d, theta)
    ang = (np.asarray(positions, dtype=np.float32)[:, None] * inv[None, :]).astype(np.float64)
    cos = np.cos(ang)[:, None, :]
    sin = np.sin(ang)[:, None, :]
    x1 = x[..., : d // 2].astype(np.float64)
    x2 = x[..., d // 2:].astype(np.float64)
    return np.concatenate([x1 * cos - x2 * sin, x2 * cos + x1 * sin], axis=-1).astype(np.float32)


def silu(x: np.ndarray) -> np.ndarray:
    xf = np.asarray(x, dtype=np.float64)
    return (xf / (1.0 + np.exp(-xf))).astype(np.float32)
