"""Restatement of the reference's LoRA linear path (test oracle).

Every function can round like the reference's bf16 torch ops (``bf16=True``:
each torch op's output is rounded to bf16, accumulation in float64 here) or
compute in plain fp32/fp64 (``bf16=False``, the reference's CPU fp32 runs).

  * lora_linear       multilora/linear.py:200-231 (LoRALinear.forward)
  * packed_qkv        model/flashinfer/packed_ops.py:105-165, 314-384
  * merge_weight      multilora/linear.py:130-172 (mode 0),
                      model/flashinfer/effective_weights.py:108-121 (mode 1)
  * shrink_seg        per-segment x . A^T of linear.py:226-227
"""

from __future__ import annotations

import numpy as np

from oracle.numerics import bf16 as _bf16


def _r(x, on: bool) -> np.ndarray:
    return _bf16(x) if on else np.asarray(x)


def linear(x, w, b=None, *, bf16: bool) -> np.ndarray:
    """F.linear(x, w, b): fp64 accumulation and a bf16 output rounding when
    emulating the bf16 path, plain fp32 BLAS otherwise (the fp32 CPU path)."""

    dt = np.float64 if bf16 else np.float32
    y = np.asarray(x, dtype=dt) @ np.asarray(w, dtype=dt).T
    if b is not None:
        y = y + np.asarray(b, dtype=dt)
    return _r(y, bf16)


def lora_linear(x, w, b, a, bmat, scale: float, *, bf16: bool) -> np.ndarray:
    """base = x W^T + b; down = x A^T; y = base + (down B^T) * scale."""

    base = linear(x, w, b, bf16=bf16)
    if a is None:
        return base
    down = linear(x, a, bf16=bf16)
    up = linear(down, bmat, bf16=bf16)
    return _r(base + _r(up * scale, bf16), bf16)


def lora_delta(x, a, bmat, scale: float, *, bf16: bool) -> np.ndarray:
    """_lora_delta (packed_ops.py:534-553): (x A^T) B^T * scale."""

    down = linear(x, a, bf16=bf16)
    return _r(linear(down, bmat, bf16=bf16) * scale, bf16)


def packed_lora_mats(loras, out_dims, *, bf16: bool) -> tuple[np.ndarray, np.ndarray]:
    """A_cat [sum r, in] and block-diagonal B_blk [sum out, sum r] with the
    scale folded in (packed_ops.py:360-375)."""

    a_cat = np.concatenate([np.asarray(a, dtype=np.float64) for a, _, _ in loras], axis=0)
    ranks = [np.asarray(a).shape[0] for a, _, _ in loras]
    b_blk = np.zeros((sum(out_dims), sum(ranks)))
    ro = oo = 0
    for (a, bm, sc), od, r in zip(loras, out_dims, ranks):
        b_blk[oo: oo + od, ro: ro + r] = _r(np.asarray(bm, dtype=np.float64) * sc, bf16)
        oo += od
        ro += r
    return a_cat, b_blk


def packed_qkv(x, ws, biases, loras, *, bf16: bool, packed_delta: bool = True) -> list[np.ndarray]:
    """Packed base projection + LoRA delta, split per module.

    ``loras`` is a list of (A, B, scale) or None per module.  When every
    module has a LoRA and packed_delta is on, the packed block-diagonal path
    of packed_ops.py:144-154 is used; otherwise per-module deltas (:156-165).
    """

    out_dims = [np.asarray(w).shape[0] for w in ws]
    w_cat = np.concatenate([np.asarray(w, dtype=np.float64) for w in ws], axis=0)
    b_cat = None
    if any(b is not None for b in biases):
        b_cat = np.concatenate([np.zeros(od) if b is None else np.asarray(b, dtype=np.float64)
                                for b, od in zip(biases, out_dims)])
    qkv = linear(x, w_cat, b_cat, bf16=bf16)
    if packed_delta and all(l is not None for l in loras):
        a_cat, b_blk = packed_lora_mats(loras, out_dims, bf16=bf16)
        down = linear(x, a_cat, bf16=bf16)
        delta = linear(down, b_blk, bf16=bf16)
        qkv = _r(qkv + delta, bf16)
        outs, off = [], 0
        for od in out_dims:
            outs.append(qkv[..., off: off + od])
            off += od
        return outs
    outs, off = [], 0
    for od, l in zip(out_dims, loras):
        part = qkv[..., off: off + od]
        if l is not None:
            part = _r(part + lora_delta(x, l[0], l[1], l[2], bf16=bf16), bf16)
        outs.append(part)
        off += od
    return outs


def merge_weight(w, a, bmat, scale: float, *, mode: int = 0, sign: int = 1, bf16: bool = True) -> np.ndarray:
    """W + sign * scale * (B @ A) with the reference's rounding points."""

    d = _r(np.asarray(bmat, dtype=np.float64) @ np.asarray(a, dtype=np.float64), bf16)
    w = np.asarray(w, dtype=np.float64)
    if mode == 0:
        return _r(w + sign * _r(d * scale, bf16), bf16)
    return _r(w + sign * scale * d, bf16)


def shrink_seg(x, a_stack, seg_indptr, seg_adapter) -> np.ndarray:
    """down[t] = x[t] . A[adapter(seg(t))]^T in float64; adapter -1 -> zeros."""

    x = np.asarray(x, dtype=np.float64)
    a_stack = np.asarray(a_stack, dtype=np.float64)
    rank = a_stack.shape[1]
    out = np.zeros((x.shape[0], rank))
    for sg in range(len(seg_adapter)):
        t0, t1, ad = int(seg_indptr[sg]), int(seg_indptr[sg + 1]), int(seg_adapter[sg])
        if ad >= 0:
            out[t0:t1] = x[t0:t1] @ a_stack[ad].T
    return out
