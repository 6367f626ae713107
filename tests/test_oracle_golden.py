"""The CPU oracle against the reference's own outputs (no GPU).

The fixtures were produced by tests/golden/make_golden.py, which runs the
reference's code: page tables (model/kvcache/flashinfer_page_table.py),
LoRALinear / packed projection / merged weights (multilora/linear.py,
model/flashinfer/packed_ops.py, model/flashinfer/effective_weights.py) and
the HF eager greedy generate path on the config-1 tiny Llama.
"""

from __future__ import annotations

import json
import math

import numpy as np
import pytest

from oracle import lora as olora
from oracle import page_table as opt
from oracle.decoder import OracleDecoder
from oracle.numerics import bf16
from oracle.paged_decode import merge_states, paged_decode, split_states
from oracle.paged_prefill import paged_prefill


def test_page_table_known_answers():
    # test/test_paged_kvcache_manager.py:429-461
    assert opt.build_batch([[(11, 0, 2), (12, 0, 1)]], 2) == ([0, 2], [11, 12], [1])
    assert opt.build_batch([[(11, 0, 2), (12, 0, 1)], [(21, 0, 2)]], 2) == ([0, 2, 3], [11, 12, 21], [1, 2])
    with pytest.raises(ValueError, match="offset 0"):
        opt.build_batch([[(1, 1, 1)]], 2)
    with pytest.raises(ValueError, match="full pages"):
        opt.build_batch([[(1, 0, 1), (2, 0, 1)]], 2)


def test_page_table_matches_reference_fixture(golden_dir):
    cases = json.loads((golden_dir / "page_tables.json").read_text())
    assert len(cases) > 300
    for case in cases:
        if "error" in case:
            with pytest.raises(ValueError) as exc:
                opt.build_batch(case["rows"], case["page_size"])
            assert str(exc.value) == case["error"]
        else:
            indptr, indices, last = opt.build_batch(case["rows"], case["page_size"])
            assert indptr == case["indptr"]
            assert indices == case["indices"]
            assert last == case["last_page_len"]


def _close_bf16(actual, expected, ulps: int = 2):
    """Within a few bf16 ulps (accumulation order differs from torch's)."""

    actual = np.asarray(actual, np.float32)
    expected = np.asarray(expected, np.float32)
    tol = ulps * np.maximum(np.abs(expected), 1e-3) * 2.0 ** -8 + 1e-6
    assert np.all(np.abs(actual - expected) <= tol), float(np.max(np.abs(actual - expected) / tol))


def test_lora_linear_matches_reference(golden_dir):
    z = np.load(golden_dir / "lora_cases.npz")
    for dt in ("f32", "bf16"):
        for case in range(3):
            pre = f"lora_linear_{dt}_{case}_"
            bias = z[pre + "bias"] if z[pre + "bias"].size else None
            y = olora.lora_linear(z[pre + "x"], z[pre + "w"], bias, z[pre + "a"], z[pre + "b"],
                                  float(z[pre + "scale"][0]), bf16=(dt == "bf16"))
            if dt == "f32":
                np.testing.assert_allclose(y, z[pre + "y"], rtol=1e-5, atol=1e-5)
            else:
                _close_bf16(y, z[pre + "y"])


def test_packed_qkv_matches_reference(golden_dir):
    z = np.load(golden_dir / "lora_cases.npz")
    for case in range(2):
        pre = f"packed_{case}_"
        sc = float(z[pre + "scale"][0])
        ws = [z[f"{pre}{m}_w"] for m in "qkv"]
        loras = [(z[f"{pre}{m}_a"], z[f"{pre}{m}_b"], sc) for m in "qkv"]
        q, k, v = olora.packed_qkv(z[pre + "x"], ws, [None] * 3, loras, bf16=True)
        _close_bf16(q, z[pre + "q"])
        _close_bf16(k, z[pre + "k"])
        _close_bf16(v, z[pre + "v"])


def test_merge_weight_matches_reference(golden_dir):
    z = np.load(golden_dir / "lora_cases.npz")
    w, a, b, sc = z["merge_w"], z["merge_a"], z["merge_b"], float(z["merge_scale"][0])
    _close_bf16(olora.merge_weight(w, a, b, sc, mode=0), z["merge_effective_linear"])
    _close_bf16(olora.merge_weight(w, a, b, sc, mode=0), z["merge_serve_merged"])
    _close_bf16(olora.merge_weight(w, a, b, sc, mode=1), z["merge_effective_packed"])
    merged = olora.merge_weight(w, a, b, sc, mode=0)
    _close_bf16(olora.merge_weight(merged, a, b, sc, mode=0, sign=-1), z["merge_serve_unmerged"])


def test_tiny_llama_greedy_matches_reference_hf_path(golden_dir):
    """BASELINE config 1 through the oracle decoder (paged KV, fp32) vs the
    reference's HF eager generate on the same weights."""

    import torch

    from pagelora_b200.synthetic import WORKLOADS, make_lora_weights, make_model_weights

    g = np.load(golden_dir / "tiny_llama_greedy.npz")
    wl = WORKLOADS["config1"]
    weights = make_model_weights(wl.model, seed=0, dtype=torch.float32)
    checksum = float(sum(float(v.double().sum()) for v in weights.values()))
    assert math.isclose(checksum, float(g["weight_checksum"][0]), rel_tol=1e-9)
    loras = make_lora_weights(wl.model, wl.lora, dtype=torch.float32)
    dec = OracleDecoder(wl.model, weights, loras, wl.lora.scale, page_size=wl.page_size, num_pages=16, bf16=False)
    tokens, first_logits = dec.generate(g["prompt"].tolist(), wl.decode_tokens)
    np.testing.assert_allclose(first_logits, g["first_logits"], rtol=1e-4, atol=1e-4)
    assert tokens == g["tokens"].tolist()


def test_decode_finite_mask_known_answer():
    """Restates test/test_flashinfer_backend.py:157-177 for decode: tokens past
    last_page_len must not win even when their scores dominate."""

    cache = np.zeros((1, 2, 2, 1, 1), np.float32)
    cache[0, 0, :, 0, 0] = [100.0, 1e4]  # K: the second slot is not valid
    cache[0, 1, :, 0, 0] = [1.0, 9.0]    # V
    q = np.full((1, 1, 1), -1000.0, np.float32)
    out, _ = paged_decode(q, cache, [0, 1], [0], [1])
    assert out[0, 0, 0] == 1.0
    out, _ = paged_decode(np.full((1, 1, 1), 0.0, np.float32), cache, [0, 1], [0], [2])
    assert out[0, 0, 0] == pytest.approx(5.0)


def test_prefill_finite_mask_known_answer():
    """Restates test/test_flashinfer_backend.py:157-177 (the reference's
    prefill test): causal query 0 sees key 0 only, query 1 sees both equal
    scores."""

    cache = np.zeros((1, 2, 2, 1, 1), np.float32)
    cache[0, 0, :, 0, 0] = 100.0
    cache[0, 1, :, 0, 0] = [1.0, 9.0]
    q = np.full((2, 1, 1), -1000.0, np.float32)
    out, _ = paged_prefill(q, cache, [0, 2], [0, 1], [0], [2])
    assert out[:, 0, 0].tolist() == [1.0, 5.0]


def test_prefill_rows_equal_decodes_over_visible_prefix():
    """Causal prefill query i (of the last qo_len positions) equals a decode
    over the first kv_len - qo_len + i + 1 keys; non-causal equals a decode
    over all keys."""

    rng = np.random.default_rng(4)
    ps, n_pages = 16, 7
    cache = bf16(rng.normal(size=(n_pages, 2, ps, 2, 64)))
    pages = list(rng.permutation(n_pages)[:5])
    kv_len, qo = 70, 9
    q = bf16(rng.normal(size=(qo, 8, 64)))
    last = kv_len - 4 * ps
    out, lse = paged_prefill(q, cache, [0, qo], [0, 5], pages, [last])
    for i in range(qo):
        vis = kv_len - qo + i + 1
        n = -(-vis // ps)
        d_out, d_lse = paged_decode(q[i:i + 1], cache, [0, n], pages[:n], [vis - (n - 1) * ps])
        np.testing.assert_allclose(out[i], d_out[0], rtol=1e-12, atol=1e-12)
        np.testing.assert_allclose(lse[i], d_lse[0], rtol=1e-12)
    out_nc, _ = paged_prefill(q, cache, [0, qo], [0, 5], pages, [last], causal=False)
    for i in range(qo):
        d_out, _ = paged_decode(q[i:i + 1], cache, [0, 5], pages, [last])
        np.testing.assert_allclose(out_nc[i], d_out[0], rtol=1e-12, atol=1e-12)


def test_split_merge_equals_full():
    rng = np.random.default_rng(3)
    cache = bf16(rng.normal(size=(12, 2, 16, 2, 64)))
    q = bf16(rng.normal(size=(1, 8, 64)))
    indptr, indices, last = [0, 9], list(rng.permutation(12)[:9]), [5]
    full, full_lse = paged_decode(q, cache, indptr, indices, last)
    for s in (1, 2, 4, 9, 12):
        v, lse = split_states(q, cache, indptr, indices, last, 0, s)
        out, out_lse = merge_states(v, lse)
        np.testing.assert_allclose(out, full[0], rtol=1e-12, atol=1e-12)
        np.testing.assert_allclose(out_lse, full_lse[0], rtol=1e-12)


def test_page_table_advance_matches_reserve_semantics():
    rows = [[], [7]]
    last = [0, 16]
    slot_p, slot_o, pos = opt.advance(rows, last, [3, 4], 16)
    assert (slot_p, slot_o, pos) == ([3, 4], [0, 0], [0, 16])
    slot_p, slot_o, pos = opt.advance(rows, last, [9, 9], 16)
    assert (slot_p, slot_o, pos) == ([3, 4], [1, 1], [1, 17])


def test_hf_eager_baseline_reproduces_reference_greedy(golden_dir):
    """The CPU baseline's restatement of the reference's HF eager path
    (oracle.hf_eager: transformers forward + the LoRALinear serve math), run
    in fp32 on BASELINE config 1, gives the reference's own 32 greedy tokens
    and first-step logits (fixture made by the reference's generate path)."""

    import torch

    from oracle.hf_eager import HFEagerDecoder
    from pagelora_b200.synthetic import WORKLOADS, make_lora_weights, make_model_weights

    z = np.load(golden_dir / "tiny_llama_greedy.npz")
    wl = WORKLOADS["config1"]
    weights = make_model_weights(wl.model, seed=0, dtype=torch.float32)
    assert math.isclose(sum(float(v.double().sum()) for v in weights.values()), float(z["weight_checksum"][0]),
                        rel_tol=1e-9)
    loras = make_lora_weights(wl.model, wl.lora, dtype=torch.float32)
    dec = HFEagerDecoder(wl.model, weights, loras, wl.lora.scale, dtype=torch.float32)
    first = dec.prefill(z["prompt"].tolist())
    assert float((dec.logits[0] - torch.from_numpy(z["first_logits"])).abs().max()) <= 1e-4
    toks = [first]
    while len(toks) < 32:
        toks.append(dec.step(toks[-1]))
    assert toks == z["tokens"].tolist()
