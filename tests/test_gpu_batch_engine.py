"""Batched multi-adapter decode (config-3 shape) on the B200 kernels vs the CPU oracle.

Rows of different context lengths, each with its own LoRA adapter (or none),
decode together: 12 rows take the tcgen05 GEMM projections, 5 rows the fused
decode GEMV.  Every row's logits are compared with an oracle decoder that
runs that row alone with its adapter (the reference serves one adapter per
call; the batch must reproduce each row's single-adapter result).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle.decoder import OracleDecoder
from pagelora_b200.synthetic import LoRASpec, ModelSpec, make_lora_weights, make_model_weights, random_prompt

pytestmark = pytest.mark.gpu

SMALL_LLAMA2 = ModelSpec("small-llama2-mha", 2, 512, 8, 8, 64, 1024, 4096, 10000.0, 1e-5)
SMALL_LORA = LoRASpec(16, 32.0, ("q", "k", "v", "o"), num_adapters=3)


def _setup(row_adapter, device):
    from pagelora_b200.batch_engine import BatchDecodeEngine

    spec, lspec = SMALL_LLAMA2, SMALL_LORA
    w = make_model_weights(spec, seed=0, dtype=torch.float32, norm_jitter=0.1)
    w = {k: v.bfloat16() for k, v in w.items()}
    adapters = [make_lora_weights(spec, lspec, adapter=a, dtype=torch.bfloat16) for a in range(3)]
    oracles = []
    for ad in row_adapter:
        lo = None if ad < 0 else {k: (a.float(), b.float()) for k, (a, b) in adapters[ad].items()}
        oracles.append(OracleDecoder(spec, {k: v.float() for k, v in w.items()}, lo, lspec.scale, page_size=16,
                                     num_pages=16, bf16=True))
    eng = BatchDecodeEngine(spec, dict(w), adapters=adapters, lora_spec=lspec, row_adapter=row_adapter,
                            page_size=16, max_context=160, device=device)
    eng.shuffle_free_pages(seed=4)
    return eng, oracles


@pytest.mark.parametrize("row_adapter", [[-1, -1, 0, 0, 0, 1, 1, 1, 1, 2, 2, 2], [-1, 0, 1, 2, 2]],
                         ids=["12rows-gemm", "5rows-gemv"])
def test_batch_decode_matches_per_row_oracle(cuda_device, row_adapter):
    eng, oracles = _setup(row_adapter, cuda_device)
    rng = np.random.default_rng(7)
    lengths = rng.integers(5, 70, size=len(row_adapter)).tolist()
    prompts = [random_prompt(SMALL_LLAMA2.vocab, n, seed=10 + i) for i, n in enumerate(lengths)]
    eng.prefill(prompts)
    nxt = []
    for r, (o, p) in enumerate(zip(oracles, prompts)):
        tok, lg = 0, None
        for t in p:
            tok, lg = o.step(t)
        err = float(np.max(np.abs(eng.prefill_logits[r].float().cpu().numpy() - lg)))
        assert err < 0.1, (r, err)
        nxt.append(tok)
    for step in range(4):
        if step == 2:
            eng.capture()  # the last steps replay the captured graph
        eng.step_host(nxt)
        got = eng.logits.float().cpu().numpy()
        new = []
        for r, o in enumerate(oracles):
            tok, lg = o.step(nxt[r])
            err = float(np.max(np.abs(got[r] - lg)))
            assert err < 0.1, (step, r, err)
            new.append(tok)
        nxt = new
    assert int(eng.status.item()) == 0


def test_batch_decode_crosses_page_boundaries_and_random_pages(cuda_device):
    """Rows sitting at a page boundary get their next page from the host each
    step; pages come from a shuffled pool."""

    eng, oracles = _setup([-1, 0, 0, 1, 1, 2, 2, 2, 2, 2], cuda_device)
    lengths = [16, 15, 31, 32, 1, 17, 47, 48, 2, 33]
    prompts = [random_prompt(SMALL_LLAMA2.vocab, n, seed=40 + i) for i, n in enumerate(lengths)]
    eng.prefill(prompts)
    nxt = []
    for o, p in zip(oracles, prompts):
        tok = 0
        for t in p:
            tok, _ = o.step(t)
        nxt.append(tok)
    eng.capture()
    for _ in range(18):  # every row crosses at least one page boundary
        eng.step_host(nxt)
        got = eng.logits.float().cpu().numpy()
        new = []
        for r, o in enumerate(oracles):
            tok, lg = o.step(nxt[r])
            assert float(np.max(np.abs(got[r] - lg))) < 0.1
            new.append(tok)
        nxt = new
    assert int(eng.status.item()) == 0


SMALL_QWEN = ModelSpec("small-qwen3", 2, 512, 8, 2, 128, 1024, 4096, 1.0e6, 1e-6, qk_norm=True)


@pytest.mark.parametrize("rows,prefix_len", [(6, 48), (10, 48), (6, 53)],
                         ids=["6rows-gemv", "10rows-gemm", "6rows-prefix-mid-page"])
def test_shared_prefix_branches_match_oracle(cuda_device, rows, prefix_len):
    """Branch batch: rows continue one shared prefix (its whole pages stored
    once, a partial last page recomputed per row as the reference's KV manager
    does) with their own suffixes; decode runs the shared-prefix pass + suffix
    pass + merge.  Every row's logits equal an oracle decoder that ran
    prefix + suffix alone."""

    from pagelora_b200.batch_engine import BatchDecodeEngine

    spec, lspec = SMALL_QWEN, LoRASpec(16, 32.0, ("q", "k", "v", "o"))
    w = make_model_weights(spec, seed=0, dtype=torch.float32, norm_jitter=0.1)
    w = {k: v.bfloat16() for k, v in w.items()}
    lo = make_lora_weights(spec, lspec, dtype=torch.bfloat16)
    eng = BatchDecodeEngine(spec, dict(w), adapters=[lo], lora_spec=lspec, row_adapter=[0] * rows, page_size=16,
                            max_context=160, device=cuda_device)
    eng.shuffle_free_pages(seed=9)
    prefix = random_prompt(spec.vocab, prefix_len, seed=1)
    rng = np.random.default_rng(rows)
    suffixes = [random_prompt(spec.vocab, int(n), seed=20 + i) for i, n in enumerate(rng.integers(1, 30, size=rows))]
    eng.prefill_shared(prefix, suffixes)
    assert eng.prefix_len == prefix_len // 16 * 16  # whole pages only
    oracles, nxt = [], []
    for suf in suffixes:
        o = OracleDecoder(spec, {k: v.float() for k, v in w.items()},
                          {k: (a.float(), b.float()) for k, (a, b) in lo.items()}, lspec.scale, page_size=16,
                          num_pages=16, bf16=True)
        tok = 0
        for t in prefix + suf:
            tok, _ = o.step(t)
        oracles.append(o)
        nxt.append(tok)
    for step in range(4):
        if step == 2:
            eng.capture()
        eng.step_host(nxt)
        got = eng.logits.float().cpu().numpy()
        new = []
        for r, o in enumerate(oracles):
            tok, lg = o.step(nxt[r])
            err = float(np.max(np.abs(got[r] - lg)))
            assert err < 0.1, (step, r, err)
            new.append(tok)
        nxt = new
    assert int(eng.status.item()) == 0
