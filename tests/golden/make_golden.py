"""Generate the golden fixtures by running the REFERENCE's own code.

Run in a container where the PageLoRA reference is importable (it is not on
the benchmark hosts, so the outputs are committed as fixtures):

    python tests/golden/make_golden.py --reference /path/to/PageLoRA

Fixtures written next to this script:
  page_tables.json        model/kvcache/flashinfer_page_table.py outputs
                          (build_flashinfer_batch_page_table) and ValueError
                          messages for seeded random span lists and the
                          reference test-suite's known answers
  lora_cases.npz          multilora/linear.py LoRALinear.forward (fp32 and
                          bf16), packed_ops.project_qkv_packed with the
                          packed LoRA delta, merge_serve_lora and
                          effective_weights.effective_linear /
                          effective_packed_linear outputs
  lora_batched_cases.npz  the same LoRA surfaces at batched-decode token
                          counts (16, 64, 128 rows), plus
                          packed_ops.project_gate_up_packed and
                          projection.project_qkv_with_optional_norm (Qwen3
                          q/k head norms), bf16
  prefix_plans.json       model/kvcache/paged_kvcache_manager.py prefix reuse
                          (radix lookup result -> match_len, prefill_from,
                          prefix_spans), the batch page table of branch
                          batches (the config-4 shape) and the admission
                          estimates
  tiny_llama_greedy.npz   BASELINE config 1: the reference's HF eager
                          generate path (model/generation.py:312-375) on a
                          random-init tiny Llama with LoRA (q, v) wrapped by
                          the reference LoRALinear -- 32 greedy tokens and
                          the first-step logits
"""

from __future__ import annotations

import argparse
import json
import os
import random
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent


def _spans_case(rng: random.Random, page_size: int) -> list[list[list[int]]]:
    """A batch of rows of spans: mostly valid tables, sometimes split into
    coalescable slices, with empty slices and occasional malformed spans."""

    rows = []
    for _ in range(rng.randint(1, 5)):
        n_pages = rng.randint(0, 7)
        pages = rng.sample(range(100), n_pages)
        spans: list[list[int]] = []
        for j, p in enumerate(pages):
            full = page_size if j < n_pages - 1 else rng.randint(1, page_size)
            if rng.random() < 0.3 and full > 1:  # split one page into adjacent slices
                cut = rng.randint(1, full - 1)
                spans.append([p, 0, cut])
                if rng.random() < 0.3:
                    spans.append([p, cut, 0])  # empty slice: skipped by the coalescer
                spans.append([p, cut, full - cut])
            else:
                spans.append([p, 0, full])
        if spans and rng.random() < 0.15:  # corrupt one span
            k = rng.randrange(len(spans))
            kind = rng.randint(0, 2)
            if kind == 0:
                spans[k][1] = rng.randint(1, page_size - 1)
            elif kind == 1:
                spans[k][2] = page_size + rng.randint(1, 5)
            else:
                spans[k][2] = max(1, spans[k][2] - 1)
        rows.append(spans)
    return rows


def make_page_tables(out: Path) -> None:
    from model.kvcache.flashinfer_page_table import build_flashinfer_batch_page_table
    from model.kvcache.radix_types import KVBlockSpan

    rng = random.Random(0)
    cases = []
    # Known answers of test/test_paged_kvcache_manager.py:429-543.
    fixed = [
        (2, [[[11, 0, 2], [12, 0, 1]]]),
        (2, [[[11, 0, 2], [12, 0, 1]], [[21, 0, 2]]]),
        (2, [[[1, 1, 1]]]),
        (2, [[[1, 0, 1], [2, 0, 1]]]),
        (2, [[[11, 0, 1]]]),
        (4, [[[2, 0, 3]], [[4, 0, 4]]]),
        (4, [[[2, 0, 4]], [[4, 0, 4], [5, 0, 1]]]),
        (16, [[]]),
        (16, [[], [[3, 0, 16], [9, 0, 5]], []]),
    ]
    batches = list(fixed)
    for _ in range(300):
        ps = rng.choice([2, 4, 16, 32])
        batches.append((ps, _spans_case(rng, ps)))
    for ps, rows in batches:
        spans = [[KVBlockSpan(*s) for s in row] for row in rows]
        case = {"page_size": ps, "rows": rows}
        try:
            t = build_flashinfer_batch_page_table(spans, page_size=ps, device=torch.device("cpu"))
            case["indptr"] = t.paged_kv_indptr.tolist()
            case["indices"] = t.paged_kv_indices.tolist()
            case["last_page_len"] = t.paged_kv_last_page_len.tolist()
        except ValueError as exc:
            case["error"] = str(exc)
        cases.append(case)
    out.write_text(json.dumps(cases))
    print(f"page_tables.json: {len(cases)} cases, {sum('error' in c for c in cases)} errors")


def _bf16_np(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().numpy()


def make_lora_cases(out: Path) -> None:
    os.environ["MINI_OPENCLAW_FLASHINFER_PACKED_QKV"] = "1"
    os.environ["MINI_OPENCLAW_FLASHINFER_PACKED_LORA_DELTA"] = "1"
    os.environ["MINI_OPENCLAW_FLASHINFER_EFFECTIVE_WEIGHTS"] = "0"
    from types import SimpleNamespace

    import torch.nn as nn

    from model.flashinfer import effective_weights as ew
    from model.flashinfer.packed_ops import project_qkv_packed
    from multilora.linear import LoRALinear

    g = torch.Generator().manual_seed(7)
    arrays: dict[str, np.ndarray] = {}

    def rnd(*shape, std=0.02, dtype=torch.float32):
        return (torch.randn(*shape, generator=g) * std).to(dtype)

    def lora_module(w, a, b, rank, alpha, bias=None):
        lin = nn.Linear(w.shape[1], w.shape[0], bias=bias is not None, dtype=w.dtype)
        with torch.no_grad():
            lin.weight.copy_(w)
            if bias is not None:
                lin.bias.copy_(bias)
        m = LoRALinear(lin, rank=rank, alpha=alpha, dropout=0.0)
        m.bind_serve(nn.Parameter(a.clone(), requires_grad=False), nn.Parameter(b.clone(), requires_grad=False))
        m.set_active_serve()
        return m

    # 1. LoRALinear.forward, fp32 and bf16, tokens 1..8, with and without bias.
    for dtype_name, dtype in (("f32", torch.float32), ("bf16", torch.bfloat16)):
        for case, (t, k, n, r, alpha, with_bias) in enumerate(
            [(1, 256, 192, 16, 32.0, False), (3, 512, 64, 8, 16.0, True), (8, 128, 320, 4, 12.0, False)]
        ):
            x = rnd(t, k, std=1.0, dtype=dtype)
            w = rnd(n, k, dtype=dtype)
            a = rnd(r, k, dtype=dtype)
            b = rnd(n, r, dtype=dtype)
            bias = rnd(n, std=0.1, dtype=dtype) if with_bias else None
            m = lora_module(w, a, b, r, alpha, bias)
            with torch.no_grad():
                y = m(x)
            pre = f"lora_linear_{dtype_name}_{case}_"
            arrays[pre + "x"] = _bf16_np(x)
            arrays[pre + "w"] = _bf16_np(w)
            arrays[pre + "a"] = _bf16_np(a)
            arrays[pre + "b"] = _bf16_np(b)
            arrays[pre + "bias"] = _bf16_np(bias) if bias is not None else np.zeros(0, np.float32)
            arrays[pre + "scale"] = np.array([alpha / r], np.float32)
            arrays[pre + "y"] = _bf16_np(y)

    # 2. Packed q/k/v projection with the packed LoRA delta (bf16).
    for case, (t, hidden, hq, hkv, d, r, alpha) in enumerate([(1, 256, 4, 2, 32, 16, 32.0), (4, 512, 8, 2, 64, 8, 16.0)]):
        dtype = torch.bfloat16
        x = rnd(1, t, hidden, std=1.0, dtype=dtype)
        mods = []
        for name, out_dim in (("q", hq * d), ("k", hkv * d), ("v", hkv * d)):
            w, a, b = rnd(out_dim, hidden, dtype=dtype), rnd(r, hidden, dtype=dtype), rnd(out_dim, r, dtype=dtype)
            mods.append(lora_module(w, a, b, r, alpha))
            pre = f"packed_{case}_{name}_"
            arrays[pre + "w"] = _bf16_np(w)
            arrays[pre + "a"] = _bf16_np(a)
            arrays[pre + "b"] = _bf16_np(b)
        attn = SimpleNamespace(q_proj=mods[0], k_proj=mods[1], v_proj=mods[2])
        plan = SimpleNamespace(modules={"self_attn.q_proj": mods[0], "self_attn.k_proj": mods[1],
                                        "self_attn.v_proj": mods[2]})
        with torch.no_grad():
            q, k, v = project_qkv_packed(SimpleNamespace(self_attn=attn), plan, x)
        pre = f"packed_{case}_"
        arrays[pre + "x"] = _bf16_np(x[0])
        arrays[pre + "scale"] = np.array([alpha / r], np.float32)
        arrays[pre + "q"] = _bf16_np(q[0])
        arrays[pre + "k"] = _bf16_np(k[0])
        arrays[pre + "v"] = _bf16_np(v[0])

    # 3. Merged weights: merge_serve_lora (mode 0), effective_linear (mode 0),
    #    effective_packed_linear (mode 1), unmerge (sign -1), bf16.
    os.environ["MINI_OPENCLAW_FLASHINFER_EFFECTIVE_WEIGHTS"] = "1"
    dtype = torch.bfloat16
    n, k, r, alpha = 96, 256, 16, 24.0
    w, a, b = rnd(n, k, dtype=dtype), rnd(r, k, dtype=dtype), rnd(n, r, dtype=dtype)
    arrays["merge_w"], arrays["merge_a"], arrays["merge_b"] = _bf16_np(w), _bf16_np(a), _bf16_np(b)
    arrays["merge_scale"] = np.array([alpha / r], np.float32)
    m = lora_module(w, a, b, r, alpha)
    eff = ew.effective_linear(m)
    arrays["merge_effective_linear"] = _bf16_np(eff.weight)
    m2 = lora_module(w, a, b, r, alpha)
    m3 = lora_module(w, a, b, r, alpha)
    owner = SimpleNamespace()
    packed = ew.effective_packed_linear(owner=owner, attr="_eff", modules=(m2, m3))
    arrays["merge_effective_packed"] = _bf16_np(packed.weight[:n])
    assert m.merge_serve_lora("adapter")
    arrays["merge_serve_merged"] = _bf16_np(m.weight)
    assert m.unmerge_serve_lora()
    arrays["merge_serve_unmerged"] = _bf16_np(m.weight)
    np.savez_compressed(out, **arrays)
    print(f"lora_cases.npz: {len(arrays)} arrays")


def make_lora_batched_cases(out: Path) -> None:
    """Batched-token LoRA surfaces: LoRALinear.forward, project_qkv_packed,
    project_gate_up_packed and project_qkv_with_optional_norm (bf16)."""

    os.environ["MINI_OPENCLAW_FLASHINFER_PACKED_QKV"] = "1"
    os.environ["MINI_OPENCLAW_FLASHINFER_PACKED_MLP"] = "1"
    os.environ["MINI_OPENCLAW_FLASHINFER_PACKED_LORA_DELTA"] = "1"
    os.environ["MINI_OPENCLAW_FLASHINFER_EFFECTIVE_WEIGHTS"] = "0"
    os.environ["MINI_OPENCLAW_FLASHINFER_QK_NORM"] = "0"
    from types import SimpleNamespace

    import torch.nn as nn
    from transformers.models.qwen3.modeling_qwen3 import Qwen3RMSNorm

    from model.flashinfer.packed_ops import project_gate_up_packed, project_qkv_packed
    from model.flashinfer.projection import project_qkv_with_optional_norm
    from multilora.linear import LoRALinear

    g = torch.Generator().manual_seed(11)
    bf = torch.bfloat16
    arrays: dict[str, np.ndarray] = {}

    def rnd(*shape, std=0.02):
        return (torch.randn(*shape, generator=g) * std).to(bf)

    def module(w, lora=None, bias=None):
        lin = nn.Linear(w.shape[1], w.shape[0], bias=bias is not None, dtype=bf)
        with torch.no_grad():
            lin.weight.copy_(w)
            if bias is not None:
                lin.bias.copy_(bias)
        if lora is None:
            return lin
        a, b, r, alpha = lora
        m = LoRALinear(lin, rank=r, alpha=alpha, dropout=0.0)
        m.bind_serve(nn.Parameter(a.clone(), requires_grad=False), nn.Parameter(b.clone(), requires_grad=False))
        m.set_active_serve()
        return m

    def put(prefix, **tensors):  # bf16 bit patterns as uint16 (half the fixture size)
        for k, v in tensors.items():
            arrays[prefix + k] = (np.zeros(0, np.uint16) if v is None
                                  else v.detach().contiguous().view(torch.int16).numpy().view(np.uint16))

    # 1. LoRALinear.forward at batched token counts ([T, K] and [1, T, K] inputs).
    for case, (t, k, n, r, alpha, with_bias, lead) in enumerate(
            [(16, 128, 192, 16, 32.0, False, False), (64, 128, 320, 8, 16.0, True, True),
             (128, 256, 128, 16, 32.0, False, False), (9, 384, 64, 16, 32.0, False, True)]):
        x = rnd(t, k, std=1.0)
        w, a, b = rnd(n, k), rnd(r, k), rnd(n, r)
        bias = rnd(n, std=0.1) if with_bias else None
        m = module(w, (a, b, r, alpha), bias)
        with torch.no_grad():
            y = m(x[None] if lead else x)
        put(f"linear_{case}_", x=x, w=w, a=a, b=b, bias=bias, y=y.reshape(t, n))
        arrays[f"linear_{case}_meta"] = np.array([r, alpha, int(lead)], np.float32)

    # 2. project_qkv_packed: packed delta (LoRA on q/k/v) and per-module deltas (LoRA on q/v).
    for case, (t, hidden, hq, hkv, d, r, alpha, targets) in enumerate(
            [(64, 128, 4, 2, 64, 16, 32.0, "qkv"), (16, 128, 4, 2, 64, 8, 16.0, "qv"),
             (128, 128, 2, 2, 64, 16, 32.0, "qkv")]):
        x = rnd(1, t, hidden, std=1.0)
        mods = []
        for name, od in (("q", hq * d), ("k", hkv * d), ("v", hkv * d)):
            w = rnd(od, hidden)
            lora = (rnd(r, hidden), rnd(od, r), r, alpha) if name in targets else None
            mods.append(module(w, lora))
            put(f"qkv_{case}_{name}_", w=w, a=None if lora is None else lora[0], b=None if lora is None else lora[1])
        attn = SimpleNamespace(q_proj=mods[0], k_proj=mods[1], v_proj=mods[2])
        plan = SimpleNamespace(modules={f"self_attn.{n}_proj": m for n, m in zip("qkv", mods)})
        with torch.no_grad():
            q, k, v = project_qkv_packed(SimpleNamespace(self_attn=attn), plan, x)
        put(f"qkv_{case}_", x=x[0], q=q[0], k=k[0], v=v[0])
        arrays[f"qkv_{case}_meta"] = np.array([r, alpha], np.float32)

    # 3. project_gate_up_packed: packed delta, per-module delta (LoRA on up only), no LoRA.
    for case, (t, hidden, inter, r, alpha, targets) in enumerate(
            [(64, 128, 256, 8, 16.0, "gu"), (16, 128, 192, 16, 32.0, "u"), (1, 256, 128, 16, 32.0, "")]):
        x = rnd(1, t, hidden, std=1.0)
        mods = {}
        for name in "gu":
            w = rnd(inter, hidden)
            lora = (rnd(r, hidden), rnd(inter, r), r, alpha) if name in targets else None
            mods[name] = module(w, lora)
            put(f"gu_{case}_{name}_", w=w, a=None if lora is None else lora[0], b=None if lora is None else lora[1])
        mlp = SimpleNamespace(gate_proj=mods["g"], up_proj=mods["u"])
        with torch.no_grad():
            y = project_gate_up_packed(mlp, x)
        put(f"gu_{case}_", x=x[0], y=y[0])
        arrays[f"gu_{case}_meta"] = np.array([r, alpha], np.float32)

    # 4. project_qkv_with_optional_norm on a Qwen3-style attention (q/k head norms).
    for case, (bsz, seqlen, hidden, hq, hkv, d, r, alpha) in enumerate(
            [(1, 1, 128, 4, 2, 64, 16, 32.0), (1, 64, 128, 4, 2, 64, 16, 32.0), (2, 32, 128, 4, 2, 128, 8, 16.0)]):
        x = rnd(bsz, seqlen, hidden, std=1.0)
        mods = []
        for name, od in (("q", hq * d), ("k", hkv * d), ("v", hkv * d)):
            w, a, b = rnd(od, hidden), rnd(r, hidden), rnd(od, r)
            mods.append(module(w, (a, b, r, alpha)))
            put(f"norm_{case}_{name}_", w=w, a=a, b=b)
        norms = []
        for name in "qk":
            nm = Qwen3RMSNorm(d, eps=1e-6).to(bf)
            with torch.no_grad():
                nm.weight.copy_((1.0 + torch.randn(d, generator=g) * 0.1).to(bf))
            norms.append(nm)
            put(f"norm_{case}_{name}norm_", w=nm.weight.detach())
        cfg = SimpleNamespace(num_attention_heads=hq, num_key_value_heads=hkv)
        attn = SimpleNamespace(config=cfg, head_dim=d, q_proj=mods[0], k_proj=mods[1], v_proj=mods[2],
                               q_norm=norms[0], k_norm=norms[1])
        plan = SimpleNamespace(modules={f"self_attn.{n}_proj": m for n, m in zip("qkv", mods)})
        with torch.no_grad():
            res = project_qkv_with_optional_norm(SimpleNamespace(self_attn=attn), plan, x)
        put(f"norm_{case}_", x=x, q=res.q_bshd, k=res.k_bshd, v=res.v_bshd)
        arrays[f"norm_{case}_meta"] = np.array([bsz, seqlen, hq, hkv, d, r, alpha], np.float32)
    np.savez_compressed(out, **arrays)
    print(f"lora_batched_cases.npz: {len(arrays)} arrays")



def make_tiny_greedy(out: Path) -> None:
    import torch.nn as nn
    from transformers import LlamaConfig, LlamaForCausalLM

    from multilora.linear import LoRALinear

    sys.path.insert(0, str(REPO))
    from pagelora_b200.synthetic import WORKLOADS, make_lora_weights, make_model_weights, random_prompt

    wl = WORKLOADS["config1"]
    spec, lspec = wl.model, wl.lora
    cfg = LlamaConfig(vocab_size=spec.vocab, hidden_size=spec.hidden, intermediate_size=spec.intermediate,
                      num_hidden_layers=spec.num_layers, num_attention_heads=spec.num_qo_heads,
                      num_key_value_heads=spec.num_kv_heads, head_dim=spec.head_dim, rms_norm_eps=spec.rms_eps,
                      rope_theta=spec.rope_theta, max_position_embeddings=4096, tie_word_embeddings=False,
                      attention_bias=False, mlp_bias=False)
    cfg._attn_implementation = "eager"
    torch.manual_seed(0)
    model = LlamaForCausalLM(cfg).float().eval()
    weights = make_model_weights(spec, seed=0, dtype=torch.float32)
    missing, unexpected = model.load_state_dict(weights, strict=False)
    assert not unexpected and all("rotary" in m for m in missing), (missing, unexpected)
    loras = make_lora_weights(spec, lspec, dtype=torch.float32)
    for i, layer in enumerate(model.model.layers):
        for t in lspec.targets:
            name = f"{t}_proj"
            wrapped = LoRALinear(getattr(layer.self_attn, name), rank=lspec.rank, alpha=lspec.alpha, dropout=0.0)
            a, b = loras[f"layers.{i}.{t}"]
            wrapped.bind_serve(nn.Parameter(a.clone(), requires_grad=False),
                               nn.Parameter(b.clone(), requires_grad=False))
            wrapped.set_active_serve()
            setattr(layer.self_attn, name, wrapped)
    prompt = random_prompt(spec.vocab, wl.prompt_len, seed=0)
    ids = torch.tensor([prompt])
    with torch.no_grad():
        res = model.generate(input_ids=ids, attention_mask=torch.ones_like(ids), max_new_tokens=wl.decode_tokens,
                             do_sample=False, eos_token_id=None, pad_token_id=0, return_dict_in_generate=True,
                             output_logits=True, repetition_penalty=1.0)
    new = res.sequences[0, len(prompt):].tolist()
    first_logits = res.logits[0][0].float().numpy()
    checksum = float(sum(float(v.double().sum()) for v in weights.values()))
    np.savez_compressed(out, prompt=np.array(prompt, np.int64), tokens=np.array(new, np.int64),
                        first_logits=first_logits.astype(np.float32), weight_checksum=np.array([checksum]))
    print(f"tiny_llama_greedy.npz: tokens {new[:8]}... checksum {checksum:.6f}")


def make_prefix_plans(out: Path) -> None:
    """model/kvcache/paged_kvcache_manager.py on CPU: commit cached prompts,
    then begin requests (single and branch batches, the config-4 shape at
    page 16) and record each radix lookup result (key_match_len, key_spans)
    with the request's match_len / prefill_from / prefix_spans, the batch page
    table and the admission answers."""

    from model.kvcache.flashinfer_page_table import build_flashinfer_batch_page_table
    from model.kvcache.paged_kvcache_manager import FlashInferPagedKVCacheManager
    from model.kvcache.radix_types import FULL_KEY

    def spans_of(spans):
        return [[int(s.block_id), int(s.start), int(s.length)] for s in spans]

    rng = random.Random(4)
    cases = []
    scenarios = [
        # (page_size, committed prompt lengths, new prompts as (base index, shared len, extra len))
        (16, [2048], [(0, 2048, 64)] * 16),               # config 4: shared prefix + 64-token suffixes
        (16, [2050], [(0, 2050, 64), (0, 2050, 0), (0, 2049, 5), (0, 17, 3)]),
        (16, [100, 40], [(0, 100, 0), (1, 33, 10), (0, 96, 1), (1, 0, 7)]),
        (4, [9, 13], [(0, 9, 2), (1, 13, 0), (1, 8, 8), (0, 4, 0)]),
    ]
    for ps, committed, news in scenarios:
        mgr = FlashInferPagedKVCacheManager(num_layers=1, page_size=ps, max_pages=4096)
        bases = []
        for n in committed:
            toks = [rng.randrange(1, 32000) for _ in range(n)]
            req = mgr.begin_request(toks, "a")
            mgr.reserve_chunk(req, n - req.prefill_from)
            mgr.commit_request(req, toks)
            bases.append(toks)
        prompts = []
        for bi, shared, extra in news:
            prompts.append(bases[bi][:shared] + [rng.randrange(1, 32000) for _ in range(extra)])
        lookups = []
        for p in prompts:
            m = mgr._prefix_cache.lookup(p, keys=(FULL_KEY("a"),))
            lookups.append({"key_match_len": int(m.key_match_len.get(FULL_KEY("a"), 0)),
                            "key_spans": spans_of(m.key_spans.get(FULL_KEY("a"), []))})
        available = int(mgr.available_pages)
        reqs = mgr.begin_batch_requests(prompts, "a")
        rows = []
        for p, r, lk in zip(prompts, reqs, lookups):
            new = len(p) - r.prefill_from
            rows.append({"prompt_len": len(p), **lk, "match_len": int(r.match_len), "prefill_from": int(r.prefill_from),
                         "prefix_spans": spans_of(r.prefix_spans),
                         "new_pages": int(mgr.estimate_request_new_pages(r, prefill_tokens=new, max_decode_tokens=128)),
                         "fits": bool(mgr.can_fit_request(r, prefill_tokens=new, max_decode_tokens=128,
                                                          reserve_pages=len(prompts))),
                         "max_decode": int(mgr.max_decode_tokens_that_fit(r, prefill_tokens=new,
                                                                          requested_decode_tokens=100000,
                                                                          reserve_pages=len(prompts)))})
        for r in reqs:
            mgr.reserve_chunk(r, len(r.token_ids) - r.prefill_from)
        table = build_flashinfer_batch_page_table([r.prefix_spans + r.new_spans for r in reqs], page_size=ps,
                                                  device=torch.device("cpu"))
        cases.append({"page_size": ps, "available_pages": available, "rows": rows,
                      "row_spans": [spans_of(r.prefix_spans + r.new_spans) for r in reqs],
                      "indptr": table.paged_kv_indptr.tolist(), "indices": table.paged_kv_indices.tolist(),
                      "last_page_len": table.paged_kv_last_page_len.tolist()})
        mgr.abort_batch_requests(reqs)
    out.write_text(json.dumps({"source": "model/kvcache/paged_kvcache_manager.py", "cases": cases}))
    print(f"prefix_plans.json: {len(cases)} scenarios, {sum(len(c['rows']) for c in cases)} requests")


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("PAGELORA_REFERENCE"),
                    help="checkout of the PageLoRA reference (or set PAGELORA_REFERENCE)")
    ap.add_argument("--only", default="")
    args = ap.parse_args()
    if not args.reference:
        ap.error("--reference (or PAGELORA_REFERENCE) is required")
    sys.path.insert(0, args.reference)
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    todo = args.only.split(",") if args.only else ["page_tables", "lora", "lora_batched", "tiny", "prefix"]
    if "page_tables" in todo:
        make_page_tables(HERE / "page_tables.json")
    if "lora" in todo:
        make_lora_cases(HERE / "lora_cases.npz")
    if "lora_batched" in todo:
        make_lora_batched_cases(HERE / "lora_batched_cases.npz")
    if "tiny" in todo:
        make_tiny_greedy(HERE / "tiny_llama_greedy.npz")
    if "prefix" in todo:
        make_prefix_plans(HERE / "prefix_plans.json")


if __name__ == "__main__":
    main()
