"""The drop-in surfaces (attention backend, page tables, LoRA linear) behave
like the reference's classes and match its outputs.  The reference's own
FlashInfer decode wrapper, when the library is importable on the box, is run
on the same inputs as a second parity anchor."""

from __future__ import annotations

import json
import math

import numpy as np
import pytest
import torch
import torch.nn as nn

from oracle import lora as olora
from oracle import page_table as opt
from oracle.numerics import bf16
from oracle.paged_decode import paged_decode as o_decode

pytestmark = pytest.mark.gpu


def _t(a, dtype=torch.bfloat16):
    return torch.as_tensor(np.asarray(a, dtype=np.float32)).to(device="cuda", dtype=dtype)


def _ulps_close(actual, expected, magnitude, ulps=2):
    actual, expected = np.asarray(actual, np.float32), np.asarray(expected, np.float32)
    mag = np.maximum(np.abs(expected), np.abs(magnitude))
    tol = ulps * np.maximum(mag, 1e-3) * 2.0 ** -8 + 1e-6
    over = np.abs(actual - expected) - tol
    if (over > 0).any():
        i = np.unravel_index(int(np.argmax(over)), over.shape)
        raise AssertionError(f"{int((over > 0).sum())} elements beyond {ulps} ulps; worst at {i}: "
                             f"got {actual[i]!r}, expected {expected[i]!r}, magnitude {np.abs(magnitude)[i]!r}")


def _paged_inputs(seed=0, batch=3, hq=32, hkv=8, d=128, ps=16, lens=(1, 40, 300)):
    rng = np.random.default_rng(seed)
    npg = [-(-L // ps) for L in lens]
    pool = sum(npg) + 5
    cache = bf16(rng.normal(size=(pool, 2, ps, hkv, d)))
    indices = rng.permutation(pool)[: sum(npg)].tolist()
    indptr = np.cumsum([0] + npg).tolist()
    last = [L - (n - 1) * ps for L, n in zip(lens, npg)]
    q = bf16(rng.normal(size=(batch, hq, 1, d)))
    return q, cache, indptr, indices, last


def test_attention_backend_plan_run_matches_oracle(cuda_device):
    from pagelora_b200.attention_backend import FlashInferAttentionBackend

    q, cache, indptr, indices, last = _paged_inputs()
    be = FlashInferAttentionBackend(device=cuda_device, workspace_mb=16, num_qo_heads=32, num_kv_heads=8,
                                    head_dim=128, page_size=16)
    be.plan_decode(paged_kv_indptr=torch.tensor(indptr, dtype=torch.int32, device="cuda"),
                   paged_kv_indices=torch.tensor(indices, dtype=torch.int32, device="cuda"),
                   paged_kv_last_page_len=torch.tensor(last, dtype=torch.int32, device="cuda"),
                   q_data_type=torch.bfloat16, kv_data_type=torch.bfloat16)
    out = be.run_decode(_t(q), _t(cache))
    assert out.shape == (3, 32, 1, 128)  # attention_backend.py:131 unsqueezes the NHD output
    ref, _ = o_decode(q[:, :, 0], cache, indptr, indices, last)
    assert np.max(np.abs(out[:, :, 0].float().cpu().numpy() - ref)) <= 2e-2
    # NHD query input returns [B, Hq, 1, D] as well
    out2 = be.run_decode(_t(q[:, :, 0]), _t(cache))
    assert torch.equal(out2, out)
    # pinned host metadata uses the async upload path with retained sources
    be.plan_decode(paged_kv_indptr=torch.tensor(indptr, dtype=torch.int32).pin_memory(),
                   paged_kv_indices=torch.tensor(indices, dtype=torch.int32).pin_memory(),
                   paged_kv_last_page_len=torch.tensor(last, dtype=torch.int32).pin_memory())
    assert len(be._decode_host_uploads) == 1
    out3 = be.run_decode(_t(q), _t(cache))
    assert torch.equal(out3, out)
    assert int(be.status.item()) == 0


def test_attention_backend_graph_signature_and_buffers(cuda_device):
    from pagelora_b200.attention_backend import B200AttentionBackend

    be = B200AttentionBackend(device=cuda_device, workspace_mb=1, num_qo_heads=28, num_kv_heads=4, head_dim=128,
                              page_size=32)
    assert be.decode_use_tensor_cores  # group 7, as the reference reports
    i32 = lambda a: torch.tensor(a, dtype=torch.int32, device="cuda")  # noqa: E731
    be.plan_decode(paged_kv_indptr=i32([0, 1]), paged_kv_indices=i32([0]), paged_kv_last_page_len=i32([1]))
    bufs = be._decode_graph_buffers
    sig = be.decode_graph_signature()
    be.plan_decode(paged_kv_indptr=i32([0, 1]), paged_kv_indices=i32([0]), paged_kv_last_page_len=i32([1]))
    assert be._decode_graph_buffers is bufs and be.decode_graph_signature() == sig
    be.plan_decode(paged_kv_indptr=i32([0, 17]), paged_kv_indices=i32(list(range(17))),
                   paged_kv_last_page_len=i32([3]))
    assert be._decode_graph_buffers is not bufs and be.decode_graph_signature() != sig
    with pytest.raises(ValueError):
        B200AttentionBackend(device=cuda_device, workspace_mb=1, num_qo_heads=28, num_kv_heads=5, head_dim=128,
                             page_size=16)


def test_attention_backend_prefill_matches_causal_attention(cuda_device):
    from pagelora_b200.attention_backend import B200AttentionBackend

    q, cache, indptr, indices, last = _paged_inputs(seed=1, batch=2, hq=8, hkv=2, d=64, lens=(20, 37))
    be = B200AttentionBackend(device=cuda_device, workspace_mb=1, num_qo_heads=8, num_kv_heads=2, head_dim=64,
                              page_size=16)
    qo = [0, 5, 12]  # the last 5 and 7 positions of each row
    rng = np.random.default_rng(2)
    qn = bf16(rng.normal(size=(12, 8, 64)))
    be.plan_prefill(qo_indptr=torch.tensor(qo), paged_kv_indptr=torch.tensor(indptr),
                    paged_kv_indices=torch.tensor(indices), paged_kv_last_page_len=torch.tensor(last))
    out = be.run_prefill(_t(qn), _t(cache)).float().cpu().numpy()
    for b, n_kv in enumerate((20, 37)):
        for j, qi in enumerate(range(qo[b], qo[b + 1])):
            visible = n_kv - (qo[b + 1] - qo[b]) + j + 1
            pages = indices[indptr[b]: indptr[b + 1]]
            sub_last = visible - (math.ceil(visible / 16) - 1) * 16
            ref, _ = o_decode(qn[qi][None], cache, [0, math.ceil(visible / 16)], pages[: math.ceil(visible / 16)],
                              [sub_last])
            assert np.max(np.abs(out[qi] - ref[0])) <= 2e-2


def test_page_table_mirror_matches_reference_fixture(cuda_device, golden_dir):
    from pagelora_b200.page_table import KVBlockSpan, build_flashinfer_batch_page_table

    cases = json.loads((golden_dir / "page_tables.json").read_text())
    for case in cases[:120]:
        spans = [[KVBlockSpan(*s) for s in row] for row in case["rows"]]
        if "error" in case:
            with pytest.raises(ValueError) as exc:
                build_flashinfer_batch_page_table(spans, page_size=case["page_size"], device=cuda_device)
            assert str(exc.value) == case["error"]
            continue
        t = build_flashinfer_batch_page_table(spans, page_size=case["page_size"], device=cuda_device)
        assert t.paged_kv_indptr.tolist() == case["indptr"]
        assert t.paged_kv_indices.tolist() == case["indices"]
        assert t.paged_kv_last_page_len.tolist() == case["last_page_len"]


def test_page_table_buffers_reuse_tensors(cuda_device):
    """test_paged_kvcache_manager.py:483-543 on the device builders."""

    from pagelora_b200.page_table import FlashInferBatchPageTableBuffer, FlashInferPageTableBuffer, KVBlockSpan

    buf = FlashInferPageTableBuffer(page_size=2, device=cuda_device, initial_capacity=1)
    first = buf.update_from_spans([KVBlockSpan(11, 0, 1)])
    second = buf.update_from_spans([KVBlockSpan(11, 0, 2), KVBlockSpan(12, 0, 1)])
    assert second.paged_kv_indptr is first.paged_kv_indptr
    assert second.paged_kv_last_page_len is first.paged_kv_last_page_len
    assert second.paged_kv_indptr.tolist() == [0, 2]
    assert second.paged_kv_indices.tolist() == [11, 12]
    assert second.paged_kv_last_page_len.tolist() == [1]
    bb = FlashInferBatchPageTableBuffer(page_size=4, device=cuda_device)
    t1 = bb.update_from_batch_spans([[KVBlockSpan(2, 0, 3)], [KVBlockSpan(4, 0, 4)]])
    ptrs = (t1.paged_kv_indptr.data_ptr(), t1.paged_kv_indices.data_ptr(), t1.paged_kv_last_page_len.data_ptr())
    t2 = bb.update_from_batch_spans([[KVBlockSpan(2, 0, 4)], [KVBlockSpan(4, 0, 4), KVBlockSpan(5, 0, 1)]])
    assert (t2.paged_kv_indptr.data_ptr(), t2.paged_kv_indices.data_ptr(),
            t2.paged_kv_last_page_len.data_ptr()) == ptrs
    assert t2.paged_kv_indptr.tolist() == [0, 1, 3]
    assert t2.paged_kv_indices.tolist() == [2, 4, 5]
    assert t2.paged_kv_last_page_len.tolist() == [4, 1]


def _lora_module(w, a, b, rank, alpha, bias=None):
    from pagelora_b200.lora import LoRALinear

    lin = nn.Linear(w.shape[1], w.shape[0], bias=bias is not None, device="cuda", dtype=torch.bfloat16)
    with torch.no_grad():
        lin.weight.copy_(_t(w))
        if bias is not None:
            lin.bias.copy_(_t(bias))
    m = LoRALinear(lin, rank=rank, alpha=alpha, dropout=0.0)
    m.bind_serve(nn.Parameter(_t(a), requires_grad=False), nn.Parameter(_t(b), requires_grad=False))
    m.set_active_serve()
    return m


def test_lora_linear_mirror_matches_reference(cuda_device, golden_dir):
    z = np.load(golden_dir / "lora_cases.npz")
    with torch.no_grad():
        for case in range(3):
            pre = f"lora_linear_bf16_{case}_"
            sc = float(z[pre + "scale"][0])
            r = z[pre + "a"].shape[0]
            bias = z[pre + "bias"] if z[pre + "bias"].size else None
            m = _lora_module(z[pre + "w"], z[pre + "a"], z[pre + "b"], r, sc * r, bias)
            y = m(_t(z[pre + "x"]))
            base = olora.linear(z[pre + "x"], z[pre + "w"], bias, bf16=True)
            _ulps_close(y.float().cpu().numpy(), z[pre + "y"], base)
            base2, down = m(_t(z[pre + "x"]), return_lora_down=True)
            _ulps_close(base2.float().cpu().numpy(), base, base)
            m.set_active_base()
            _ulps_close(m(_t(z[pre + "x"])).float().cpu().numpy(), base, base)


def test_merge_and_effective_weights_match_reference(cuda_device, golden_dir, monkeypatch):
    from types import SimpleNamespace

    from pagelora_b200 import lora as pl_lora

    monkeypatch.setenv("MINI_OPENCLAW_FLASHINFER_EFFECTIVE_WEIGHTS", "1")
    z = np.load(golden_dir / "lora_cases.npz")
    w, a, b, sc = z["merge_w"], z["merge_a"], z["merge_b"], float(z["merge_scale"][0])
    r = a.shape[0]
    mag = np.abs(w) + 1.0
    with torch.no_grad():
        m = _lora_module(w, a, b, r, sc * r)
        eff = pl_lora.effective_linear(m)
        _ulps_close(eff.weight.float().cpu().numpy(), z["merge_effective_linear"], mag)
        assert pl_lora.effective_linear(m) is eff  # cached
        packed = pl_lora.effective_packed_linear(owner=SimpleNamespace(), attr="_e",
                                                 modules=(_lora_module(w, a, b, r, sc * r),
                                                          _lora_module(w, a, b, r, sc * r)))
        _ulps_close(packed.weight[: w.shape[0]].float().cpu().numpy(), z["merge_effective_packed"], mag)
        assert m.merge_serve_lora("adapter")
        _ulps_close(m.weight.float().cpu().numpy(), z["merge_serve_merged"], mag)
        assert m.unmerge_serve_lora()
        _ulps_close(m.weight.float().cpu().numpy(), z["merge_serve_unmerged"], mag)
        pl_lora.clear_flashinfer_effective_weight_cache(m)
        assert not hasattr(m, "_flashinfer_effective_linear")


def test_project_qkv_packed_mirror_matches_reference(cuda_device, golden_dir, monkeypatch):
    from types import SimpleNamespace

    from pagelora_b200.lora import project_qkv_packed

    monkeypatch.setenv("MINI_OPENCLAW_FLASHINFER_EFFECTIVE_WEIGHTS", "0")
    z = np.load(golden_dir / "lora_cases.npz")
    with torch.no_grad():
        for case in range(2):
            pre = f"packed_{case}_"
            sc = float(z[pre + "scale"][0])
            mods = []
            for m in "qkv":
                r = z[f"{pre}{m}_a"].shape[0]
                mods.append(_lora_module(z[f"{pre}{m}_w"], z[f"{pre}{m}_a"], z[f"{pre}{m}_b"], r, sc * r))
            attn = SimpleNamespace(q_proj=mods[0], k_proj=mods[1], v_proj=mods[2])
            plan = SimpleNamespace(modules={"self_attn.q_proj": mods[0], "self_attn.k_proj": mods[1],
                                            "self_attn.v_proj": mods[2]})
            x = z[pre + "x"]
            q, k, v = project_qkv_packed(SimpleNamespace(self_attn=attn), plan, _t(x)[None])
            w_cat = np.concatenate([z[f"{pre}{m}_w"] for m in "qkv"])
            base = olora.linear(x, w_cat, bf16=True)
            got = torch.cat([q[0], k[0], v[0]], -1).float().cpu().numpy()
            _ulps_close(got, np.concatenate([z[pre + "q"], z[pre + "k"], z[pre + "v"]], -1), base)


def test_decode_matches_flashinfer_reference_path(cuda_device):
    """The reference's decode call (attention_backend.py:97,128: q/16 with
    sm_scale 16/sqrt(D), pos_encoding NONE, NHD) through the FlashInfer
    library installed on this image, against the B200 kernel."""

    flashinfer = pytest.importorskip("flashinfer")
    from pagelora_b200 import kernels as K

    q, cache, indptr, indices, last = _paged_inputs(seed=7, batch=4, lens=(16, 2112, 33, 700))
    qd, cd = _t(q[:, :, 0]), _t(cache)
    ws = torch.zeros(128 << 20, dtype=torch.uint8, device="cuda")
    try:
        wrapper = flashinfer.BatchDecodeWithPagedKVCacheWrapper(ws, kv_layout="NHD")
        wrapper.plan(torch.tensor(indptr, dtype=torch.int32, device="cuda"),
                     torch.tensor(indices, dtype=torch.int32, device="cuda"),
                     torch.tensor(last, dtype=torch.int32, device="cuda"), 32, 8, 128, 16,
                     pos_encoding_mode="NONE", sm_scale=16.0 / math.sqrt(128), q_data_type=torch.bfloat16,
                     kv_data_type=torch.bfloat16)
        ref = wrapper.run(qd / 16.0, cd)
    except Exception as exc:  # JIT toolchain or version issues on the box
        pytest.skip(f"flashinfer decode unavailable: {exc}")
    plan = K.decode_plan(4, 32, 8, 128, 16, len(indices))
    mine = K.paged_decode(qd, cd, torch.tensor(indptr, dtype=torch.int32, device="cuda"),
                          torch.tensor(indices, dtype=torch.int32, device="cuda"),
                          torch.tensor(last, dtype=torch.int32, device="cuda"), num_splits=plan.num_splits,
                          workspace=torch.zeros(max(1 << 16, plan.workspace_bytes), dtype=torch.uint8,
                                                device="cuda"))
    torch.cuda.synchronize()
    err = (mine.float() - ref.float()).abs().max().item()
    print(f"max |B200 - FlashInfer {flashinfer.__version__}| = {err:.3e}")
    assert err <= 2e-2


# ---------------------------------------------------------------- batched
def _bf(z, key):
    """A bf16 fixture array (stored as uint16 bit patterns) on the GPU, or None."""

    a = z[key]
    if a.size == 0:
        return None
    return torch.from_numpy(a.view(np.int16).copy()).view(torch.bfloat16).cuda()


def _same_bits_or_ulps(got, ref, base, ulps=3):
    """Within ``ulps`` units of 2^-8 |value| (two bf16 ulps in the worst binade
    position): the base projection, the LoRA down values and the delta may
    each round the other way when fp32 sums are ordered differently."""

    _ulps_close(*(t.detach().float().cpu().numpy() for t in (got, ref, base)), ulps)


def _lora_mod(w, a, b, rank, alpha, bias=None):
    from pagelora_b200.lora import LoRALinear

    lin = nn.Linear(w.shape[1], w.shape[0], bias=bias is not None, device="cuda", dtype=torch.bfloat16)
    with torch.no_grad():
        lin.weight.copy_(w)
        if bias is not None:
            lin.bias.copy_(bias)
    m = LoRALinear(lin, rank=rank, alpha=alpha, dropout=0.0)
    if a is not None:
        m.bind_serve(nn.Parameter(a, requires_grad=False), nn.Parameter(b, requires_grad=False))
        m.set_active_serve()
    return m


def test_batched_lora_linear_matches_reference(cuda_device, golden_dir, monkeypatch):
    """LoRALinear.forward at 9-128 tokens (the tcgen05 GEMM path) vs the
    reference module's bf16 outputs (multilora/linear.py:200-231)."""

    from pagelora_b200 import lora as L

    monkeypatch.setenv("MINI_OPENCLAW_FLASHINFER_EFFECTIVE_WEIGHTS", "0")
    z = np.load(golden_dir / "lora_batched_cases.npz")
    for case in range(4):
        p = f"linear_{case}_"
        r, alpha, lead = z[p + "meta"]
        x, w = _bf(z, p + "x"), _bf(z, p + "w")
        m = _lora_mod(w, _bf(z, p + "a"), _bf(z, p + "b"), int(r), float(alpha), _bf(z, p + "bias"))
        with torch.no_grad():
            assert L._kernel_kind(x, x.shape[1]) == "gemm", case
            y = m(x[None] if lead else x).reshape(x.shape[0], -1)
        _same_bits_or_ulps(y, _bf(z, p + "y"), torch.nn.functional.linear(x, w).float())


def test_batched_project_qkv_packed_matches_reference(cuda_device, golden_dir, monkeypatch):
    """project_qkv_packed at 16-128 tokens: the packed LoRA delta (q/k/v) and
    the per-module deltas (q/v only), packed_ops.py:105-165."""

    from types import SimpleNamespace

    from pagelora_b200.lora import project_qkv_packed

    monkeypatch.setenv("MINI_OPENCLAW_FLASHINFER_EFFECTIVE_WEIGHTS", "0")
    z = np.load(golden_dir / "lora_batched_cases.npz")
    for case in range(3):
        p = f"qkv_{case}_"
        r, alpha = z[p + "meta"]
        mods = [_lora_mod(_bf(z, f"{p}{n}_w"), _bf(z, f"{p}{n}_a"), _bf(z, f"{p}{n}_b"), int(r), float(alpha))
                for n in "qkv"]
        attn = SimpleNamespace(q_proj=mods[0], k_proj=mods[1], v_proj=mods[2])
        plan = SimpleNamespace(modules={f"self_attn.{n}_proj": m for n, m in zip("qkv", mods)})
        x = _bf(z, p + "x")
        with torch.no_grad():
            q, k, v = project_qkv_packed(SimpleNamespace(self_attn=attn), plan, x[None])
        base = torch.cat([torch.nn.functional.linear(x, m.weight.detach()) for m in mods], -1)
        got = torch.cat([q[0], k[0], v[0]], -1)
        ref = torch.cat([_bf(z, p + "q"), _bf(z, p + "k"), _bf(z, p + "v")], -1)
        try:
            _same_bits_or_ulps(got, ref, base)
        except AssertionError as exc:
            raise AssertionError(f"case {case}: {exc}") from None


def test_batched_project_gate_up_packed_matches_reference(cuda_device, golden_dir, monkeypatch):
    """project_gate_up_packed (packed_ops.py:168-203): packed delta, a delta on
    one module only, and no LoRA."""

    from types import SimpleNamespace

    from pagelora_b200.lora import project_gate_up_packed

    monkeypatch.setenv("MINI_OPENCLAW_FLASHINFER_EFFECTIVE_WEIGHTS", "0")
    z = np.load(golden_dir / "lora_batched_cases.npz")
    for case in range(3):
        p = f"gu_{case}_"
        r, alpha = z[p + "meta"]
        mods = {n: _lora_mod(_bf(z, f"{p}{n}_w"), _bf(z, f"{p}{n}_a"), _bf(z, f"{p}{n}_b"), int(r), float(alpha))
                for n in "gu"}
        mlp = SimpleNamespace(gate_proj=mods["g"], up_proj=mods["u"])
        x = _bf(z, p + "x")
        with torch.no_grad():
            y = project_gate_up_packed(mlp, x[None])[0]
        base = torch.cat([torch.nn.functional.linear(x, mods[n].weight.detach()) for n in "gu"], -1)
        _same_bits_or_ulps(y, _bf(z, p + "y"), base)


def test_project_qkv_with_optional_norm_matches_reference(cuda_device, golden_dir, monkeypatch):
    """project_qkv_with_optional_norm (projection.py:34-110) with Qwen3 q/k head
    norms in the Hugging Face rounding, at 1, 64 and 2 x 32 tokens."""

    from types import SimpleNamespace

    from pagelora_b200.lora import project_qkv_with_optional_norm

    monkeypatch.setenv("MINI_OPENCLAW_FLASHINFER_EFFECTIVE_WEIGHTS", "0")
    monkeypatch.setenv("MINI_OPENCLAW_FLASHINFER_QK_NORM", "0")
    z = np.load(golden_dir / "lora_batched_cases.npz")
    for case in range(3):
        p = f"norm_{case}_"
        bsz, seqlen, hq, hkv, d, r, alpha = (float(v) for v in z[p + "meta"])
        bsz, seqlen, hq, hkv, d, r = (int(v) for v in (bsz, seqlen, hq, hkv, d, r))
        mods = [_lora_mod(_bf(z, f"{p}{n}_w"), _bf(z, f"{p}{n}_a"), _bf(z, f"{p}{n}_b"), r, alpha) for n in "qkv"]
        norms = [SimpleNamespace(weight=_bf(z, f"{p}{n}norm_w"), variance_epsilon=1e-6) for n in "qk"]
        attn = SimpleNamespace(config=SimpleNamespace(num_attention_heads=hq, num_key_value_heads=hkv), head_dim=d,
                               q_proj=mods[0], k_proj=mods[1], v_proj=mods[2], q_norm=norms[0], k_norm=norms[1])
        plan = SimpleNamespace(modules={f"self_attn.{n}_proj": m for n, m in zip("qkv", mods)})
        x = _bf(z, p + "x")
        with torch.no_grad():
            res = project_qkv_with_optional_norm(SimpleNamespace(self_attn=attn), plan, x)
        for name, got in (("q", res.q_bshd), ("k", res.k_bshd), ("v", res.v_bshd)):
            ref = _bf(z, p + name)
            # head norms renormalise, so the magnitude scale is the output's own
            _same_bits_or_ulps(got.reshape(ref.shape), ref, ref)
        if bsz > 1:
            assert torch.equal(res.v_bhsd, res.v_bshd.transpose(1, 2))
