"""The drop-in attention backend against the reference's own FlashInfer calls
at the benchmark workloads' layer shapes.

The reference's decode and prefill arithmetic is third-party: FlashInfer's
BatchDecodeWithPagedKVCacheWrapper / BatchPrefillWithPagedKVCacheWrapper,
called by model/flashinfer/attention_backend.py with q / 16 and
sm_scale = 16 / sqrt(D), pos_encoding_mode "NONE", the NHD page layout and,
for decode, the tensor-core kernel only for GQA groups outside {1, 2, 4, 8}
(attention_backend.py:41-56, 63-131, 133-190).  ``_flashinfer_decode`` and
``_flashinfer_prefill`` restate those calls against the FlashInfer library
of this image (0.6.11.post2; the reference pins 0.6.6), and every case runs
the same inputs through ``B200AttentionBackend``.

Bound, per output element: |B200 - FlashInfer| <= max(2e-2, 2^-7 |out|),
the stated bf16 tolerance or, for outputs above 2.56, one bf16 ulp (both
sides round a fp32 result to bf16); and max |B200 - FlashInfer| <= 2^-6 of
the largest output magnitude.  Inputs: q ~ N(0, 3^2) so that the softmax is
peaked, K and V ~ N(0, 1), pages drawn from a shuffled pool.
"""

from __future__ import annotations

import math

import pytest
import torch

pytestmark = pytest.mark.gpu

flashinfer = pytest.importorskip("flashinfer")


def _pool_and_table(lens, hkv, d, ps, *, seed, shared_prefix_pages=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    npg = [-(-L // ps) for L in lens]
    own = [n - shared_prefix_pages for n in npg]
    total = shared_prefix_pages + sum(own)
    pool_pages = total + 7
    cache = torch.randn((pool_pages, 2, ps, hkv, d), generator=g, device="cuda").bfloat16()
    perm = torch.randperm(pool_pages, generator=g, device="cuda").tolist()
    prefix, rest = perm[:shared_prefix_pages], perm[shared_prefix_pages:]
    indices, indptr = [], [0]
    for n in own:
        indices += prefix + rest[:n]
        rest = rest[n:]
        indptr.append(len(indices))
    last = [L - (n - 1) * ps for L, n in zip(lens, npg)]
    i32 = lambda a: torch.tensor(a, dtype=torch.int32, device="cuda")  # noqa: E731
    return cache, i32(indptr), i32(indices), i32(last)


def _flashinfer_decode(q, cache, indptr, indices, last, hq, hkv, d, ps):
    """attention_backend.py:41-56, 89-131 against the installed FlashInfer."""

    ws = torch.empty(128 << 20, dtype=torch.uint8, device="cuda")
    tensor_cores = hq // hkv not in (1, 2, 4, 8)
    try:
        wrapper = flashinfer.BatchDecodeWithPagedKVCacheWrapper(ws, kv_layout="NHD", use_tensor_cores=tensor_cores)
        wrapper.plan(indptr, indices, last, hq, hkv, d, ps, pos_encoding_mode="NONE", sm_scale=16.0 / math.sqrt(d),
                     q_data_type=torch.bfloat16, kv_data_type=torch.bfloat16)
        out = wrapper.run(q / 16.0, cache)
    except Exception as exc:  # JIT toolchain or version issues on the box
        pytest.skip(f"flashinfer decode unavailable: {exc}")
    return out[0] if isinstance(out, tuple) else out


def _flashinfer_prefill(q, cache, qo_indptr, indptr, indices, last, hq, hkv, d, ps, causal):
    """attention_backend.py:133-190 against the installed FlashInfer."""

    ws = torch.empty(128 << 20, dtype=torch.uint8, device="cuda")
    try:
        wrapper = flashinfer.BatchPrefillWithPagedKVCacheWrapper(ws, kv_layout="NHD")
        wrapper.plan(qo_indptr, indptr, indices, last, hq, hkv, d, ps, causal=causal, pos_encoding_mode="NONE",
                     sm_scale=16.0 / math.sqrt(d), q_data_type=torch.bfloat16, kv_data_type=torch.bfloat16)
        out = wrapper.run(q / 16.0, cache)
    except Exception as exc:
        pytest.skip(f"flashinfer prefill unavailable: {exc}")
    return out[0] if isinstance(out, tuple) else out


def _check(mine, ref, label):
    diff = (mine.float() - ref.float()).abs()
    err = diff.max().item()
    scale = ref.float().abs().max().item()
    print(f"{label}: max |B200 - FlashInfer {flashinfer.__version__}| = {err:.3e} (max |out| {scale:.3e})")
    bound = torch.clamp(ref.float().abs() * 2.0 ** -7, min=2e-2)
    assert bool((diff <= bound).all()), (err, scale)
    assert err <= scale * 2.0 ** -6, (err, scale)


DECODE_CASES = {
    # name: (lens, hq, hkv, shared prefix pages)
    "config2_qwen3_8b_ctx2112": ([2112], 32, 8, 0),
    "config3_llama2_7b_64rows": (None, 32, 32, 0),  # lens U[512, 4096], seed 0
    "config4_qwen3_8b_16branches": ([2048 + 64 + 5] * 16, 32, 8, 128),
    "config5_llama3_8b_8x32k": ([32768] * 8, 32, 8, 0),
}


@pytest.mark.parametrize("case", list(DECODE_CASES))
def test_decode_matches_flashinfer_at_workload_shapes(cuda_device, case):
    from pagelora_b200.attention_backend import B200AttentionBackend

    lens, hq, hkv, shared = DECODE_CASES[case]
    if lens is None:
        g = torch.Generator().manual_seed(0)
        lens = torch.randint(512, 4097, (64,), generator=g).tolist()
    d, ps = 128, 16
    cache, indptr, indices, last = _pool_and_table(lens, hkv, d, ps, seed=11, shared_prefix_pages=shared)
    q = (3.0 * torch.randn((len(lens), hq, d), generator=torch.Generator(device="cuda").manual_seed(5),
                           device="cuda")).bfloat16()
    ref = _flashinfer_decode(q, cache, indptr, indices, last, hq, hkv, d, ps)
    be = B200AttentionBackend(device=cuda_device, workspace_mb=128, num_qo_heads=hq, num_kv_heads=hkv, head_dim=d,
                              page_size=ps)
    be.plan_decode(paged_kv_indptr=indptr, paged_kv_indices=indices, paged_kv_last_page_len=last,
                   q_data_type=torch.bfloat16, kv_data_type=torch.bfloat16)
    mine = be.run_decode(q.unsqueeze(2), cache)[:, :, 0]
    torch.cuda.synchronize()
    assert int(be.status.item()) == 0
    _check(mine, ref, f"decode {case}")


PREFILL_CASES = {
    # name: (query lens, kv lens, hq, hkv, causal)
    "qwen3_ragged_causal_with_cached_prefix": ([37, 1, 200, 64], [37, 129, 512, 64], 32, 8, True),
    "qwen3_prompt_2048_causal": ([2048], [2048], 32, 8, True),
    "llama2_mha_ragged_causal": ([100, 300], [164, 300], 32, 32, True),
    "qwen3_ragged_noncausal": ([16, 48], [80, 48], 32, 8, False),
}


@pytest.mark.parametrize("case", list(PREFILL_CASES))
def test_prefill_matches_flashinfer(cuda_device, case):
    from pagelora_b200.attention_backend import B200AttentionBackend

    qlens, kvlens, hq, hkv, causal = PREFILL_CASES[case]
    d, ps = 128, 16
    cache, indptr, indices, last = _pool_and_table(kvlens, hkv, d, ps, seed=3)
    qo = [0]
    for n in qlens:
        qo.append(qo[-1] + n)
    qo_indptr = torch.tensor(qo, dtype=torch.int32, device="cuda")
    q = (3.0 * torch.randn((qo[-1], hq, d), generator=torch.Generator(device="cuda").manual_seed(9),
                           device="cuda")).bfloat16()
    ref = _flashinfer_prefill(q, cache, qo_indptr, indptr, indices, last, hq, hkv, d, ps, causal)
    be = B200AttentionBackend(device=cuda_device, workspace_mb=16, num_qo_heads=hq, num_kv_heads=hkv, head_dim=d,
                              page_size=ps)
    be.plan_prefill(qo_indptr=qo_indptr, paged_kv_indptr=indptr, paged_kv_indices=indices,
                    paged_kv_last_page_len=last, causal=causal, q_data_type=torch.bfloat16,
                    kv_data_type=torch.bfloat16)
    mine = be.run_prefill(q, cache)
    torch.cuda.synchronize()
    assert int(be.status.item()) == 0
    _check(mine, ref, f"prefill {case}")
