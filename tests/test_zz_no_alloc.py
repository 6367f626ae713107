"""pl_paged_decode_fixed_scratch (split partials in a fixed device array)
against pl_paged_decode (caller workspace), both called through the C ABI.

Collected last so that it runs both after every other GPU test and, with
`pytest tests/test_zz_no_alloc.py`, alone in a fresh process.  Outputs must
agree within the decode tolerance of the other kernel tests (max |err| <=
2e-2 on bf16 O, 1e-3 on the LSE) on two calls in a row.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle.numerics import bf16

pytestmark = pytest.mark.gpu

ATOL = 2e-2
FIXED_SCRATCH_BYTES = 4 * 1024 * 1024  # PL_FIXED_SCRATCH_BYTES


def _case(seed, *, batch_lens, hq, hkv, d, ps):
    rng = np.random.default_rng(seed)
    pages = [-(-L // ps) for L in batch_lens]
    total = sum(pages)
    pool = total + 5
    cache = bf16(rng.normal(size=(pool, 2, ps, hkv, d)))
    indices = rng.permutation(pool)[:total].astype(np.int32)
    indptr = np.cumsum([0] + pages).astype(np.int32)
    last = np.array([L - (n - 1) * ps if n else 0 for L, n in zip(batch_lens, pages)], np.int32)
    q = bf16(rng.normal(size=(len(batch_lens), hq, d)) * 1.5)
    dev = "cuda"
    return (
        torch.as_tensor(q).to(dev, torch.bfloat16),
        torch.as_tensor(cache).to(dev, torch.bfloat16),
        torch.as_tensor(indptr).to(dev),
        torch.as_tensor(indices if total else np.zeros(1, np.int32)).to(dev),
        torch.as_tensor(last).to(dev),
    )


def _run(fn, q, cache, indptr, indices, last, splits, workspace=None):
    from pagelora_b200._capi import call, ptr, stream_handle

    b, hq, d = q.shape
    pages, _, ps, hkv, _ = cache.shape
    out = torch.full_like(q, float("nan"))
    lse = torch.full((b, hq), float("nan"), dtype=torch.float32, device=q.device)
    status = torch.zeros(1, dtype=torch.int32, device=q.device)
    common = (ptr(q), q.stride(0), q.stride(1), ptr(cache), int(pages), ptr(indptr), ptr(indices), ptr(last),
              int(b), int(hq), int(hkv), int(d), int(ps), float(d) ** -0.5, int(splits), ptr(out), out.stride(0),
              out.stride(1), ptr(lse))
    if fn == "pl_paged_decode":
        call(fn, *common, ptr(workspace), workspace.numel(), ptr(status), stream_handle())
    else:
        call(fn, *common, ptr(status), stream_handle())
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    return out.float().cpu().numpy(), lse.cpu().numpy()


@pytest.mark.parametrize("hq,hkv,d,ps,splits", [(32, 8, 128, 16, 16), (16, 2, 64, 32, 3), (8, 8, 128, 16, 1)])
def test_fixed_scratch_matches_workspace_entry_point(cuda_device, hq, hkv, d, ps, splits):
    lens = [1, ps, ps + 1, 5 * ps - 3, 300, 0]
    ws = torch.zeros(8 << 20, dtype=torch.uint8, device="cuda")
    for seed in (11, 12):  # two calls in a row on different inputs
        args = _case(seed + hq + d, batch_lens=lens, hq=hq, hkv=hkv, d=d, ps=ps)
        ref_o, ref_lse = _run("pl_paged_decode", *args, splits, workspace=ws)
        o, lse = _run("pl_paged_decode_fixed_scratch", *args, splits)
        assert np.max(np.abs(o - ref_o)) <= ATOL
        np.testing.assert_allclose(lse, ref_lse, rtol=1e-3, atol=1e-3)
        assert np.all(o[-1] == 0) and np.all(np.isneginf(lse[-1]))
    # the same inputs twice: the counters left by the first call are zero
    args = _case(99, batch_lens=lens, hq=hq, hkv=hkv, d=d, ps=ps)
    first = _run("pl_paged_decode_fixed_scratch", *args, splits)
    second = _run("pl_paged_decode_fixed_scratch", *args, splits)
    ref_o, ref_lse = _run("pl_paged_decode", *args, splits, workspace=ws)
    for o, lse in (first, second):
        assert np.max(np.abs(o - ref_o)) <= ATOL
        np.testing.assert_allclose(lse, ref_lse, rtol=1e-3, atol=1e-3)


def test_fixed_scratch_calls_of_different_shapes_in_a_row(cuda_device):
    """The array is shared by every call: a call with few (row, kv head)
    pairs followed by one with many must still find zeroed counters."""

    small = _case(31, batch_lens=[300, 17], hq=32, hkv=8, d=128, ps=16)
    large = _case(32, batch_lens=[40, 300, 1, 77, 500, 16, 33], hq=16, hkv=16, d=128, ps=16)
    ws = {k: torch.zeros(8 << 20, dtype=torch.uint8, device="cuda") for k in ("s", "l")}
    for _ in range(2):
        for name, args in (("s", small), ("l", large)):
            ref_o, ref_lse = _run("pl_paged_decode", *args, 7, workspace=ws[name])
            o, lse = _run("pl_paged_decode_fixed_scratch", *args, 7)
            assert np.max(np.abs(o - ref_o)) <= ATOL
            np.testing.assert_allclose(lse, ref_lse, rtol=1e-3, atol=1e-3)


def test_fixed_scratch_rejects_shapes_beyond_its_size(cuda_device):
    from pagelora_b200._capi import PL_ERR_WORKSPACE_TOO_SMALL, PageLoRAError

    # partials alone: batch * hq * splits * d * 4 bytes = 64 * 32 * 64 * 128 * 4 = 64 MiB
    batch, hq, hkv, d, ps, splits = 64, 32, 8, 128, 16, 64
    assert batch * hq * splits * d * 4 > FIXED_SCRATCH_BYTES
    args = _case(3, batch_lens=[20] * batch, hq=hq, hkv=hkv, d=d, ps=ps)
    with pytest.raises(PageLoRAError) as err:
        _run("pl_paged_decode_fixed_scratch", *args, splits)
    assert err.value.status == PL_ERR_WORKSPACE_TOO_SMALL


def test_fixed_scratch_rejects_too_many_row_head_pairs(cuda_device):
    """The counter region holds 16384 (row, kv head) pairs: 2100 rows x 8 kv
    heads is rejected before any launch, even with one split (no partials)."""

    from pagelora_b200._capi import PL_ERR_WORKSPACE_TOO_SMALL, PageLoRAError, call, ptr, stream_handle

    batch, hq, hkv, d, ps = 2100, 32, 8, 128, 16
    assert batch * hkv > 16384
    q = torch.zeros((batch, hq, d), dtype=torch.bfloat16, device="cuda")
    cache = torch.zeros((1, 2, ps, hkv, d), dtype=torch.bfloat16, device="cuda")
    indptr = torch.zeros(batch + 1, dtype=torch.int32, device="cuda")
    indices = torch.zeros(1, dtype=torch.int32, device="cuda")
    last = torch.zeros(batch, dtype=torch.int32, device="cuda")
    out = torch.zeros_like(q)
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    with pytest.raises(PageLoRAError) as err:
        call("pl_paged_decode_fixed_scratch", ptr(q), q.stride(0), q.stride(1), ptr(cache), 1, ptr(indptr),
             ptr(indices), ptr(last), batch, hq, hkv, d, ps, d ** -0.5, 1, ptr(out), out.stride(0), out.stride(1),
             None, ptr(status), stream_handle())
    assert err.value.status == PL_ERR_WORKSPACE_TOO_SMALL


def test_fixed_scratch_clear_then_calls_match(cuda_device):
    """pl_fixed_scratch_clear (the reset after a PL_ERR_TIMEOUT status) leaves
    the array ready: the following calls match the workspace entry point."""

    from pagelora_b200._capi import call, stream_handle

    args = _case(41, batch_lens=[300, 17, 1000], hq=32, hkv=8, d=128, ps=16)
    ws = torch.zeros(8 << 20, dtype=torch.uint8, device="cuda")
    ref_o, ref_lse = _run("pl_paged_decode", *args, 9, workspace=ws)
    for _ in range(2):
        call("pl_fixed_scratch_clear", stream_handle())
        o, lse = _run("pl_paged_decode_fixed_scratch", *args, 9)
        assert np.max(np.abs(o - ref_o)) <= ATOL
        np.testing.assert_allclose(lse, ref_lse, rtol=1e-3, atol=1e-3)
