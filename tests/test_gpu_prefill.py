"""Parity of the tcgen05 paged prefill kernel (pl_paged_prefill, called
through the C ABI) with the CPU oracle.

bf16 outputs must be within max |err| <= 2e-2 of the fp64 restatement
(oracle/paged_prefill.py, the tolerance stated for this path) and the LSE
within 2e-3.  The pool is filled with NaN everywhere except the tokens the
requests own, so slots past a request's last token and unused pages must
never reach the result.  Long causal cases use a plain PyTorch fp32
attention of the same op as the reference (the fp64 oracle is too slow
there).
"""

from __future__ import annotations

import math

import numpy as np
import pytest
import torch

from oracle.paged_prefill import paged_prefill as o_prefill

pytestmark = pytest.mark.gpu

ATOL = 2e-2


@pytest.fixture(scope="module")
def K(cuda_device):
    from pagelora_b200 import kernels

    return kernels


def _case(reqs, hq, hkv, d, ps, seed, poison=True, extra_pages=5):
    """reqs: (qo_len, kv_len) per request; the queries are the last qo_len
    of the kv_len positions.  Returns numpy and device copies."""

    rng = np.random.default_rng(seed)
    n_pages = [-(-kv // ps) for _, kv in reqs]
    total_pages = sum(n_pages) + extra_pages
    perm = rng.permutation(total_pages)
    fill = np.nan if poison else 0.0
    cache = np.full((total_pages, 2, ps, hkv, d), fill, dtype=np.float32)
    kv_indptr, kv_indices, last = [0], [], []
    p = 0
    for (_, kv), n in zip(reqs, n_pages):
        pages = [int(x) for x in perm[p:p + n]]
        p += n
        kv_indices += pages
        kv_indptr.append(len(kv_indices))
        last.append(kv - (n - 1) * ps if n else 0)
        for t in range(kv):
            pg, off = pages[t // ps], t % ps
            cache[pg, :, off] = rng.normal(size=(2, hkv, d))
    qo_indptr = np.cumsum([0] + [q for q, _ in reqs]).tolist()
    q = rng.normal(size=(qo_indptr[-1], hq, d)).astype(np.float32)
    # bf16 round trip so that the oracle sees the kernel's inputs
    cache_t = torch.as_tensor(cache).to(torch.bfloat16)
    q_t = torch.as_tensor(q).to(torch.bfloat16)
    host = dict(q=q_t.float().numpy(), cache=cache_t.float().numpy(), qo_indptr=qo_indptr, kv_indptr=kv_indptr,
                kv_indices=kv_indices or [0], last=last)
    dev = dict(q=q_t.cuda(), cache=cache_t.cuda(),
               qo_indptr=torch.tensor(qo_indptr, dtype=torch.int32, device="cuda"),
               kv_indptr=torch.tensor(kv_indptr, dtype=torch.int32, device="cuda"),
               kv_indices=torch.tensor(kv_indices or [0], dtype=torch.int32, device="cuda"),
               last=torch.tensor(last, dtype=torch.int32, device="cuda"))
    return host, dev


def _run(K, dev, causal, lse=False):
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    out_lse = (torch.full(dev["q"].shape[:2], 7.0, dtype=torch.float32, device="cuda") if lse else None)
    out = K.paged_prefill(dev["q"], dev["cache"], dev["qo_indptr"], dev["kv_indptr"], dev["kv_indices"],
                          dev["last"], causal=causal, out_lse=out_lse, status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    return out, out_lse


# ragged batch: single token, multi-tile, cached prefix, empty request, a
# request whose last page is partial, one exactly tile-sized
REQS = [(37, 37), (1, 1), (130, 194), (0, 20), (300, 317), (128, 128), (5, 260)]


@pytest.mark.parametrize("d,ps", [(128, 16), (128, 32), (64, 16), (128, 64)])
@pytest.mark.parametrize("hq,hkv", [(32, 8), (8, 8), (28, 4), (16, 1)])
@pytest.mark.parametrize("causal", [True, False])
def test_prefill_matches_oracle(K, d, ps, hq, hkv, causal):
    reqs = REQS if hq * d <= 2048 else REQS[:5]
    host, dev = _case(reqs, hq, hkv, d, ps, seed=hq * 7 + d + ps)
    out, lse = _run(K, dev, causal, lse=True)
    want, want_lse = o_prefill(host["q"], host["cache"], host["qo_indptr"], host["kv_indptr"], host["kv_indices"],
                               host["last"], causal=causal)
    got = out.float().cpu().numpy()
    assert np.isfinite(got).all()
    err = np.abs(got - want).max()
    assert err <= ATOL, err
    got_lse = lse.cpu().numpy()
    assert np.allclose(got_lse, want_lse, atol=2e-3, rtol=0), np.abs(got_lse - want_lse).max()


def test_prefill_last_row_equals_decode(K):
    """The last query of each request sees exactly what a decode of that
    token sees: prefill's last rows equal pl_paged_decode on the same pages."""

    reqs = [(40, 100), (17, 17), (64, 300)]
    host, dev = _case(reqs, 32, 8, 128, 16, seed=5)
    out, _ = _run(K, dev, True)
    last_rows = torch.tensor([q1 - 1 for q1 in host["qo_indptr"][1:]], device="cuda")
    q_dec = dev["q"][last_rows].contiguous()
    plan = K.decode_plan(len(reqs), 32, 8, 128, 16, len(host["kv_indices"]))
    ws = torch.zeros(max(256, int(plan.workspace_bytes)), dtype=torch.uint8, device="cuda")
    dec = K.paged_decode(q_dec, dev["cache"], dev["kv_indptr"], dev["kv_indices"], dev["last"],
                         num_splits=int(plan.num_splits), workspace=ws)
    torch.cuda.synchronize()
    diff = (out[last_rows].float() - dec.float()).abs().max().item()
    assert diff <= ATOL, diff


def _torch_reference(q, cache, qo_indptr, kv_indptr, kv_indices, last, causal):
    """Plain PyTorch fp32 attention of the same op (gathered pages)."""

    total_q, hq, d = q.shape
    _, _, ps, hkv, _ = cache.shape
    group = hq // hkv
    out = torch.zeros(total_q, hq, d, dtype=torch.float32, device=q.device)
    for b in range(len(qo_indptr) - 1):
        q0, q1 = qo_indptr[b], qo_indptr[b + 1]
        pages = kv_indices[kv_indptr[b]:kv_indptr[b + 1]]
        n_kv = (len(pages) - 1) * ps + last[b]
        k = cache[pages, 0].reshape(-1, hkv, d)[:n_kv].float().repeat_interleave(group, dim=1)
        v = cache[pages, 1].reshape(-1, hkv, d)[:n_kv].float().repeat_interleave(group, dim=1)
        s = torch.einsum("qhd,khd->hqk", q[q0:q1].float(), k) / math.sqrt(d)
        if causal:
            i = torch.arange(q1 - q0, device=q.device)[:, None] + (n_kv - (q1 - q0))
            j = torch.arange(n_kv, device=q.device)[None, :]
            s = s.masked_fill(j > i, float("-inf"))
        out[q0:q1] = torch.einsum("hqk,khd->qhd", torch.softmax(s, dim=-1), v)
    return out


@pytest.mark.parametrize("qo,kv", [(2048, 2048), (1000, 3000)])
def test_prefill_long_causal_vs_torch_fp32(K, qo, kv):
    host, dev = _case([(qo, kv)], 32, 8, 128, 16, seed=qo + kv, poison=False)
    out, _ = _run(K, dev, True)
    ref = _torch_reference(dev["q"], dev["cache"], host["qo_indptr"], host["kv_indptr"],
                           torch.tensor(host["kv_indices"], device="cuda"), host["last"], True)
    err = (out.float() - ref).abs().max().item()
    assert err <= ATOL, err


def test_prefill_backend_bhsd_and_nhd(K):
    """run_prefill through the drop-in backend: BHSD in, BHSD out (the
    reference's shape handling, attention_backend.py:172-190)."""

    from pagelora_b200.attention_backend import B200AttentionBackend
    from oracle.paged_prefill import paged_prefill_bhsd

    reqs = [(24, 40), (24, 24)]
    host, dev = _case(reqs, 16, 4, 128, 16, seed=3)
    be = B200AttentionBackend(device=torch.device("cuda"), workspace_mb=8, num_qo_heads=16, num_kv_heads=4,
                              head_dim=128, page_size=16)
    be.plan_prefill(qo_indptr=dev["qo_indptr"], paged_kv_indptr=dev["kv_indptr"],
                    paged_kv_indices=dev["kv_indices"], paged_kv_last_page_len=dev["last"], causal=True)
    q_bhsd = dev["q"].view(2, 24, 16, 128).transpose(1, 2).contiguous()
    out = be.run_prefill(q_bhsd, dev["cache"])
    torch.cuda.synchronize()
    assert out.shape == (2, 16, 24, 128)
    want = paged_prefill_bhsd(host["q"].reshape(2, 24, 16, 128).transpose(0, 2, 1, 3), host["cache"],
                              host["qo_indptr"], host["kv_indptr"], host["kv_indices"], host["last"])
    assert np.abs(out.float().cpu().numpy() - want).max() <= ATOL
    out_nhd = be.run_prefill(dev["q"], dev["cache"])
    torch.cuda.synchronize()
    assert torch.equal(out_nhd.view(2, 24, 16, 128).transpose(1, 2), out)
    assert int(be.status.item()) == 0


def test_prefill_bad_page_reports_and_reads_zero(K):
    host, dev = _case([(16, 16)], 8, 8, 128, 16, seed=9, poison=False)
    bad = dev["kv_indices"].clone()
    bad[0] = 10_000
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    out = K.paged_prefill(dev["q"], dev["cache"], dev["qo_indptr"], dev["kv_indptr"], bad, dev["last"],
                          status=status)
    torch.cuda.synchronize()
    from pagelora_b200._capi import PL_ERR_PAGE_OUT_OF_RANGE

    assert int(status.item()) == PL_ERR_PAGE_OUT_OF_RANGE
    assert torch.isfinite(out.float()).all()


def test_prefill_finite_mask_known_answer(K):
    """The reference's prefill test (test/test_flashinfer_backend.py:157-177)
    at head_dim 64: causal query 0 sees key 0 only -> 1, query 1 sees two
    equal scores -> (1 + 9) / 2; both exact in bf16."""

    cache = torch.zeros(1, 2, 16, 1, 64, dtype=torch.bfloat16, device="cuda")
    cache[0, 0, :2, 0, 0] = 100.0
    cache[0, 1, 0, 0, 0], cache[0, 1, 1, 0, 0] = 1.0, 9.0
    q = torch.zeros(2, 1, 64, dtype=torch.bfloat16, device="cuda")
    q[:, 0, 0] = -1000.0
    i32 = dict(dtype=torch.int32, device="cuda")
    out = K.paged_prefill(q, cache, torch.tensor([0, 2], **i32), torch.tensor([0, 1], **i32),
                          torch.tensor([0], **i32), torch.tensor([2], **i32))
    torch.cuda.synchronize()
    assert out[:, 0, 0].float().tolist() == [1.0, 5.0]
