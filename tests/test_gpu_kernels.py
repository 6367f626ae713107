"""Parity of every CUDA kernel (called through the C ABI) with the CPU oracle.

Integer work (page tables) must be bit-exact; bf16 attention / LoRA outputs
must be within max |err| <= 2e-2 of the fp64 oracle (the tolerance stated
for this path), and LoRA outputs that mimic the reference's rounding points
must match the reference's own bf16 outputs to within 2 bf16 ulps.
"""

from __future__ import annotations

import json
import math

import numpy as np
import pytest
import torch

from oracle import lora as olora
from oracle import page_table as opt
from oracle.numerics import apply_rope, bf16, rmsnorm_fused, rmsnorm_hf, silu
from oracle.paged_decode import merge_states as o_merge
from oracle.paged_decode import paged_decode as o_decode

pytestmark = pytest.mark.gpu

ATOL = 2e-2


@pytest.fixture(scope="module")
def K(cuda_device):
    from pagelora_b200 import kernels

    return kernels


def _t(a, dtype=torch.bfloat16, dev="cuda"):
    return torch.as_tensor(np.asarray(a, dtype=np.float32)).to(device=dev, dtype=dtype)


def _i32(a, dev="cuda"):
    return torch.as_tensor(np.asarray(a, dtype=np.int32)).to(dev)


def _np(t):
    return t.detach().float().cpu().numpy()


def _ulps_close(actual, expected, ulps=2, magnitude=None):
    """Within ``ulps`` bf16 ulps of the larger of |expected| and |magnitude|
    (the summands' size: fp32 accumulation order may flip one rounding of a
    summand, which a cancelling sum cannot shrink)."""

    actual = np.asarray(actual, np.float32)
    expected = np.asarray(expected, np.float32)
    mag = np.abs(expected) if magnitude is None else np.maximum(np.abs(expected), np.abs(magnitude))
    tol = ulps * np.maximum(mag, 1e-3) * 2.0 ** -8 + 1e-6
    bad = np.abs(actual - expected) > tol
    assert not bad.any(), f"{bad.sum()} elements off; worst {float(np.max(np.abs(actual - expected) / tol)):.2f} tol"


# ------------------------------------------------------------ page tables
def _build_dev(K, rows, page_size):
    flat = [s for row in rows for s in row]
    row_indptr = np.cumsum([0] + [len(r) for r in rows])
    blk = _i32([s[0] for s in flat] or [0])
    st = _i32([s[1] for s in flat] or [0])
    ln = _i32([s[2] for s in flat] or [0])
    n_rows = len(rows)
    out_indptr = torch.full((n_rows + 1,), -7, dtype=torch.int32, device="cuda")
    out_indices = torch.full((max(1, len(flat)),), -7, dtype=torch.int32, device="cuda")
    out_last = torch.full((max(1, n_rows),), -7, dtype=torch.int32, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    err_row = torch.full((1,), -1, dtype=torch.int32, device="cuda")
    K.page_table_build(blk, st, ln, _i32(row_indptr), page_size, out_indptr, out_indices, out_last, status, err_row)
    torch.cuda.synchronize()
    return out_indptr.cpu().tolist(), out_indices.cpu().tolist(), out_last.cpu().tolist(), int(status.item())


def test_page_table_build_bit_exact_vs_reference_fixture(K, golden_dir):
    from pagelora_b200._capi import SPAN_ERROR_MESSAGES

    cases = json.loads((golden_dir / "page_tables.json").read_text())
    for case in cases:
        indptr, indices, last, status = _build_dev(K, case["rows"], case["page_size"])
        if "error" in case:
            assert status != 0 and SPAN_ERROR_MESSAGES[status] == case["error"], case
            assert indptr == [-7] * len(indptr)  # nothing written on error
        else:
            assert status == 0
            assert indptr == case["indptr"]
            n = case["indptr"][-1]
            assert indices[:n] == case["indices"]
            assert last[: len(case["rows"])] == case["last_page_len"]


def test_page_table_build_large_rows_vs_oracle(K):
    rng = np.random.default_rng(11)
    rows = []
    for _ in range(40):
        n = int(rng.integers(0, 300))
        pages = rng.permutation(5000)[:n]
        row = []
        for j, p in enumerate(pages):
            ln = 16 if j < n - 1 else int(rng.integers(1, 17))
            if rng.random() < 0.2 and ln > 1:
                c = int(rng.integers(1, ln))
                row += [[int(p), 0, c], [int(p), c, 0], [int(p), c, ln - c]]
            else:
                row.append([int(p), 0, ln])
        rows.append(row)
    got = _build_dev(K, rows, 16)
    want = opt.build_batch(rows, 16)
    assert got[3] == 0
    assert got[0] == want[0] and got[1][: want[0][-1]] == want[1] and got[2] == want[2]


def test_page_table_advance_vs_oracle(K):
    rows, cap, ps = 5, 8, 4
    row_pages = [[], [3], [5, 6], [7], [9, 10, 11]]
    last = [0, 4, 2, 1, 4]
    dev_pages = torch.zeros(rows, cap, dtype=torch.int32, device="cuda")
    for r, pg in enumerate(row_pages):
        if pg:
            dev_pages[r, : len(pg)] = torch.tensor(pg, dtype=torch.int32)
    n = _i32([len(p) for p in row_pages])
    dl = _i32(last)
    indptr = torch.zeros(rows + 1, dtype=torch.int32, device="cuda")
    indices = torch.zeros(rows * cap, dtype=torch.int32, device="cuda")
    sp, so, pos = (torch.zeros(rows, dtype=torch.int32, device="cuda") for _ in range(3))
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    for step in range(9):
        new = [100 + 10 * step + r for r in range(rows)]
        K.page_table_advance(n, dl, dev_pages, _i32(new), ps, indptr, indices, sp, so, pos, status)
        want = opt.advance(row_pages, last, new, ps)
        assert (sp.tolist(), so.tolist(), pos.tolist()) == tuple(list(x) for x in want)
        ip, idx, ll = opt.build_batch([[(p, 0, ps) for p in pg[:-1]] + [(pg[-1], 0, last[r])]
                                       for r, pg in enumerate(row_pages)], ps)
        assert indptr.tolist() == ip and indices.tolist()[: ip[-1]] == idx and dl.tolist() == ll
    assert int(status.item()) == 0


# ------------------------------------------------------- decode attention
def _decode_case(K, *, batch, hq, hkv, d, ps, lens, num_splits, seed, n_pages_pool=None, ws_mb=8, poison=False):
    rng = np.random.default_rng(seed)
    pages_per_row = [-(-L // ps) for L in lens]
    total = sum(pages_per_row)
    pool = n_pages_pool or total + 3
    cache = bf16(rng.normal(size=(pool, 2, ps, hkv, d)))
    perm = rng.permutation(pool)[:total]
    indptr = np.cumsum([0] + pages_per_row).tolist()
    indices = perm.tolist()
    last = [L - (n - 1) * ps if n else 0 for L, n in zip(lens, pages_per_row)]
    if poison:
        # NaN in every slot no row owns (the reference's pool is uninitialised)
        owned = np.zeros((pool, ps), dtype=bool)
        for r in range(batch):
            for j, pg in enumerate(indices[indptr[r]:indptr[r + 1]]):
                owned[pg, : (ps if j < pages_per_row[r] - 1 else last[r])] = True
        cache = np.where(owned[:, None, :, None, None], cache, np.float32(np.nan)).astype(np.float32)
    q = bf16(rng.normal(size=(batch, hq, d)) * 1.5)
    ws = torch.zeros(ws_mb << 20, dtype=torch.uint8, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    lse = torch.zeros(batch, hq, dtype=torch.float32, device="cuda")
    out = K.paged_decode(_t(q), _t(cache), _i32(indptr), _i32(indices or [0]), _i32(last),
                         num_splits=num_splits, workspace=ws, status=status, out_lse=lse)
    torch.cuda.synchronize()
    ref, ref_lse = o_decode(q, cache, indptr, indices, last)
    assert int(status.item()) == 0
    # counters are left at zero for the next call
    assert int(ws[: 4 * batch * hkv].view(torch.int32).abs().sum().item()) == 0
    return _np(out), _np(lse), ref, ref_lse


@pytest.mark.parametrize("d,ps", [(128, 16), (64, 16), (128, 32), (64, 32)])
@pytest.mark.parametrize("hq,hkv", [(32, 8), (8, 8), (16, 2), (16, 1)])
def test_paged_decode_vs_oracle(K, d, ps, hq, hkv):
    lens = [1, ps, ps + 1, 5 * ps - 3, 300]
    for splits in (1, 3, 16):
        out, lse, ref, ref_lse = _decode_case(K, batch=len(lens), hq=hq, hkv=hkv, d=d, ps=ps, lens=lens,
                                              num_splits=splits, seed=hq * 7 + d + ps + splits)
        assert np.max(np.abs(out - ref)) <= ATOL
        np.testing.assert_allclose(lse, ref_lse, rtol=1e-3, atol=1e-3)


@pytest.mark.parametrize("d,ps", [(128, 16), (64, 32)])
def test_paged_decode_ignores_nan_past_last_token(K, d, ps):
    """Slots past a row's last token (and pages no row owns) hold NaN: p = 0
    there must not turn into 0 * NaN."""

    lens = [1, ps - 3, 3 * ps + 5, 200]
    for splits in (1, 4):
        out, lse, ref, ref_lse = _decode_case(K, batch=len(lens), hq=16, hkv=4, d=d, ps=ps, lens=lens,
                                              num_splits=splits, seed=splits + d, poison=True)
        assert np.isfinite(out).all() and np.isfinite(lse).all()
        assert np.max(np.abs(out - ref)) <= ATOL
        np.testing.assert_allclose(lse, ref_lse, rtol=1e-3, atol=1e-3)


@pytest.mark.parametrize("batch,hq,hkv,lens_scale", [(1, 32, 8, 132), (3, 16, 2, 40), (2, 8, 8, 9)])
def test_paged_decode_cluster_merge_matches_workspace_merge(K, batch, hq, hkv, lens_scale):
    """The split merge through a thread-block cluster (DSMEM) and the one
    through the workspace give the same output and LSE, both within the
    oracle tolerance (splits 2..16, empty splits included)."""

    from pagelora_b200._capi import load_library

    lib = load_library()
    rng = np.random.default_rng(batch * 100 + hkv)
    lens = [int(lens_scale * 16 - rng.integers(0, 16)) for _ in range(batch)]
    lens[0] = max(lens[0], 1)
    for splits in (2, 5, 16):
        res = []
        for cluster in (1, 0):
            assert lib.pl_decode_set_cluster_merge(cluster) == 0
            try:
                res.append(_decode_case(K, batch=batch, hq=hq, hkv=hkv, d=128, ps=16, lens=lens,
                                        num_splits=splits, seed=splits))
            finally:
                lib.pl_decode_set_cluster_merge(1)
        (o1, l1, ref, ref_lse), (o0, l0, _, _) = res
        assert np.max(np.abs(o1 - ref)) <= ATOL and np.max(np.abs(o0 - ref)) <= ATOL
        assert np.max(np.abs(o1 - o0)) <= 2 ** -7 * max(1.0, float(np.max(np.abs(o0))))
        np.testing.assert_allclose(l1, l0, rtol=1e-5, atol=1e-5)
        np.testing.assert_allclose(l1, ref_lse, rtol=1e-3, atol=1e-3)


@pytest.mark.parametrize("d,hq,hkv,qk_norm", [(128, 32, 8, True), (64, 8, 2, False), (128, 16, 16, False)])
def test_paged_decode_qkv_matches_rope_then_decode(K, d, hq, hkv, qk_norm):
    """The fused launch (head norm + RoPE + append + decode) equals the two
    launches it replaces: same output, LSE, rotated q and appended K/V, for
    new tokens mid-page and at a fresh page, with multi-adapter LoRA, split
    counts 1 / 3 / 16; and a row whose slot is not its last page appends
    nothing (a split-KV shard without the tail)."""

    rng = np.random.default_rng(d + hq + hkv)
    ps, r, n_ad = 16, 16, 2
    lens = [1, 17, 40, 300]               # tokens including the new one
    b = len(lens)
    pages_per_row = [-(-n // ps) for n in lens]
    pool = sum(pages_per_row) + 6
    cache = _t(bf16(rng.normal(size=(pool, 2, ps, hkv, d))))
    perm = rng.permutation(pool)
    indptr = np.cumsum([0] + pages_per_row)
    indices = perm[: indptr[-1]]
    last = [n - (p - 1) * ps for n, p in zip(lens, pages_per_row)]
    slot_page = [int(indices[indptr[i + 1] - 1]) for i in range(b)]
    slot_off = [l - 1 for l in last]
    slot_page[2] = int(perm[-1])          # row 2's slot is elsewhere: no append, no injection
    n_heads = hq + 2 * hkv
    qkv = _t(bf16(rng.normal(size=(b, n_heads * d))))
    down = _t(rng.normal(size=(b, 3 * r)).astype(np.float32), torch.float32)
    lb = _t(bf16(rng.normal(size=(n_ad, n_heads * d, r)) * 0.05))
    tok_ad = _i32([0, 1, -1, 1])
    qn = _t(bf16(1 + rng.normal(size=d) * 0.1)) if qk_norm else None
    kn = _t(bf16(1 + rng.normal(size=d) * 0.1)) if qk_norm else None
    pos = _i32([n - 1 for n in lens])
    dev_ip, dev_idx, dev_last = _i32(indptr), _i32(indices), _i32(last)
    sp, so = _i32(slot_page), _i32(slot_off)
    ws = torch.zeros(8 << 20, dtype=torch.uint8, device="cuda")
    common = dict(lora_down=down, lora_b=lb, lora_scale=1.0, tok_adapter=tok_ad, q_norm_weight=qn,
                  k_norm_weight=kn, norm_eps=1e-6)
    for splits in (1, 3, 16):
        c_ref = cache.clone()
        q_ref = torch.empty(b, hq, d, dtype=torch.bfloat16, device="cuda")
        K.qkv_rope_append(qkv, num_qo_heads=hq, num_kv_heads=hkv, head_dim=d, positions=pos, rope_theta=1e6,
                          kv_cache=c_ref, page_id=sp, page_offset=so, q_out=q_ref, **common)
        lse_ref = torch.empty(b, hq, device="cuda")
        o_ref = K.paged_decode(q_ref, c_ref, dev_ip, dev_idx, dev_last, num_splits=splits, workspace=ws,
                               out_lse=lse_ref)
        c_f = cache.clone()
        q_f = torch.zeros(b, hq, d, dtype=torch.bfloat16, device="cuda")
        lse_f = torch.empty(b, hq, device="cuda")
        status = torch.zeros(1, dtype=torch.int32, device="cuda")
        o_f = K.paged_decode_qkv(qkv, c_f, dev_ip, dev_idx, dev_last, num_qo_heads=hq, num_kv_heads=hkv,
                                 positions=pos, rope_theta=1e6, slot_page=sp, slot_offset=so, num_splits=splits,
                                 workspace=ws, out_lse=lse_f, q_out=q_f, status=status, **common)
        # the same launch reading the step's RoPE table instead of evaluating the angles
        c_t = cache.clone()
        q_t = torch.zeros_like(q_f)
        lse_t = torch.empty_like(lse_f)
        o_t = K.paged_decode_qkv(qkv, c_t, dev_ip, dev_idx, dev_last, num_qo_heads=hq, num_kv_heads=hkv,
                                 positions=pos, rope_theta=1e6, slot_page=sp, slot_offset=so, num_splits=splits,
                                 workspace=ws, out_lse=lse_t, q_out=q_t, status=status,
                                 rope_cos_sin=K.rope_cos_sin(pos, d, 1e6), **common)
        torch.cuda.synchronize()
        assert int(status.item()) == 0
        assert torch.equal(q_t, q_f) and torch.equal(o_t, o_f) and torch.equal(c_t, c_f)
        assert torch.equal(lse_t, lse_f)
        assert torch.equal(q_f, q_ref)
        # appended K/V: identical where the row owns its slot; row 2's slot page untouched by the fused call
        for i in (0, 1, 3):
            assert torch.equal(c_f[slot_page[i], :, slot_off[i]], c_ref[slot_page[i], :, slot_off[i]])
        assert torch.equal(c_f[slot_page[2]], cache[slot_page[2]])
        keep = [0, 1, 3]
        assert np.max(np.abs(_np(o_f)[keep] - _np(o_ref)[keep])) <= 2 ** -7 * 4
        np.testing.assert_allclose(_np(lse_f)[keep], _np(lse_ref)[keep], rtol=1e-5, atol=1e-5)
        # row 2: attention over its pages as they are (no new token)
        np.testing.assert_allclose(_np(o_f)[2], _np(K.paged_decode(q_f[2:3], cache, _i32([0, pages_per_row[2]]),
                                                                   _i32(indices[indptr[2]:indptr[3]]),
                                                                   _i32([last[2]]), num_splits=1,
                                                                   workspace=ws))[0], atol=2 ** -7 * 4)


@pytest.mark.parametrize("cluster", [True, False])
@pytest.mark.parametrize("hq,hkv", [(32, 8), (16, 16)])
def test_paged_decode_merge_prior_equals_separate_merge(K, hq, hkv, cluster):
    """pl_paged_decode_merge_prior: merging a prior state into the bf16 output
    gives the same bits as writing this launch's fp32 state and merging the
    two with pl_merge_states_strided, for one split, the cluster merge and
    the workspace merge; rows with no pages take the prior state alone."""

    from pagelora_b200._capi import load_library

    lib = load_library()
    g = torch.Generator(device="cuda").manual_seed(hq + hkv)
    d, ps = 128, 16
    lens = [0, 5, 40, 300]
    b = len(lens)
    pages = [-(-n // ps) for n in lens]
    pool = sum(pages) + 3
    cache = torch.randn(pool, 2, ps, hkv, d, generator=g, device="cuda").bfloat16()
    perm = torch.randperm(pool, generator=g, device="cuda")[: sum(pages)].to(torch.int32)
    indptr = _i32(np.cumsum([0] + pages))
    last = _i32([n - (p - 1) * ps if p else 0 for n, p in zip(lens, pages)])
    q = torch.randn(b, hq, d, generator=g, device="cuda").bfloat16()
    prior_o = torch.randn(b, hq, d, generator=g, device="cuda")
    prior_lse = torch.randn(b, hq, generator=g, device="cuda") * 3
    ws = torch.zeros(8 << 20, dtype=torch.uint8, device="cuda")
    assert lib.pl_decode_set_cluster_merge(1 if cluster else 0) == 0
    try:
        for splits in (1, 3, 8):
            o32 = torch.empty(b, hq, d, device="cuda")
            lse = torch.empty(b, hq, device="cuda")
            K.paged_decode(q, cache, indptr, perm, last, num_splits=splits, workspace=ws, out=o32, out_lse=lse)
            ref = torch.empty(b * hq, d, dtype=torch.bfloat16, device="cuda")
            K.merge_states_strided(torch.stack([prior_o.view(b * hq, d), o32.view(b * hq, d)], 1),
                                   torch.stack([prior_lse.view(-1), lse.view(-1)], 1), ref)
            got = K.paged_decode(q, cache, indptr, perm, last, num_splits=splits, workspace=ws,
                                 out=torch.empty(b, hq, d, dtype=torch.bfloat16, device="cuda"),
                                 prior=(prior_o, prior_lse))
            torch.cuda.synchronize()
            assert torch.equal(got.view(b * hq, d), ref), splits
            assert torch.equal(got[0].float(), prior_o[0].bfloat16().float())  # no pages: the prior alone
    finally:
        assert lib.pl_decode_set_cluster_merge(1) == 0


@pytest.mark.parametrize("rows,hq,hkv,fold", [(7, 32, 8, 4), (5, 16, 16, 16), (6, 8, 2, 3)])
def test_paged_decode_shared_folded_rows(K, rows, hq, hkv, fold):
    """Rows folded onto shared page-table rows (fold x group tile rows) equal
    plain decode with the page lists repeated per row, for one split, the
    cluster merge and the workspace merge; padding rows of the last fold are
    not written."""

    from pagelora_b200._capi import load_library

    lib = load_library()
    rng = np.random.default_rng(rows * 10 + fold)
    ps, d = 16, 128
    vrows = -(-rows // fold)
    lens = rng.integers(1, 400, size=vrows).tolist()
    pages = [-(-n // ps) for n in lens]
    pool = sum(pages) + 4
    cache = _t(bf16(rng.normal(size=(pool, 2, ps, hkv, d))))
    perm = rng.permutation(pool).tolist()
    lists, off = [], 0
    for n in pages:
        lists.append(perm[off:off + n])
        off += n
    last = [n - (p - 1) * ps for n, p in zip(lens, pages)]
    q = _t(bf16(rng.normal(size=(rows, hq, d)) * 1.5))
    v_indptr = _i32(np.cumsum([0] + pages))
    v_idx = _i32([x for l in lists for x in l])
    v_last = _i32(last)
    row_lists = [lists[b // fold] for b in range(rows)]
    r_indptr = _i32(np.cumsum([0] + [len(l) for l in row_lists]))
    r_idx = _i32([x for l in row_lists for x in l])
    r_last = _i32([last[b // fold] for b in range(rows)])
    ws = torch.zeros(8 << 20, dtype=torch.uint8, device="cuda")      # one workspace per shape
    ws_ref = torch.zeros(8 << 20, dtype=torch.uint8, device="cuda")
    for splits in (1, 3, 16):
        for cluster in (1, 0):
            lib.pl_decode_set_cluster_merge(cluster)
            try:
                out = torch.full((rows, hq, d), float("nan"), device="cuda")
                lse = torch.full((rows, hq), float("nan"), device="cuda")
                K.paged_decode_shared(q, cache, v_indptr, v_idx, v_last, fold=fold, num_splits=splits, workspace=ws,
                                      out=out, out_lse=lse)
                ref_lse = torch.empty(rows, hq, device="cuda")
                ref = K.paged_decode(q, cache, r_indptr, r_idx, r_last, num_splits=splits, workspace=ws_ref,
                                     out=torch.empty(rows, hq, d, device="cuda"), out_lse=ref_lse)
                torch.cuda.synchronize()
            finally:
                lib.pl_decode_set_cluster_merge(1)
            assert torch.isfinite(out).all() and torch.isfinite(lse).all()
            assert float((out - ref).abs().max()) <= 1e-4
            assert float((lse - ref_lse).abs().max()) <= 1e-4


def test_paged_decode_empty_row_and_long_context(K):
    out, lse, ref, ref_lse = _decode_case(K, batch=3, hq=32, hkv=8, d=128, ps=16, lens=[0, 2112, 7],
                                          num_splits=37, seed=5)
    assert np.all(out[0] == 0) and np.all(np.isneginf(lse[0]))
    assert np.max(np.abs(out - ref)) <= ATOL
    np.testing.assert_allclose(lse[1:], ref_lse[1:], rtol=1e-3, atol=1e-3)


@pytest.mark.parametrize("hq,hkv,splits", [(32, 8, 2), (32, 32, 1)])
def test_paged_decode_many_ring_laps_is_deterministic(K, hq, hkv, splits):
    """Splits of hundreds of pages cycle the stage ring many times (the
    config-3 / config-5 regime).  Every launch must finish with status 0, give
    bit-identical outputs, and agree with a torch fp32 reference."""

    rows, ctx, d, ps = 4, 8192 - 5, 128, 16
    g = torch.Generator(device="cuda").manual_seed(7)
    pages = -(-ctx // ps)
    pool = rows * pages + 8
    cache = torch.randn(pool, 2, ps, hkv, d, device="cuda", dtype=torch.bfloat16, generator=g)
    perm = torch.randperm(pool, device="cuda", generator=g)[: rows * pages].to(torch.int32)
    indptr = _i32(np.arange(rows + 1) * pages)
    last = _i32([ctx - (pages - 1) * ps] * rows)
    q = torch.randn(rows, hq, d, device="cuda", dtype=torch.bfloat16, generator=g)
    ws = torch.zeros(rows * hq * splits * (d + 1) * 4 + (1 << 20), dtype=torch.uint8, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    outs = []
    for _ in range(12):
        outs.append(K.paged_decode(q, cache, indptr, perm, last, num_splits=splits, workspace=ws, status=status))
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    for o in outs[1:]:
        assert torch.equal(o, outs[0])
    # torch fp32 reference over the gathered pages
    kv = cache[perm.long()].view(rows, pages, 2, ps, hkv, d).float()
    k = kv[:, :, 0].reshape(rows, pages * ps, hkv, d)[:, :ctx]
    v = kv[:, :, 1].reshape(rows, pages * ps, hkv, d)[:, :ctx]
    grp = hq // hkv
    qf = q.float().view(rows, hkv, grp, d)
    s = torch.einsum("bhgd,bthd->bhgt", qf, k) / math.sqrt(d)
    ref = torch.einsum("bhgt,bthd->bhgd", torch.softmax(s, dim=-1), v).reshape(rows, hq, d)
    assert float((outs[0].float() - ref).abs().max()) <= ATOL


def test_paged_decode_reports_out_of_range_page(K):
    cache = torch.zeros(4, 2, 16, 2, 64, dtype=torch.bfloat16, device="cuda")
    q = torch.ones(1, 4, 64, dtype=torch.bfloat16, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    ws = torch.zeros(1 << 16, dtype=torch.uint8, device="cuda")
    K.paged_decode(q, cache, _i32([0, 2]), _i32([1, 99]), _i32([16]), num_splits=1, workspace=ws, status=status)
    torch.cuda.synchronize()
    from pagelora_b200._capi import PL_ERR_PAGE_OUT_OF_RANGE

    assert int(status.item()) == PL_ERR_PAGE_OUT_OF_RANGE


@pytest.mark.parametrize("world", [2, 3])
def test_split_kv_shards_merge_to_full_decode(K, world):
    """Split-KV across shards on one GPU: each shard's fp32 partial (O, LSE)
    over its page range (pl_paged_decode_f32), stacked like an all-gather
    [shard][rows][D] and merged with pl_merge_states_strided, equals the
    full decode."""

    from pagelora_b200.split_kv import shard_row

    rng = np.random.default_rng(60 + world)
    ps, hq, hkv, d = 16, 32, 8, 128
    lengths = [1, 16, 17, 300, 2112, 45]
    pages_per_row = [-(-n // ps) for n in lengths]
    pool = sum(pages_per_row) + 5
    cache = bf16(rng.normal(size=(pool, 2, ps, hkv, d)))
    perm = rng.permutation(pool)
    indptr = np.cumsum([0] + pages_per_row)
    indices = perm[: indptr[-1]]
    last = [n - (p - 1) * ps for n, p in zip(lengths, pages_per_row)]
    q = bf16(rng.normal(size=(len(lengths), hq, d)) * 1.5)
    qt, ct = _t(q), _t(cache)
    rows = len(lengths)
    gathered = torch.zeros(world, rows * hq * (d + 1), device="cuda")
    ws = torch.zeros(8 << 20, dtype=torch.uint8, device="cuda")
    for r in range(world):
        sh_indptr, sh_indices, sh_last = [0], [], []
        for b, n in enumerate(lengths):
            p0, p1, kept_last = shard_row(n, ps, r, world)
            sh_indices += indices[indptr[b] + p0: indptr[b] + p1].tolist()
            sh_indptr.append(len(sh_indices))
            sh_last.append(kept_last)
        nd = rows * hq * d
        o_part = gathered[r, :nd].view(rows, hq, d)
        lse_part = gathered[r, nd:].view(rows, hq)
        K.paged_decode(qt, ct, _i32(sh_indptr), _i32(sh_indices or [0]), _i32(sh_last), num_splits=3,
                       workspace=ws, out=o_part, out_lse=lse_part)
    nd = rows * hq * d
    v = gathered[:, :nd].view(world, rows * hq, d).permute(1, 0, 2)
    lse = gathered[:, nd:].permute(1, 0)
    out = torch.empty(rows * hq, d, dtype=torch.bfloat16, device="cuda")
    out_lse = torch.empty(rows * hq, dtype=torch.float32, device="cuda")
    K.merge_states_strided(v, lse, out, out_lse)
    torch.cuda.synchronize()
    ref, ref_lse = o_decode(q, cache, indptr.tolist(), indices.tolist(), last)
    assert np.max(np.abs(_np(out).reshape(rows, hq, d) - ref)) <= ATOL
    np.testing.assert_allclose(_np(out_lse).reshape(rows, hq), ref_lse, rtol=1e-3, atol=1e-3)


def test_merge_states_vs_oracle(K):
    rng = np.random.default_rng(2)
    v = rng.normal(size=(37, 6, 128)).astype(np.float32)
    lse = rng.normal(size=(37, 6)).astype(np.float32) * 3
    lse[3, :] = -np.inf
    lse[5, 2] = -np.inf
    out_lse = torch.zeros(37, dtype=torch.float32, device="cuda")
    out = K.merge_states(_t(v, torch.float32), _t(lse, torch.float32), out_lse=out_lse)
    ref, ref_lse = o_merge(np.moveaxis(v, 1, 0), lse.T)
    assert np.max(np.abs(_np(out) - ref)) <= ATOL
    np.testing.assert_allclose(_np(out_lse)[np.isfinite(ref_lse)], ref_lse[np.isfinite(ref_lse)], rtol=1e-5)
    assert np.all(np.isneginf(_np(out_lse)[3]))


# ------------------------------------------------------------ LoRA kernels
def test_lora_shrink_seg_vs_oracle(K):
    rng = np.random.default_rng(4)
    x = bf16(rng.normal(size=(13, 512)))
    a = bf16(rng.normal(size=(3, 16, 512)) * 0.02)
    seg_indptr, seg_adapter = [0, 2, 2, 9, 13], [1, 0, 2, -1]
    out = K.lora_shrink_seg(_t(x), _t(a), _i32(seg_indptr), _i32(seg_adapter))
    torch.cuda.synchronize()
    ref = olora.shrink_seg(x, a, seg_indptr, seg_adapter)
    np.testing.assert_allclose(_np(out), ref, rtol=1e-4, atol=1e-4)


def test_linear_lora_matches_reference_lora_linear(K, golden_dir):
    """The fused kernel reproduces multilora/linear.py LoRALinear.forward (bf16)."""

    z = np.load(golden_dir / "lora_cases.npz")
    for case in range(3):
        pre = f"lora_linear_bf16_{case}_"
        x, w, a, b = z[pre + "x"], z[pre + "w"], z[pre + "a"], z[pre + "b"]
        sc = float(z[pre + "scale"][0])
        bias = _t(z[pre + "bias"]) if z[pre + "bias"].size else None
        t = x.shape[0]
        down = K.lora_shrink_seg(_t(x), _t(a)[None], _i32([0, t]), _i32([0]))
        y = K.linear_lora_fused(_t(x), _t(w), bias=bias, lora_down=down, lora_b=_t(b)[None], lora_scale=sc)
        torch.cuda.synchronize()
        base = olora.linear(x, w, z[pre + "bias"] if z[pre + "bias"].size else None, bf16=True)
        _ulps_close(_np(y), z[pre + "y"], magnitude=base)


def test_packed_qkv_matches_reference(K, golden_dir):
    """Packed q/k/v + packed LoRA delta (packed_ops.py) via the shrink rows
    of the fused kernel and the expand of qkv_rope_append's LoRA step."""

    z = np.load(golden_dir / "lora_cases.npz")
    for case in range(2):
        pre = f"packed_{case}_"
        sc = float(z[pre + "scale"][0])
        x = z[pre + "x"]
        w = np.concatenate([z[f"{pre}{m}_w"] for m in "qkv"])
        a = np.concatenate([z[f"{pre}{m}_a"] for m in "qkv"])
        b = np.concatenate([bf16(z[f"{pre}{m}_b"] * sc) for m in "qkv"])
        dq, dk = z[pre + "q"].shape[-1], z[pre + "k"].shape[-1]
        down = torch.zeros(x.shape[0], a.shape[0], dtype=torch.float32, device="cuda")
        base = K.linear_lora_fused(_t(x), _t(w), shrink_a=_t(a), shrink_out=down)
        # expand exactly as the decode path does: slices q | k | v with rank r
        y = K.linear_lora_fused(_t(x), _t(w), lora_down=down, lora_b=_t(b)[None], slice_ends=(dq, dq + dk))
        torch.cuda.synchronize()
        ref = np.concatenate([z[pre + "q"], z[pre + "k"], z[pre + "v"]], -1)
        _ulps_close(_np(y), ref, magnitude=olora.linear(x, w, bf16=True))
        _ulps_close(_np(base), olora.linear(x, w, bf16=True))


# GEMV variants: TMA ring (mode 1), register-direct loads with 4 or 8 warps
# (mode 2, with and without the L2 prefetch of the first tiles), by size (mode 0).
GEMV_TUNINGS = {
    "tma": ((1, 3, 2048, 8, 1), 0),
    "tma_4w2c": ((1, 4, 1024, 4, 2), 0),
    "ldg_4w4c": ((2, 2, 256, 4, 4), 0),
    "ldg_8w2c_pf": ((2, 2, 256, 8, 2), 64 << 20),
    "auto_pf": ((0, 2, 256, 4, 1), 32 << 20),
}


@pytest.fixture(params=sorted(GEMV_TUNINGS))
def gemv_tuning(request, K):
    from pagelora_b200._capi import load_library

    lib = load_library()
    tune, pf = GEMV_TUNINGS[request.param]
    if tune[0] == 0:
        assert lib.pl_linear_set_tuning(2, 2, 256, 4, 4) == 0
    assert lib.pl_linear_set_tuning(*tune) == 0
    assert lib.pl_linear_set_l2_prefetch(pf) == 0
    yield request.param
    assert lib.pl_linear_set_tuning(-1, 0, 0, 0, 0) == 0


@pytest.mark.parametrize("t", [1, 2, 5, 8])
def test_linear_lora_fused_prologues_and_epilogues_vs_oracle(K, t, gemv_tuning):
    rng = np.random.default_rng(100 + t)
    k_in, n, r, n_ad = 1024, 700, 16, 3
    x = bf16(rng.normal(size=(t, k_in)))
    res = bf16(rng.normal(size=(t, n)))
    w = bf16(rng.normal(size=(n, k_in)) * 0.02)
    bias = bf16(rng.normal(size=n) * 0.1)
    nw = bf16(1 + rng.normal(size=k_in) * 0.1)
    down = rng.normal(size=(t, 2 * r)).astype(np.float32)
    bmat = bf16(rng.normal(size=(n_ad, n, r)) * 0.05)
    tok_ad = rng.integers(-1, n_ad, size=t)
    a_rows = bf16(rng.normal(size=(24, k_in)) * 0.02)
    shrink = torch.zeros(t, 24, dtype=torch.float32, device="cuda")
    y = K.linear_lora_fused(_t(x), _t(w), bias=_t(bias), prologue=1, norm_weight=_t(nw), norm_eps=1e-6,
                            lora_down=_t(down, torch.float32), lora_b=_t(bmat), slice_ends=(300,),
                            tok_adapter=_i32(tok_ad), residual=_t(res), shrink_a=_t(a_rows), shrink_out=shrink)
    torch.cuda.synchronize()
    xn = rmsnorm_fused(x, nw, 1e-6)
    base = bf16(xn.astype(np.float64) @ w.T.astype(np.float64) + bias)
    want = np.zeros((t, n), np.float32)
    for i in range(t):
        yi = base[i]
        if tok_ad[i] >= 0:
            d = np.concatenate([bmat[tok_ad[i], :300] @ bf16(down[i, :r]), bmat[tok_ad[i], 300:] @ bf16(down[i, r:])])
            yi = bf16(yi + bf16(d))
        want[i] = bf16(res[i] + yi)
    _ulps_close(_np(y), want, ulps=3)
    np.testing.assert_allclose(_np(shrink), xn.astype(np.float64) @ a_rows.T.astype(np.float64), rtol=1e-3, atol=1e-3)
    # SiLU-and-mul prologue
    gu = bf16(rng.normal(size=(t, 2 * k_in)))
    y2 = K.linear_lora_fused(_t(gu), _t(w))
    y3 = K.linear_lora_fused(_t(gu), _t(w), prologue=2)
    torch.cuda.synchronize()
    act = bf16(silu(gu[:, :k_in]) * gu[:, k_in:])
    _ulps_close(_np(y3), bf16(act.astype(np.float64) @ w.T.astype(np.float64)), ulps=3)
    _ulps_close(_np(y2), bf16(gu[:, :k_in].astype(np.float64) @ w.T.astype(np.float64)), ulps=3)


@pytest.mark.parametrize("t,r", [(1, 16), (5, 16), (8, 32), (3, 64)])
def test_linear_lora_fused_down_from_x_vs_oracle(K, t, r):
    """PL_FLAG_DOWN_FROM_X: the LoRA down x . A^T computed in the GEMV's
    prologue (per-token adapters, one with no LoRA) gives the reference's
    LoRALinear output (multilora/linear.py:226-231 rounding points)."""

    rng = np.random.default_rng(7 * t + r)
    k_in, n, n_ad = 4096, 1000, 3
    x = bf16(rng.normal(size=(t, k_in)))
    res = bf16(rng.normal(size=(t, n)))
    w = bf16(rng.normal(size=(n, k_in)) * 0.02)
    a_st = bf16(rng.normal(size=(n_ad, r, k_in)) * 0.02)
    bmat = bf16(rng.normal(size=(n_ad, n, r)) * 0.05)
    tok_ad = rng.integers(-1, n_ad, size=t)
    tok_ad[0] = 1
    y = K.linear_lora_fused(_t(x), _t(w), lora_a=_t(a_st), lora_b=_t(bmat), lora_scale=0.5,
                            tok_adapter=_i32(tok_ad), residual=_t(res), weights_static=True)
    torch.cuda.synchronize()
    base = bf16(x.astype(np.float64) @ w.T.astype(np.float64))
    want = np.zeros((t, n), np.float32)
    for i in range(t):
        yi = base[i]
        if tok_ad[i] >= 0:
            down = bf16(x[i].astype(np.float64) @ a_st[tok_ad[i]].T.astype(np.float64))
            yi = bf16(yi + bf16(bf16(bmat[tok_ad[i]] @ down) * 0.5))
        want[i] = bf16(res[i] + yi)
    # the fp32 down sum order may move bf16(down) by one ulp
    _ulps_close(_np(y), want, ulps=3, magnitude=np.abs(base))


def test_linear_lora_fused_large_shapes(K, gemv_tuning):
    """Decode shapes of Qwen3-8B (qkv, o, gate_up, down) at one token."""

    g = torch.Generator(device="cuda").manual_seed(0)
    for n, k in ((6144, 4096), (4096, 4096), (24576, 4096), (4096, 12288)):
        w = (torch.randn(n, k, generator=g, device="cuda") * 0.02).bfloat16()
        x = torch.randn(1, k, generator=g, device="cuda").bfloat16()
        y = K.linear_lora_fused(x, w, weights_static=True)
        ref = (x.double() @ w.double().T)
        # one bf16 rounding of the fp32 accumulation: within 1 ulp of |ref| (+ fp32 sum noise)
        tol = torch.abs(ref) * 2.0 ** -8 + 1e-3
        assert bool(torch.all(torch.abs(y.double() - ref) <= tol))


@pytest.mark.parametrize("t", [1, 3, 8])
def test_linear_lora_chain_equals_single_launches(K, t):
    """pl_linear_lora_chain: five dependent projections (LoRA down from x +
    residual in place, RMSNorm, SiLU-and-mul + residual, RMSNorm + bias +
    sliced LoRA + shrink rows, plain) in one persistent launch give the same
    bits as the same projections launched one by one (each of which is held
    to the oracle above), and the grid barrier is back at zero."""

    g = torch.Generator(device="cuda").manual_seed(40 + t)

    def rnd(*shape, s=1.0):
        return (torch.randn(*shape, generator=g, device="cuda") * s).bfloat16()

    H, Q, I, N4, r = 768, 512, 1024, 640, 16
    attn, x0 = rnd(t, Q), rnd(t, H)
    w_o, a_o, b_o = rnd(H, Q, s=0.03), rnd(2, r, Q, s=0.03), rnd(2, H, r, s=0.05)
    w_gu, n1 = rnd(2 * I, H, s=0.03), (1 + 0.1 * torch.randn(H, generator=g, device="cuda")).bfloat16()
    w_dn = rnd(H, I, s=0.03)
    w_4, n2, bias4 = rnd(N4, H, s=0.03), (1 + 0.1 * torch.randn(H, generator=g, device="cuda")).bfloat16(), rnd(N4)
    a_4 = rnd(48, H, s=0.03)
    b_4, down4 = rnd(3, N4, r, s=0.05), torch.randn(t, 3 * r, generator=g, device="cuda")
    w_5 = rnd(300, N4, s=0.03)
    tok_ad = torch.tensor([(i % 3) - 1 for i in range(t)], dtype=torch.int32, device="cuda")
    tok_ad[0] = 1

    def phases(x, gu, y4, sh4, y5):
        return [
            (attn, w_o, dict(lora_a=a_o, lora_b=b_o, lora_scale=0.5, tok_adapter=tok_ad.clamp(max=1),
                             residual=x, out=x, weights_static=True)),
            (x, w_gu, dict(prologue=1, norm_weight=n1, norm_eps=1e-6, out=gu, weights_static=True)),
            (gu, w_dn, dict(prologue=2, residual=x, out=x, weights_static=True)),
            (x, w_4, dict(prologue=1, norm_weight=n2, norm_eps=1e-6, bias=bias4, lora_down=down4, lora_b=b_4,
                          slice_ends=(200, 420), tok_adapter=tok_ad, out=y4, shrink_a=a_4, shrink_out=sh4,
                          weights_static=True)),
            (y4, w_5, dict(out=y5, weights_static=True)),
        ]

    def bufs():
        return (x0.clone(), torch.empty(t, 2 * I, dtype=torch.bfloat16, device="cuda"),
                torch.empty(t, N4, dtype=torch.bfloat16, device="cuda"),
                torch.empty(t, 48, dtype=torch.float32, device="cuda"),
                torch.empty(t, 300, dtype=torch.bfloat16, device="cuda"))

    ref = bufs()
    for x_, w_, kw in phases(*ref):
        K.linear_lora_fused(x_, w_, **kw)
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    barrier = torch.zeros(1, dtype=torch.int32, device="cuda")
    for _ in range(2):  # the second call reuses the barrier the first one reset
        got = bufs()
        K.linear_lora_chain(phases(*got), grid_barrier=barrier, status=status)
        torch.cuda.synchronize()
        for a, b in zip(got, ref):
            assert torch.equal(a, b)
        assert int(barrier.item()) == 0 and int(status.item()) == 0
    # one phase: no barrier needed
    one = bufs()
    K.linear_lora_chain(phases(*one)[1:2], grid_barrier=None, status=status)
    y_gu = K.linear_lora_fused(x0, w_gu, prologue=1, norm_weight=n1, norm_eps=1e-6)
    torch.cuda.synchronize()
    assert torch.equal(one[1], y_gu)


@pytest.mark.parametrize("t,units", [(1, 1), (1, 5), (4, 2)])
def test_linear_lora_fused_l2_handover_same_bits(K, t, units):
    """pl_linear_lora_phase: the L2 hand-over to the next projection (with
    shrink rows, and past the end of a CTA's share when `units` is large)
    leaves this launch's and the next launch's outputs bit-identical."""

    g = torch.Generator(device="cuda").manual_seed(9 + t)
    x = torch.randn(t, 4096, generator=g, device="cuda").bfloat16()
    w1 = (torch.randn(4096, 4096, generator=g, device="cuda") * 0.02).bfloat16()
    w2 = (torch.randn(2000, 4096, generator=g, device="cuda") * 0.02).bfloat16()
    a2 = (torch.randn(48, 4096, generator=g, device="cuda") * 0.02).bfloat16()
    nw = (1 + 0.1 * torch.randn(4096, generator=g, device="cuda")).bfloat16()
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    nxt_kw = dict(prologue=1, norm_weight=nw, shrink_a=a2, weights_static=True)
    y_ref = K.linear_lora_fused(x, w1, residual=x, weights_static=True)
    z_ref = K.linear_lora_fused(y_ref, w2, **nxt_kw)
    y = K.linear_lora_fused(x, w1, residual=x, weights_static=True, status=status, prefetch_next=(y_ref, w2, nxt_kw),
                            prefetch_units=units)
    z = K.linear_lora_fused(y, w2, status=status, **nxt_kw)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    assert torch.equal(y, y_ref) and torch.equal(z, z_ref)


@pytest.mark.parametrize("t,k,r", [(1, 4096, 48), (16, 4096, 16), (64, 4096, 48), (5, 8192, 30), (3, 600, 24)])
def test_lora_shrink_rows_vs_rmsnorm_and_oracle(K, t, k, r):
    """pl_lora_shrink_rows: the normalised rows are bit-identical to
    pl_rmsnorm's, and the per-row-adapter shrink (adapters -1 and out of
    range give zeros; rank not a multiple of the 4-row block) matches the
    fp64 product of those rows within fp32 rounding, with and without the
    norm."""

    g = torch.Generator(device="cuda").manual_seed(t * 7 + r)
    x = torch.randn(t, k, generator=g, device="cuda").bfloat16()
    nw = (1 + 0.1 * torch.randn(k, generator=g, device="cuda")).bfloat16()
    a = (torch.randn(3, r, k, generator=g, device="cuda") * 0.03).bfloat16()
    ad = torch.tensor([(i % 5) - 1 for i in range(t)], dtype=torch.int32, device="cuda")  # -1, 0, 1, 2, 3
    xn = torch.zeros_like(x)
    down = K.lora_shrink_rows(x, a, tok_adapter=ad, norm_weight=nw, norm_eps=1e-6, xn_out=xn)
    down_plain = K.lora_shrink_rows(x, a, tok_adapter=ad)
    xn_ref = K.rmsnorm(x, nw, 1e-6)
    torch.cuda.synchronize()
    assert torch.equal(xn, xn_ref)
    adl = ad.cpu().tolist()
    for src, got in ((xn_ref, down), (x, down_plain)):
        want = np.zeros((t, r))
        for i in range(t):
            if 0 <= adl[i] < 3:
                want[i] = src[i].double().cpu().numpy() @ a[adl[i]].double().cpu().numpy().T
        np.testing.assert_allclose(_np(got), want, rtol=1e-4, atol=1e-4)


@pytest.mark.parametrize("t", [9, 16, 64, 128])
def test_linear_lora_gemm_silu_pairs_vs_oracle(K, t):
    """PL_FLAG_SILU_PAIRS: the GEMM over the interleaved gate/up stack writes
    bf16(silu(bf16(g)) * bf16(u)) (the reference's bf16 gate_up output, then
    SiLU-and-mul), checked against the fp64 products; and it agrees with the
    plain GEMM followed by pl_silu_mul."""

    rng = np.random.default_rng(31 + t)
    k_in, inter = 1024, 1536
    x = bf16(rng.normal(size=(t, k_in)))
    w = bf16(rng.normal(size=(2 * inter, k_in)) * 0.03)
    wt = _t(w)
    act = K.linear_lora_gemm(_t(x), K.interleave_gate_up(wt), silu_pairs=True)
    plain = K.silu_mul(K.linear_lora_gemm(_t(x), wt))
    torch.cuda.synchronize()
    gu = x.astype(np.float64) @ w.T.astype(np.float64)
    g, u = bf16(gu[:, :inter]), bf16(gu[:, inter:])
    want = bf16(silu(g) * u)
    # a 1-ulp difference in bf16(g) or bf16(u) moves the product by about one ulp of it
    _ulps_close(_np(act), want, ulps=3, magnitude=np.abs(g * u))
    _ulps_close(_np(act), _np(plain), ulps=3, magnitude=np.abs(g * u))


def _gemm_oracle(x, w, bias, down, bmat, tok_ad, split_at, res, scale=1.0):
    """fp64 restatement of the multi-token LoRA linear epilogue (per-token adapter)."""

    t, n = x.shape[0], w.shape[0]
    r = bmat.shape[-1]
    base = bf16(x.astype(np.float64) @ w.T.astype(np.float64) + (0 if bias is None else bias))
    want = np.zeros((t, n), np.float32)
    mag = np.abs(base).astype(np.float32)  # size of the summands (cancellation bound)
    for i in range(t):
        yi = base[i]
        if tok_ad[i] >= 0:
            d = np.concatenate([bmat[tok_ad[i], :split_at] @ bf16(down[i, :r]),
                                bmat[tok_ad[i], split_at:] @ bf16(down[i, r:2 * r])])
            yi = bf16(yi + bf16(bf16(d) * scale))
        mag[i] = np.maximum(mag[i], np.abs(yi))
        if res is not None:
            mag[i] = np.maximum(mag[i], np.abs(res[i]))
        want[i] = bf16(res[i] + yi) if res is not None else yi
    return mag, want


@pytest.mark.parametrize("k_in", [600, 640])
@pytest.mark.parametrize("t", [1, 9, 16, 33, 64, 100, 128])
def test_linear_lora_gemm_vs_oracle(K, t, k_in):
    """tcgen05 multi-token linear: multi-adapter LoRA epilogue, partial row
    tile, K tails (600: 2-D tiles with a partial 64-column chunk; 640: 3-D
    tiles, last K block half empty), grids of 1 CTA (whole tiles), one per
    SM and 7 CTAs (tiles shared between CTAs, partials merged in order)."""

    rng = np.random.default_rng(300 + t + k_in)
    n, r, n_ad = 700, 16, 3
    x = bf16(rng.normal(size=(t, k_in)))
    w = bf16(rng.normal(size=(n, k_in)) * 0.05)
    bias = bf16(rng.normal(size=n) * 0.1)
    res = bf16(rng.normal(size=(t, n)))
    down = rng.normal(size=(t, 2 * r)).astype(np.float32)
    bmat = bf16(rng.normal(size=(n_ad, n, r)) * 0.05)
    tok_ad = rng.integers(-1, n_ad, size=t)
    mag, want = _gemm_oracle(x, w, bias, down, bmat, tok_ad, 300, res, scale=2.0)
    if t == 16:  # these shapes compute the last tile's LoRA terms ahead (that path is covered here)
        from pagelora_b200._capi import load_library

        lib = load_library()
        assert all(lib.pl_linear_gemm_lora_precompute(t, k_in, n, c, r, 2) == 1 for c in (1, 7))
    outs = []
    for ctas in (1, 0, 7):
        y = K.linear_lora_gemm(_t(x), _t(w), bias=_t(bias), lora_down=_t(down, torch.float32), lora_b=_t(bmat),
                               lora_scale=2.0, slice_ends=(300,), tok_adapter=_i32(tok_ad), residual=_t(res),
                               num_ctas=ctas)
        torch.cuda.synchronize()
        outs.append(_np(y))
        _ulps_close(outs[-1], want, ulps=3, magnitude=mag)
    # plain projection, no epilogue extras
    y = K.linear_lora_gemm(_t(x), _t(w))
    torch.cuda.synchronize()
    _ulps_close(_np(y), bf16(x.astype(np.float64) @ w.T.astype(np.float64)), ulps=2)


def test_linear_lora_gemm_llama2_shapes(K):
    """Batched-decode shapes of Llama-2-7B (q/k/v, o, gate_up, down) at 64 tokens."""

    g = torch.Generator(device="cuda").manual_seed(1)
    for n, k in ((12288, 4096), (4096, 4096), (22016, 4096), (4096, 11008)):
        w = (torch.randn(n, k, generator=g, device="cuda") * 0.02).bfloat16()
        x = torch.randn(64, k, generator=g, device="cuda").bfloat16()
        y = K.linear_lora_gemm(x, w, weights_static=True)
        ref = x.double() @ w.double().T
        tol = torch.abs(ref) * 2.0 ** -8 + 1e-3
        assert bool(torch.all(torch.abs(y.double() - ref) <= tol)), (n, k)
        y2 = K.linear_lora_gemm(x, w, weights_static=True)  # counters were left at zero
        assert torch.equal(y, y2)


@pytest.mark.parametrize("t", [16, 64])
def test_linear_lora_gemm_qwen3_shapes_and_bands(K, t):
    """Qwen3-8B projections (q/k/v 6144, gate_up 24576 and lm_head 151936
    rows: tiles shared by several CTAs, and CTAs with many whole tiles) with
    rank-16 LoRA on 4 adapters and a residual, against an fp64 reference on
    the GPU."""

    g = torch.Generator(device="cuda").manual_seed(2)
    for n, k, lora in ((6144, 4096, True), (24576, 4096, False), (151936, 4096, True)):
        w = (torch.randn(n, k, generator=g, device="cuda") * 0.02).bfloat16()
        x = torch.randn(t, k, generator=g, device="cuda").bfloat16()
        kw = {}
        ref = x.double() @ w.double().T
        mag = ref.abs()
        if lora:
            down = torch.randn(t, 16, generator=g, device="cuda")
            bmat = (torch.randn(4, n, 16, generator=g, device="cuda") * 0.05).bfloat16()
            tok_ad = torch.arange(t, device="cuda", dtype=torch.int32) % 5 - 1  # -1: no adapter
            res = torch.randn(t, n, generator=g, device="cuda").bfloat16()
            kw = dict(lora_down=down, lora_b=bmat, lora_scale=2.0, tok_adapter=tok_ad, residual=res)
            delta = torch.einsum("tnr,tr->tn", bmat[tok_ad.clamp(min=0).long()].double(),
                                 down.bfloat16().double()) * 2.0
            delta[tok_ad < 0] = 0
            ref = res.double() + ref + delta
            mag = torch.maximum(mag, torch.maximum(res.double().abs(), ref.abs()))
        y = K.linear_lora_gemm(x, w, weights_static=True, **kw)
        # a few bf16 roundings of fp32 results (base, delta, sum, residual)
        tol = mag * 2.0 ** -6 + 1e-3
        assert bool(torch.all(torch.abs(y.double() - ref) <= tol)), (n, k)
        del w


def test_rmsnorm_and_silu_mul_vs_oracle(K):
    rng = np.random.default_rng(8)
    x = bf16(rng.normal(size=(37, 4096)) * 3)
    wn = bf16(1 + rng.normal(size=4096) * 0.1)
    y = K.rmsnorm(_t(x), _t(wn), 1e-6)
    gu = bf16(rng.normal(size=(37, 2 * 11008)))
    z = K.silu_mul(_t(gu))
    torch.cuda.synchronize()
    # one bf16 rounding of an fp32 result: the fp32 sum order may move it by one ulp
    _ulps_close(_np(y), rmsnorm_fused(x, wn, 1e-6), ulps=2)
    _ulps_close(_np(z), bf16(silu(gu[:, :11008]) * gu[:, 11008:]), ulps=2)


def test_lora_merge_weight_matches_reference(K, golden_dir):
    z = np.load(golden_dir / "lora_cases.npz")
    w, a, b, sc = _t(z["merge_w"]), _t(z["merge_a"]), _t(z["merge_b"]), float(z["merge_scale"][0])
    m0 = K.lora_merge_weight(w, a, b, sc, mode=0)
    m1 = K.lora_merge_weight(w, a, b, sc, mode=1)
    un = K.lora_merge_weight(m0, a, b, sc, mode=0, sign=-1)
    torch.cuda.synchronize()
    _ulps_close(_np(m0), z["merge_serve_merged"])
    _ulps_close(_np(m0), z["merge_effective_linear"])
    _ulps_close(_np(m1), z["merge_effective_packed"])
    _ulps_close(_np(un), z["merge_serve_unmerged"])


# ------------------------------------------------------------- glue kernels
def test_kv_append_matches_index_put(K):
    cache = torch.zeros(6, 2, 16, 4, 128, dtype=torch.bfloat16, device="cuda")
    ref = cache.clone()
    k = torch.randn(5, 4, 128, device="cuda").bfloat16()
    v = torch.randn(5, 4, 128, device="cuda").bfloat16()
    pid = _i32([3, 0, 5, 3, 1])
    off = _i32([0, 15, 7, 1, 9])
    K.kv_append(k, v, cache, pid, off)
    ref.index_put_((pid.long(), torch.zeros_like(pid).long(), off.long()), k)
    ref.index_put_((pid.long(), torch.ones_like(pid).long(), off.long()), v)
    torch.cuda.synchronize()
    assert torch.equal(cache, ref)


@pytest.mark.parametrize("qk_norm", [False, True])
def test_qkv_rope_append_vs_oracle(K, qk_norm):
    rng = np.random.default_rng(9)
    t, hq, hkv, d, r, ps = 3, 8, 2, 128, 16, 16
    n_all = (hq + 2 * hkv) * d
    qkv = bf16(rng.normal(size=(t, n_all)))
    down = rng.normal(size=(t, 3 * r)).astype(np.float32)
    bmat = bf16(rng.normal(size=(1, n_all, r)) * 0.05)
    qn = bf16(1 + rng.normal(size=d) * 0.1)
    kn = bf16(1 + rng.normal(size=d) * 0.1)
    pos = np.array([0, 17, 2047], np.int32)
    pid, off = np.array([2, 0, 3], np.int32), np.array([0, 5, 15], np.int32)
    cache = torch.zeros(4, 2, ps, hkv, d, dtype=torch.bfloat16, device="cuda")
    q_out = torch.zeros(t, hq, d, dtype=torch.bfloat16, device="cuda")
    K.qkv_rope_append(_t(qkv), num_qo_heads=hq, num_kv_heads=hkv, head_dim=d, positions=_i32(pos),
                      rope_theta=1e6, kv_cache=cache, page_id=_i32(pid), page_offset=_i32(off), q_out=q_out,
                      lora_down=_t(down, torch.float32), lora_b=_t(bmat),
                      q_norm_weight=_t(qn) if qk_norm else None, k_norm_weight=_t(kn) if qk_norm else None)
    torch.cuda.synchronize()
    full = np.zeros_like(qkv)
    for i in range(t):
        for sl, (c0, c1) in enumerate(((0, hq * d), (hq * d, (hq + hkv) * d), ((hq + hkv) * d, n_all))):
            dl = bmat[0, c0:c1] @ bf16(down[i, sl * r:(sl + 1) * r])
            full[i, c0:c1] = bf16(qkv[i, c0:c1] + bf16(dl))
    q = full[:, : hq * d].reshape(t, hq, d)
    k = full[:, hq * d:(hq + hkv) * d].reshape(t, hkv, d)
    v = full[:, (hq + hkv) * d:].reshape(t, hkv, d)
    if qk_norm:
        q, k = rmsnorm_hf(q, qn, 1e-6), rmsnorm_hf(k, kn, 1e-6)
    q, k = bf16(apply_rope(q, pos, 1e6)), bf16(apply_rope(k, pos, 1e6))
    assert np.max(np.abs(_np(q_out) - q)) <= ATOL
    c = _np(cache)
    for i in range(t):
        assert np.max(np.abs(c[pid[i], 0, off[i]] - k[i])) <= ATOL
        assert np.array_equal(c[pid[i], 1, off[i]], v[i])


def test_embed_and_argmax(K):
    table = torch.randn(1000, 256, device="cuda").bfloat16()
    ids = torch.tensor([5, 999, 0], device="cuda")
    out = torch.zeros(3, 256, dtype=torch.bfloat16, device="cuda")
    K.embed(ids, table, out)
    logits = torch.randn(4, 151936, device="cuda").bfloat16()
    logits[2, 77] = 50.0
    logits[2, 78] = 50.0  # tie: first index wins (torch.argmax)
    am = torch.zeros(4, dtype=torch.int64, device="cuda")
    K.argmax(logits, am)
    torch.cuda.synchronize()
    assert torch.equal(out, table[ids])
    assert torch.equal(am, torch.argmax(logits, -1))
    assert am[2].item() == 77
