"""Shared-prefix (cascade) decode vs plain paged decode over each row's full page list.

Rows share a prefix of pages; the cascade reads the prefix once per group of
rows folded into one tensor-core tile and merges that state with each row's
suffix state.  The result must equal plain decode over prefix + suffix pages
within the attention tolerance (max |err| <= 2e-2), and the prefix bytes read
must shrink by the folding factor.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle.numerics import bf16
from oracle.paged_decode import paged_decode as o_decode

pytestmark = pytest.mark.gpu

ATOL = 2e-2


@pytest.mark.parametrize("rows,hq,hkv,prefix_tokens", [(16, 32, 8, 2048), (5, 32, 8, 200), (3, 16, 16, 64),
                                                       (9, 8, 2, 31)])
def test_cascade_matches_full_decode(cuda_device, rows, hq, hkv, prefix_tokens):
    from pagelora_b200 import kernels as K
    from pagelora_b200.cascade import SharedPrefixDecode, fold_rows

    rng = np.random.default_rng(rows + hq + prefix_tokens)
    ps, d = 16, 128
    n_pre = -(-prefix_tokens // ps)
    pre_last = prefix_tokens - (n_pre - 1) * ps
    suf_lens = rng.integers(1, 90, size=rows).tolist()
    suf_pages = [-(-n // ps) for n in suf_lens]
    pool = n_pre + sum(suf_pages) + 3
    cache = bf16(rng.normal(size=(pool, 2, ps, hkv, d)))
    perm = rng.permutation(pool).tolist()
    prefix = perm[:n_pre]
    suffix, off = [], n_pre
    for n in suf_pages:
        suffix.append(perm[off:off + n])
        off += n
    q = bf16(rng.normal(size=(rows, hq, d)) * 1.5)
    dev = "cuda"
    ct = torch.as_tensor(cache).to(dev, torch.bfloat16)
    qt = torch.as_tensor(q).to(dev, torch.bfloat16)
    s_indptr = torch.tensor(np.cumsum([0] + suf_pages), dtype=torch.int32, device=dev)
    s_indices = torch.tensor([p for s in suffix for p in s], dtype=torch.int32, device=dev)
    s_last = torch.tensor([n - (p - 1) * ps for n, p in zip(suf_lens, suf_pages)], dtype=torch.int32, device=dev)
    casc = SharedPrefixDecode(num_rows=rows, num_qo_heads=hq, num_kv_heads=hkv, head_dim=d, page_size=ps,
                              prefix_pages=prefix, prefix_last_len=pre_last, device=dev, max_suffix_pages=max(suf_pages))
    out = torch.empty(rows, hq, d, dtype=torch.bfloat16, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    casc.run(qt, ct, s_indptr, s_indices, s_last, out, status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    # reference: each row over prefix + suffix pages.  The prefix's last page may be
    # partial, so the oracle sees it as a separate row segment via two passes merged.
    ref = np.zeros((rows, hq, d))
    from oracle.paged_decode import merge_states

    o1, l1 = o_decode(q, cache, [i * n_pre for i in range(rows + 1)], prefix * rows, [pre_last] * rows)
    o2, l2 = o_decode(q, cache, np.cumsum([0] + suf_pages).tolist(), [p for s in suffix for p in s],
                      [n - (p - 1) * ps for n, p in zip(suf_lens, suf_pages)])
    ref, _ = merge_states(np.stack([o1, o2]), np.stack([l1, l2]))
    got = out.float().cpu().numpy()
    assert np.max(np.abs(got - ref)) <= ATOL
    # when the prefix ends on a page boundary, plain decode over the concatenated
    # page lists is the same attention
    if pre_last == ps:
        full_indptr = np.cumsum([0] + [n_pre + p for p in suf_pages])
        full_idx = [x for s in suffix for x in prefix + s]
        full_last = [n - (p - 1) * ps for n, p in zip(suf_lens, suf_pages)]
        ws = torch.zeros(8 << 20, dtype=torch.uint8, device=dev)
        plain = K.paged_decode(qt, ct, torch.tensor(full_indptr, dtype=torch.int32, device=dev),
                               torch.tensor(full_idx, dtype=torch.int32, device=dev),
                               torch.tensor(full_last, dtype=torch.int32, device=dev), num_splits=4, workspace=ws)
        torch.cuda.synchronize()
        assert np.max(np.abs(plain.float().cpu().numpy() - got)) <= ATOL
    r = fold_rows(rows, hq, hkv)
    assert casc.Bv == -(-rows // r)  # the prefix is read once per folded group of r rows
    assert casc.prefix_bytes_per_layer() == casc.Bv * n_pre * ps * hkv * d * 4
