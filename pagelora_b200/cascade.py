"""Shared-prefix (cascade) decode: rows that share a prefix read its pages once
per group of query rows instead of once per row.

The reference's branch batches (model/flashinfer/generation.py:872-1132)
give every branch a page table that repeats the shared prefix pages, so a
decode step reads the prefix once per branch.  Here the step is split in two
attention passes whose partial states are merged by log-sum-exp:

  prefix pass  the GQA group of R rows is folded into one virtual row: for
               kv head h the M rows of the tensor-core tile are the q heads of
               h of R different rows (R * group <= 16), so each prefix page is
               read once per R rows (R = 16 / group: 4 for Qwen3's group 4,
               16 for MHA);
  suffix pass  every row over its own pages (the branch suffix and the
               decoded tokens);
  merge        the log-sum-exp merge of the two states, done by the suffix
               pass as it writes its output.

The prefix pass is pl_paged_decode_shared (the folding happens in the
kernel's q staging and output addressing), the suffix pass
pl_paged_decode_merge_prior (pl_merge_states_strided's arithmetic over
[prefix, suffix], bit-identical to a separate merge launch); two launches,
no copies.
"""

from __future__ import annotations

import torch

from pagelora_b200 import kernels as K


def fold_rows(num_rows: int, num_qo_heads: int, num_kv_heads: int) -> int:
    """Rows folded into one virtual row of the prefix pass (R * group <= 16)."""

    group = num_qo_heads // num_kv_heads
    return max(1, min(16 // group, num_rows))


class SharedPrefixDecode:
    """Decode attention for `num_rows` rows that share `prefix_pages`.

    ``prefix_pages`` are the pool pages of the shared prefix (all full except
    possibly the last, holding ``prefix_last_len`` tokens; a prefix that the
    rows continue must end on a page boundary, as the reference's usable
    prefix does, model/kvcache/paged_kvcache_manager.py:763-778).  Buffers are
    allocated once; :meth:`run` is graph-capturable."""

    def __init__(self, *, num_rows: int, num_qo_heads: int, num_kv_heads: int, head_dim: int, page_size: int,
                 prefix_pages: list[int], prefix_last_len: int, device, max_suffix_pages: int) -> None:
        self.B, self.Hq, self.Hkv, self.D = num_rows, num_qo_heads, num_kv_heads, head_dim
        self.group = num_qo_heads // num_kv_heads
        self.R = fold_rows(num_rows, num_qo_heads, num_kv_heads)
        self.Bv = -(-num_rows // self.R)
        self.page_size = page_size
        dev = torch.device(device)
        i32 = dict(device=dev, dtype=torch.int32)
        n_pre = len(prefix_pages)
        self.n_prefix_pages = n_pre
        # every virtual row lists the prefix pages
        self.pre_indptr = torch.arange(0, (self.Bv + 1) * n_pre, n_pre, **i32)
        self.pre_indices = torch.tensor(prefix_pages * self.Bv if n_pre else [0], **i32)
        self.pre_last = torch.full((self.Bv,), prefix_last_len if n_pre else 0, **i32)
        f32 = dict(device=dev, dtype=torch.float32)
        # the prefix pass's state, merged into the suffix pass's output:
        # [1][B*Hq][D] O and [1][B*Hq] LSE
        self.o_parts = torch.zeros(1, self.B * self.Hq, self.D, **f32)
        self.lse_parts = torch.zeros(1, self.B * self.Hq, **f32)
        p_pre = K.decode_plan(self.Bv, self.Hkv * self.R * self.group, self.Hkv, self.D, page_size,
                              max(1, self.Bv * n_pre))
        p_suf = K.decode_plan(self.B, self.Hq, self.Hkv, self.D, page_size, max(1, self.B * max_suffix_pages))
        self.splits_pre, self.splits_suf = int(p_pre.num_splits), int(p_suf.num_splits)
        self.ws_pre = torch.zeros(max(256, int(p_pre.workspace_bytes)), device=dev, dtype=torch.uint8)
        self.ws_suf = torch.zeros(max(256, int(p_suf.workspace_bytes)), device=dev, dtype=torch.uint8)

    def run(self, q: torch.Tensor, kv_cache: torch.Tensor, suffix_indptr: torch.Tensor,
            suffix_indices: torch.Tensor, suffix_last_len: torch.Tensor, out: torch.Tensor,
            status: torch.Tensor | None = None) -> torch.Tensor:
        """Attention of q [B, Hq, D] over prefix + each row's suffix pages -> out [B, Hq, D] bf16."""

        K.paged_decode_shared(q, kv_cache, self.pre_indptr, self.pre_indices, self.pre_last, fold=self.R,
                              num_splits=self.splits_pre, workspace=self.ws_pre, status=status,
                              out=self.o_parts[0].view(self.B, self.Hq, self.D),
                              out_lse=self.lse_parts[0].view(self.B, self.Hq))
        # the suffix pass merges the prefix pass's state into its output
        # (the log-sum-exp merge of pl_merge_states_strided, no extra launch)
        K.paged_decode(q, kv_cache, suffix_indptr, suffix_indices, suffix_last_len, num_splits=self.splits_suf,
                       workspace=self.ws_suf, status=status, out=out,
                       prior=(self.o_parts[0], self.lse_parts[0]))
        return out

    def prefix_bytes_per_layer(self) -> int:
        """KV bytes of the prefix read per layer by the prefix pass (once per virtual row)."""

        return self.Bv * self.n_prefix_pages * self.page_size * self.Hkv * self.D * 2 * 2
