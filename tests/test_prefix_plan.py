"""Prefix reuse and page admission (pagelora_b200/prefix_plan.py) against the
reference's own KV manager (tests/golden/prefix_plans.json, written by
tests/golden/make_golden.py from model/kvcache/paged_kvcache_manager.py).

Each fixture request holds the radix lookup result the reference computed
(key_match_len, key_spans) and what the manager made of it (match_len,
prefill_from, prefix_spans, admission answers); each scenario holds the
batch page table of the rows' prefix + new spans.  Everything is integer
work and must match exactly.  The first scenario is BASELINE config 4: a
2048-token prefix shared by 16 branches of 64 new tokens at page size 16.
"""

from __future__ import annotations

import json

import pytest

from oracle import page_table as opt
from pagelora_b200 import prefix_plan as pp
from pagelora_b200.page_table import KVBlockSpan


@pytest.fixture(scope="module")
def cases(golden_dir):
    return json.loads((golden_dir / "prefix_plans.json").read_text())["cases"]


def _spans(rows):
    return [KVBlockSpan(*s) for s in rows]


def test_plan_prefix_matches_reference_manager(cases):
    n = 0
    for case in cases:
        ps = case["page_size"]
        for row in case["rows"]:
            plan = pp.plan_prefix(row["prompt_len"], row["key_match_len"], _spans(row["key_spans"]), ps)
            assert plan.match_len == row["match_len"]
            assert plan.prefill_from == row["prefill_from"]
            assert [[s.block_id, s.start, s.length] for s in plan.prefix_spans] == row["prefix_spans"]
            n += 1
    assert n == sum(len(c["rows"]) for c in cases) >= 28


def test_admission_matches_reference_manager(cases):
    for case in cases:
        ps, avail, reserve = case["page_size"], case["available_pages"], len(case["rows"])
        for row in case["rows"]:
            new = row["prompt_len"] - row["prefill_from"]
            assert pp.estimate_request_new_pages(new, 128, ps) == row["new_pages"]
            assert pp.can_fit_request(new, 128, ps, avail, reserve_pages=reserve) == row["fits"]
            assert pp.max_decode_tokens_that_fit(new, 100000, ps, avail, reserve_pages=reserve) == row["max_decode"]


def test_branch_batch_page_tables_match_reference(cases):
    for case in cases:
        indptr, indices, last = opt.build_batch(case["row_spans"], case["page_size"])
        assert (indptr, indices, last) == (case["indptr"], case["indices"], case["last_page_len"])


def test_config4_branches_share_the_prefix_pages(cases):
    c4 = cases[0]
    assert c4["page_size"] == 16 and len(c4["rows"]) == 16
    prefix_pages = {tuple(tuple(s) for s in row["prefix_spans"]) for row in c4["rows"]}
    assert len(prefix_pages) == 1  # every branch reuses the same 128 pages
    (spans,) = prefix_pages
    assert len(spans) == 128 and all(s[1] == 0 and s[2] == 16 for s in spans)
    assert all(row["prefill_from"] == 2048 for row in c4["rows"])


def test_usable_prefix_and_slicing_edge_cases():
    sp = _spans([[5, 0, 16], [6, 0, 16], [7, 0, 3]])
    assert pp.usable_prefix_len(sp, 35, 16) == 32
    assert pp.usable_prefix_len(sp, 20, 16) == 16
    assert pp.usable_prefix_len(sp, 0, 16) == 0
    assert pp.usable_prefix_len(_spans([[5, 1, 15]]), 15, 16) == 0  # not from offset 0
    # adjacent slices of one page coalesce into a whole page
    assert pp.usable_prefix_len(_spans([[9, 0, 8], [9, 8, 8], [3, 0, 2]]), 18, 16) == 16
    assert pp.slice_block_spans(sp, 10, 10) == [KVBlockSpan(5, 10, 6), KVBlockSpan(6, 0, 4)]
    with pytest.raises(ValueError, match="out of range"):
        pp.slice_block_spans(sp, 30, 10)
    with pytest.raises(ValueError, match="non-negative"):
        pp.slice_block_spans(sp, -1, 1)
    # a full-prompt hit replays the last prompt token
    plan = pp.plan_prefix(32, 32, sp, 16)
    assert plan.match_len == 32 and plan.prefill_from == 16
