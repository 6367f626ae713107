"""The C-ABI library loads and exports every entry point the header declares
(no compute calls: this runs without a GPU)."""

from __future__ import annotations

import re
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent


def _declared() -> set[str]:
    names = set()
    for h in (REPO / "include").glob("*.h"):
        text = h.read_text()
        names |= set(re.findall(r"^\s*(?:int32_t|const char \*)\s*(pl_\w+)\s*\(", text, flags=re.M))
    return names


@pytest.fixture(scope="module")
def lib():
    from pagelora_b200 import _capi, build

    if build.is_stale():
        build.build()
    return _capi.load_library()


def test_header_declares_the_core_entry_points():
    names = _declared()
    for n in ("pl_page_table_build", "pl_decode_plan", "pl_paged_decode", "pl_merge_states", "pl_lora_shrink_seg",
              "pl_linear_lora_expand_fused", "pl_lora_merge_weight"):
        assert n in names


def test_library_exports_every_declared_symbol(lib):
    from pagelora_b200 import _capi

    declared = _declared()
    assert declared == set(_capi.EXPORTED_SYMBOLS)
    for name in declared:
        assert hasattr(lib, name), name


def test_abi_version_and_status_strings(lib):
    assert lib.pl_abi_version() == 1
    assert lib.pl_status_string(0) == b"ok"
    assert b"offset 0" in lib.pl_status_string(5)


def test_decode_plan_is_host_only(lib):
    from pagelora_b200._capi import DecodePlan

    plan = DecodePlan()
    # batch 1, Qwen3-8B heads, 132 pages: splits fill the device (no device access needed)
    assert lib.pl_decode_plan(1, 32, 8, 128, 16, 132, 0, plan) == 0
    assert plan.num_splits > 1 and plan.ctas == 8 * plan.num_splits
    assert plan.workspace_bytes >= 32 * plan.num_splits * 128 * 4
    # large batches need no split
    assert lib.pl_decode_plan(64, 32, 32, 128, 16, 64 * 145, 0, plan) == 0
    assert plan.num_splits == 1
    # invalid heads are rejected like the reference (Q heads % KV heads)
    assert lib.pl_decode_plan(1, 28, 5, 128, 16, 10, 0, plan) == 1


def test_kernels_refuse_cpu_tensors():
    import torch

    from pagelora_b200 import kernels

    with pytest.raises(RuntimeError, match="CUDA"):
        kernels.paged_decode(torch.zeros(1, 2, 64, dtype=torch.bfloat16), torch.zeros(1, 2, 16, 2, 64),
                             torch.zeros(2, dtype=torch.int32), torch.zeros(1, dtype=torch.int32),
                             torch.zeros(1, dtype=torch.int32), num_splits=1, workspace=None)
