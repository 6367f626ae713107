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


def test_gemv_phase_struct_matches_the_header(tmp_path):
    """ctypes GemvPhase has the size and field offsets of the C PlGemvPhase."""

    import ctypes
    import shutil
    import subprocess

    from pagelora_b200._capi import GemvPhase

    gcc = shutil.which("gcc")
    if gcc is None:
        pytest.skip("gcc not available")
    fields = [f[0] for f in GemvPhase._fields_]
    src = tmp_path / "layout.c"
    src.write_text(
        '#include <stddef.h>\n#include <stdio.h>\n#include "pagelora_b200.h"\n'
        "int main(void) {\n"
        '  printf("size %zu\\n", sizeof(PlGemvPhase));\n'
        + "".join(f'  printf("{f} %zu\\n", offsetof(PlGemvPhase, {f}));\n' for f in fields)
        + "  return 0;\n}\n")
    exe = tmp_path / "layout"
    subprocess.run([gcc, "-std=c11", "-I", str(REPO / "include"), str(src), "-o", str(exe)], check=True)
    out = dict(line.split() for line in subprocess.run([str(exe)], check=True, capture_output=True,
                                                       text=True).stdout.splitlines())
    assert int(out["size"]) == ctypes.sizeof(GemvPhase)
    for f in fields:
        assert int(out[f]) == getattr(GemvPhase, f).offset, f


def _phase(tokens=1, k=64, n=32, **over):
    from pagelora_b200._capi import GemvPhase

    ph = GemvPhase()
    # aligned placeholder addresses: the host checks never dereference them
    ph.x, ph.x_stride, ph.num_tokens, ph.k_in = 0x10000, k, tokens, k
    ph.w, ph.n_out, ph.y, ph.y_stride, ph.num_slices = 0x20000, n, 0x30000, n, 1
    for key, v in over.items():
        setattr(ph, key, v)
    return ph


def test_linear_lora_chain_host_checks(lib):
    """Argument errors of pl_linear_lora_chain are found on the host, before
    any device call."""

    from pagelora_b200._capi import GemvPhase

    arr = (GemvPhase * 7)(*[_phase() for _ in range(7)])
    barrier = 0x40000  # placeholder device address
    assert lib.pl_linear_lora_chain(arr, 0, None, None, None) == 0          # nothing to do
    assert lib.pl_linear_lora_chain(arr, 7, barrier, None, None) == 2       # more than 6 phases
    assert lib.pl_linear_lora_chain(arr, 2, None, None, None) == 1          # no grid barrier
    assert lib.pl_linear_lora_chain(arr, 2, barrier + 2, None, None) == 1  # misaligned barrier
    mixed = (GemvPhase * 2)(_phase(tokens=1), _phase(tokens=2))
    assert lib.pl_linear_lora_chain(mixed, 2, barrier, None, None) == 1     # token counts differ
    big = (GemvPhase * 1)(_phase(tokens=9))
    assert lib.pl_linear_lora_chain(big, 1, None, None, None) == 1          # > 8 tokens
    odd = (GemvPhase * 1)(_phase(k=40))
    assert lib.pl_linear_lora_chain(odd, 1, None, None, None) == 2          # K % 16
    # a phase reading the shrink output of an earlier phase as its LoRA down
    shrink = _phase(shrink_a=0x50000, n_shrink=48, shrink_out=0x60000, shrink_stride=48)
    reader = _phase(lora_b=0x70000, lora_rank=16, lora_down=0x60000 + 16 * 4, down_stride=48)
    dep = (GemvPhase * 2)(shrink, reader)
    assert lib.pl_linear_lora_chain(dep, 2, barrier, None, None) == 2
