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
        names |= set(re.findall(r"^\s*(?:int32_t|int64_t|const char \*)\s*(pl_\w+)\s*\(", text, flags=re.M))
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


@pytest.mark.parametrize("struct_name", ["GemvPhase", "GemvPrefetch"])
def test_gemv_structs_match_the_header(tmp_path, struct_name):
    """The ctypes GemvPhase / GemvPrefetch have the size and field offsets of
    the C PlGemvPhase / PlGemvPrefetch."""

    import ctypes
    import shutil
    import subprocess

    from pagelora_b200 import _capi

    gcc = shutil.which("gcc")
    if gcc is None:
        pytest.skip("gcc not available")
    cls = getattr(_capi, struct_name)
    c_name = "Pl" + struct_name
    fields = [f[0] for f in cls._fields_]
    src = tmp_path / "layout.c"
    src.write_text(
        '#include <stddef.h>\n#include <stdio.h>\n#include "pagelora_b200.h"\n'
        "int main(void) {\n"
        f'  printf("size %zu\\n", sizeof({c_name}));\n'
        + "".join(f'  printf("{f} %zu\\n", offsetof({c_name}, {f}));\n' for f in fields)
        + "  return 0;\n}\n")
    exe = tmp_path / "layout"
    subprocess.run([gcc, "-std=c11", "-I", str(REPO / "include"), str(src), "-o", str(exe)], check=True)
    out = dict(line.split() for line in subprocess.run([str(exe)], check=True, capture_output=True,
                                                       text=True).stdout.splitlines())
    assert int(out["size"]) == ctypes.sizeof(cls)
    for f in fields:
        assert int(out[f]) == getattr(cls, f).offset, f


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


def test_linear_lora_phase_host_checks(lib):
    """Argument errors of pl_linear_lora_phase's hand-over are found on the
    host, before any device call."""

    import ctypes

    from pagelora_b200._capi import GemvPrefetch

    ph = _phase()
    def pf(**over):
        p = GemvPrefetch()
        p.w, p.n_out, p.k_in, p.num_tokens, p.units = 0x20000, 64, 64, 1, 1
        for k, v in over.items():
            setattr(p, k, v)
        return ctypes.byref(p)
    assert lib.pl_linear_lora_phase(None, None, None, None) == 1
    assert lib.pl_linear_lora_phase(ctypes.byref(ph), pf(w=None), None, None) == 1
    assert lib.pl_linear_lora_phase(ctypes.byref(ph), pf(units=-1), None, None) == 1
    assert lib.pl_linear_lora_phase(ctypes.byref(ph), pf(num_tokens=9), None, None) == 1
    assert lib.pl_linear_lora_phase(ctypes.byref(ph), pf(n_shrink=8), None, None) == 1   # rows without a matrix
    assert lib.pl_linear_lora_phase(ctypes.byref(ph), pf(w=0x20008), None, None) == 1    # misaligned
    assert lib.pl_linear_lora_phase(ctypes.byref(ph), pf(k_in=40), None, None) == 2      # K % 16
