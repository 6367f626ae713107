"""ctypes binding of the C ABI in ``include/pagelora_b200.h``.

This module is the only place that touches the shared library.  It loads
``pagelora_b200/lib/libpagelora_b200.so`` (built in-tree by
``python -m pagelora_b200.build``), declares every entry point's argument
types, and turns non-zero status codes into Python exceptions.  There is no
fallback: if the library or a CUDA device is missing, calls raise.
"""

from __future__ import annotations

import ctypes
import threading
from ctypes import POINTER, Structure, c_char_p, c_float, c_int32, c_int64, c_void_p
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "lib" / "libpagelora_b200.so"

PL_OK = 0
PL_ERR_INVALID_ARGUMENT = 1
PL_ERR_UNSUPPORTED = 2
PL_ERR_PAGE_OUT_OF_RANGE = 3
PL_ERR_WORKSPACE_TOO_SMALL = 4
PL_ERR_SPAN_START = 5
PL_ERR_SPAN_LENGTH = 6
PL_ERR_SPAN_NOT_FULL = 7
PL_ERR_CUDA = 8
PL_ERR_TIMEOUT = 9
PL_ERR_NO_DEVICE = 10

PL_PROLOGUE_NONE = 0
PL_PROLOGUE_RMSNORM = 1
PL_PROLOGUE_SILU_MUL = 2
PL_FLAG_WEIGHTS_STATIC = 1
PL_FLAG_DOWN_FROM_X = 2
PL_FLAG_SILU_PAIRS = 8
PL_DECODE_OUT_F32 = 1

# Messages of the reference's ValueErrors for malformed spans
# (model/kvcache/flashinfer_page_table.py:213-218).
SPAN_ERROR_MESSAGES = {
    PL_ERR_SPAN_START: "FlashInfer page spans must start at page offset 0",
    PL_ERR_SPAN_LENGTH: "FlashInfer page span length is out of range",
    PL_ERR_SPAN_NOT_FULL: "non-last FlashInfer page spans must be full pages",
}


class DecodePlan(Structure):
    _fields_ = [("num_splits", c_int32), ("ctas", c_int32), ("workspace_bytes", c_int64)]


class GemmPlan(Structure):
    _fields_ = [("ctas", c_int32), ("max_slots", c_int32), ("workspace_bytes", c_int64)]


class GemvPhase(Structure):
    """PlGemvPhase: one projection of pl_linear_lora_chain."""

    _fields_ = [("x", c_void_p), ("x_stride", c_int64), ("num_tokens", c_int32), ("k_in", c_int32),
                ("prologue", c_int32), ("norm_w", c_void_p), ("norm_eps", c_float), ("w", c_void_p),
                ("n_out", c_int32), ("bias", c_void_p), ("lora_down", c_void_p), ("down_stride", c_int64),
                ("lora_b", c_void_p), ("lora_rank", c_int32), ("lora_scale", c_float),
                ("slice_end", c_int32 * 3), ("num_slices", c_int32), ("tok_adapter", c_void_p),
                ("residual", c_void_p), ("res_stride", c_int64), ("y", c_void_p), ("y_stride", c_int64),
                ("shrink_a", c_void_p), ("n_shrink", c_int32), ("shrink_out", c_void_p),
                ("shrink_stride", c_int64), ("flags", c_int32)]


class GemvPrefetch(Structure):
    """PlGemvPrefetch: the next projection of pl_linear_lora_phase's L2 hand-over."""

    _fields_ = [("w", c_void_p), ("n_out", c_int32), ("shrink_a", c_void_p), ("n_shrink", c_int32),
                ("k_in", c_int32), ("num_tokens", c_int32), ("units", c_int32)]


_P = c_void_p
_I32 = c_int32
_I64 = c_int64
_F = c_float

# name -> (restype, argtypes)
_SIGNATURES: dict[str, tuple[object, list[object]]] = {
    "pl_abi_version": (_I32, []),
    "pl_status_string": (c_char_p, [_I32]),
    "pl_last_cuda_error": (c_char_p, []),
    "pl_device_sm_count": (_I32, []),
    "pl_page_table_build": (_I32, [_P, _P, _P, _P, _I32, _I32, _P, _P, _P, _P, _P, _P]),
    "pl_page_table_advance": (_I32, [_P, _P, _P, _P, _I32, _I32, _I32, _P, _P, _P, _P, _P, _P, _P]),
    "pl_decode_plan": (_I32, [_I32, _I32, _I32, _I32, _I32, _I64, _I32, POINTER(DecodePlan)]),
    "pl_paged_decode": (
        _I32,
        [_P, _I64, _I64, _P, _I64, _P, _P, _P, _I32, _I32, _I32, _I32, _I32, _F, _I32, _P, _I64, _I64, _P, _P,
         _I64, _P, _P],
    ),
    "pl_paged_decode_fixed_scratch": (
        _I32,
        [_P, _I64, _I64, _P, _I64, _P, _P, _P, _I32, _I32, _I32, _I32, _I32, _F, _I32, _P, _I64, _I64, _P, _P, _P],
    ),
    "pl_fixed_scratch_clear": (_I32, [_P]),
    "pl_paged_decode_f32": (
        _I32,
        [_P, _I64, _I64, _P, _I64, _P, _P, _P, _I32, _I32, _I32, _I32, _I32, _F, _I32, _P, _I64, _I64, _P, _P,
         _I64, _P, _P],
    ),
    "pl_paged_decode_qkv": (
        _I32,
        [_P, _I64, _P, _I64, _P, _I32, _F, _P, _P, _P, _F, _P, _F, _P, _P, _P, _P, _P, _I64, _P, _P, _P, _I32,
         _I32, _I32, _I32, _I32, _F, _I32, _P, _I64, _I64, _P, _I32, _P, _I64, _P, _P],
    ),
    "pl_rope_cos_sin": (_I32, [_P, _I32, _I32, _F, _P, _P]),
    "pl_paged_decode_shared": (
        _I32,
        [_P, _I64, _I64, _P, _I64, _P, _P, _P, _I32, _I32, _I32, _I32, _I32, _I32, _F, _I32, _P, _I64, _I64, _P,
         _I32, _P, _I64, _P, _P],
    ),
    "pl_decode_set_cluster_merge": (_I32, [_I32]),
    "pl_decode_cluster_capacity": (_I32, [_I32, _I32, _I32]),
    "pl_merge_states": (_I32, [_P, _P, _I32, _I32, _I32, _P, _I64, _P, _P]),
    "pl_merge_states_strided": (_I32, [_P, _I64, _I64, _P, _I64, _I64, _I32, _I32, _I32, _P, _I64, _P, _P]),
    "pl_paged_decode_merge_prior": (
        _I32,
        [_P, _I64, _I64, _P, _I64, _P, _P, _P, _I32, _I32, _I32, _I32, _I32, _F, _I32, _P, _I64, _I64, _P, _P, _P,
         _I64, _P, _P],
    ),
    "pl_ipc_handle_bytes": (_I32, []),
    "pl_ipc_export": (_I32, [_P, _P, POINTER(c_int64)]),
    "pl_ipc_import": (_I32, [_P, _I64, POINTER(c_void_p)]),
    "pl_ipc_close": (_I32, [_P, _I64]),
    "pl_splitkv_exchange_slot_floats": (_I64, [_I32, _I32]),
    "pl_splitkv_exchange_ctas": (_I32, [_I32, _I32]),
    "pl_splitkv_exchange_merge": (_I32, [_P, _P, _P, _P, _P, _I32, _I32, _I32, _I32, _I32, _P, _P, _P]),
    "pl_paged_prefill": (
        _I32,
        [_P, _I64, _I64, _P, _I64, _P, _P, _P, _P, _I32, _I32, _I32, _I32, _I32, _I32, _F, _I32, _P, _I64, _I64,
         _P, _P, _P],
    ),
    "pl_lora_shrink_seg": (_I32, [_P, _I64, _P, _I32, _I32, _I32, _P, _P, _I32, _I32, _P, _I64, _P]),
    "pl_lora_shrink_rows": (_I32, [_P, _I64, _I32, _I32, _P, _F, _P, _I64, _P, _I32, _I32, _P, _P, _I64, _P]),
    "pl_linear_lora_expand_fused": (
        _I32,
        [_P, _I64, _I32, _I32, _I32, _P, _F, _P, _I32, _P, _P, _I64, _P, _I32, _F, _P, _I32, _P, _P, _I64, _P,
         _I64, _P, _I32, _P, _I64, _I32, _P, _P],
    ),
    "pl_linear_lora_chain": (_I32, [POINTER(GemvPhase), _I32, _P, _P, _P]),
    "pl_linear_lora_phase": (_I32, [POINTER(GemvPhase), POINTER(GemvPrefetch), _P, _P]),
    "pl_linear_set_tuning": (_I32, [_I32, _I32, _I32, _I32, _I32]),
    "pl_linear_set_l2_prefetch": (_I32, [_I64]),
    "pl_linear_gemm_plan": (_I32, [_I32, _I32, _I32, _I32, POINTER(GemmPlan)]),
    "pl_linear_gemm_lora_precompute": (_I32, [_I32, _I32, _I32, _I32, _I32, _I32]),
    "pl_linear_lora_gemm": (
        _I32,
        [_P, _I64, _I32, _I32, _P, _I32, _P, _P, _I64, _P, _I32, _F, _P, _I32, _P, _P, _I64, _P, _I64, _I32, _P,
         _I64, _I32, _P, _P],
    ),
    "pl_rmsnorm": (_I32, [_P, _I64, _I32, _I32, _P, _F, _P, _I64, _P]),
    "pl_rmsnorm_hf": (_I32, [_P, _I64, _I32, _I32, _P, _F, _P, _I64, _P]),
    "pl_silu_mul": (_I32, [_P, _I64, _I32, _I32, _P, _I64, _P]),
    "pl_lora_merge_weight": (_I32, [_P, _P, _P, _P, _I32, _I32, _I32, _F, _I32, _I32, _P]),
    "pl_kv_append": (_I32, [_P, _I64, _P, _I64, _P, _I64, _P, _P, _I32, _I32, _I32, _I32, _P, _P]),
    "pl_qkv_rope_append": (
        _I32,
        [_P, _I64, _P, _I64, _P, _I32, _F, _P, _P, _P, _F, _P, _F, _P, _P, _I64, _P, _P, _I32, _I32, _I32,
         _I32, _I32, _P, _P],
    ),
    "pl_embed": (_I32, [_P, _P, _I64, _I32, _I32, _P, _P, _P]),
    "pl_argmax": (_I32, [_P, _I64, _I32, _I32, _P, _P, _I64, _P]),
}

EXPORTED_SYMBOLS = tuple(_SIGNATURES)

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


class PageLoRAError(RuntimeError):
    """A C-ABI call returned a non-zero status."""

    def __init__(self, fn: str, status: int, detail: str = "") -> None:
        self.fn = fn
        self.status = status
        msg = f"{fn} failed: {status_string(status)} (status {status})"
        if detail:
            msg += f": {detail}"
        super().__init__(msg)


def load_library(path: Path | None = None) -> ctypes.CDLL:
    """Load (once) and return the shared library with typed entry points."""

    global _lib
    with _lock:
        if _lib is not None and path is None:
            return _lib
        lib_path = Path(path) if path is not None else LIB_PATH
        if not lib_path.exists():
            raise RuntimeError(
                f"{lib_path} is not built; run `python -m pagelora_b200.build` (nvcc, sm_100a)"
            )
        lib = ctypes.CDLL(str(lib_path))
        for name, (restype, argtypes) in _SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = restype
            fn.argtypes = argtypes
        if lib.pl_abi_version() != 1:
            raise RuntimeError(f"{lib_path} has ABI {lib.pl_abi_version()}, expected 1")
        if path is None:
            _lib = lib
        return lib


def status_string(status: int) -> str:
    try:
        return load_library().pl_status_string(int(status)).decode()
    except Exception:  # library unavailable while formatting an error
        return f"status {status}"


def check(fn: str, status: int) -> None:
    """Raise for a non-zero status returned by ``fn``."""

    if status == PL_OK:
        return
    detail = ""
    if status == PL_ERR_CUDA:
        detail = load_library().pl_last_cuda_error().decode()
    if status in SPAN_ERROR_MESSAGES:
        raise ValueError(SPAN_ERROR_MESSAGES[status])
    raise PageLoRAError(fn, status, detail)


def call(fn: str, *args) -> None:
    """Call ``fn`` from the library and raise on a non-zero status."""

    lib = load_library()
    check(fn, getattr(lib, fn)(*args))


def ptr(tensor) -> int | None:
    """Raw device pointer of a tensor (None for None)."""

    if tensor is None:
        return None
    return int(tensor.data_ptr())


def stream_handle(stream=None) -> int:
    """cudaStream_t of a torch stream (the current stream by default)."""

    import torch

    if stream is None:
        stream = torch.cuda.current_stream()
    return int(stream.cuda_stream)
