"""Split-KV exchange of partial attention states over NVLink peer memory.

Split-KV decode over GPUs (configs 5-style: one long context spread over the
GPUs' memories) merges per layer the partial (O, LSE) states of every GPU.
The reference runs on one GPU, so there is no reference counterpart; the
plain form is an NCCL all-gather of the packed partials plus a merge launch
(``BatchDecodeEngine`` with ``exchange="nccl"``).  ``PeerExchange`` does the
exchange and the merge in one kernel (``pl_splitkv_exchange_merge``): each GPU
stores its partial straight into the other GPUs' gather buffers through
CUDA IPC mappings, raises per-CTA flags there, waits (bounded) for theirs and
merges locally, bit-identically to the all-gather path.

torch.distributed is used only at set-up, to swap the IPC handles.  Buffers
are ordinary torch allocations; the library allocates nothing.
"""

from __future__ import annotations

import ctypes

import torch

from pagelora_b200 import _capi
from pagelora_b200._capi import call, ptr, stream_handle


class PeerExchangeUnavailable(RuntimeError):
    """The peer mappings could not be set up on every rank (raised on all of them)."""


class PeerExchange:
    """Per-GPU state of the peer exchange for partials of ``rows_h`` rows of
    ``head_dim``; every rank of ``group`` constructs one with the same shape,
    in the same order (the constructor runs collectives)."""

    def __init__(self, rows_h: int, head_dim: int, *, group=None, device=None, rows_per_cta: int = 2) -> None:
        import torch.distributed as dist

        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        if self.world < 2:
            raise ValueError("the peer exchange needs at least two GPUs")
        self.group = group
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.rows_h, self.head_dim, self.rows_per_cta = int(rows_h), int(head_dim), int(rows_per_cta)
        lib = _capi.load_library()
        self.slot = int(lib.pl_splitkv_exchange_slot_floats(self.rows_h, self.head_dim))
        self.ctas = int(lib.pl_splitkv_exchange_ctas(self.rows_h, self.rows_per_cta))
        dev = self.device
        self.gather = torch.zeros(2, self.world, self.slot, device=dev, dtype=torch.float32)
        self.flags = torch.zeros(self.world, self.ctas, device=dev, dtype=torch.int32)
        self.epochs = torch.zeros(self.ctas, device=dev, dtype=torch.int32)
        if dev.type == "cuda":
            torch.cuda.synchronize(dev)
        # Swap (handle, offset) of both buffers with every rank.
        hb = int(lib.pl_ipc_handle_bytes())
        mine = []
        error = None
        try:
            for t in (self.gather, self.flags):
                h = (ctypes.c_uint8 * hb)()
                off = ctypes.c_int64(0)
                call("pl_ipc_export", ptr(t), h, ctypes.byref(off))
                mine.append((bytes(h), off.value))
        except Exception as e:  # noqa: BLE001 - every rank still joins the collectives below
            error, mine = e, [(bytes(hb), 0), (bytes(hb), 0)]
        blob = torch.zeros(2 * (hb + 8), dtype=torch.uint8)
        for i, (h, off) in enumerate(mine):
            blob[i * (hb + 8): i * (hb + 8) + hb] = torch.frombuffer(bytearray(h), dtype=torch.uint8)
            blob[i * (hb + 8) + hb: (i + 1) * (hb + 8)] = torch.frombuffer(
                bytearray(off.to_bytes(8, "little", signed=True)), dtype=torch.uint8)
        send = blob.to(dev)
        recv = torch.zeros(self.world * send.numel(), dtype=torch.uint8, device=dev)
        dist.all_gather_into_tensor(recv, send, group=group)
        recv = recv.cpu().view(self.world, send.numel())
        self._opened: list[tuple[int, int]] = []  # (mapped pointer, offset) to close
        gptrs, fptrs = [], []
        try:
            if error is not None:
                raise error
            for p in range(self.world):
                if p == self.rank:
                    gptrs.append(ptr(self.gather))
                    fptrs.append(ptr(self.flags))
                    continue
                row = recv[p]
                for i, dst in enumerate((gptrs, fptrs)):
                    base = i * (hb + 8)
                    h = (ctypes.c_uint8 * hb)(*row[base: base + hb].tolist())
                    off = int.from_bytes(bytes(row[base + hb: base + hb + 8].tolist()), "little", signed=True)
                    out = ctypes.c_void_p()
                    call("pl_ipc_import", h, off, ctypes.byref(out))
                    self._opened.append((out.value, off))
                    dst.append(out.value)
        except Exception as e:  # noqa: BLE001 - reported on every rank below
            error = e
        # every rank learns whether all of them mapped their peers
        ok = torch.tensor([0 if error is not None else 1], dtype=torch.int32, device=dev)
        dist.all_reduce(ok, op=dist.ReduceOp.MIN, group=group)
        if int(ok.item()) == 0:
            self.close()
            raise PeerExchangeUnavailable(f"peer mappings failed on some rank ({error or 'another rank'})")
        self.peer_gather = torch.tensor(gptrs, dtype=torch.int64, device=dev)
        self.peer_flags = torch.tensor(fptrs, dtype=torch.int64, device=dev)
        if dev.type == "cuda":
            torch.cuda.synchronize(dev)
        dist.barrier(group=group)

    def merge(self, part: torch.Tensor, out: torch.Tensor, status: torch.Tensor | None = None) -> torch.Tensor:
        """Exchange this GPU's packed partial ``part`` (O [rows_h, D] fp32
        then LSE [rows_h]) with every other GPU and write the merged bf16
        ``out`` [rows_h, D] (graph-capturable; every rank must call it)."""

        if part.dtype != torch.float32 or not part.is_contiguous() or part.numel() < self.rows_h * (self.head_dim + 1):
            raise ValueError("part must be a contiguous fp32 [rows_h * (D + 1)] tensor")
        if out.dtype != torch.bfloat16 or not out.is_contiguous() or out.numel() != self.rows_h * self.head_dim:
            raise ValueError("out must be a contiguous bf16 [rows_h, D] tensor")
        call("pl_splitkv_exchange_merge", ptr(part), ptr(self.peer_gather), ptr(self.peer_flags), ptr(self.flags),
             ptr(self.epochs), self.rank, self.world, self.rows_h, self.head_dim, self.rows_per_cta, ptr(out),
             ptr(status), stream_handle())
        return out

    def close(self) -> None:
        """Unmap the peers' buffers.  Call it on every rank after the last
        exchange has completed everywhere (e.g. after a barrier), and before
        the buffers' owners free them."""

        for p, off in self._opened:
            call("pl_ipc_close", p, off)
        self._opened = []
