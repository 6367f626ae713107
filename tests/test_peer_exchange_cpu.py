"""Set-up of the split-KV peer exchange (pagelora_b200.peer_exchange) on two
gloo ranks on the CPU, with the CUDA IPC entry points replaced by fakes.

What is checked is the agreement that keeps ranks from waiting on each other
for ever: when the peer mapping fails on one rank, every rank raises
PeerExchangeUnavailable at the same point (and closes what it had mapped),
so a caller can fall back to the all-gather on all ranks together; when it
succeeds everywhere, every rank holds the peers' pointers in rank order.
"""

from __future__ import annotations

import os
import socket

import pytest


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, fail_rank: int, results) -> None:
    import torch.distributed as dist

    from pagelora_b200 import peer_exchange as pe

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    closed = []

    def fake_call(fn, *args):
        if fn == "pl_ipc_export":
            dev_ptr, handle, offset = args
            # handle bytes: the exporting rank's id; offset: low bits of the pointer
            for i in range(len(handle)):
                handle[i] = rank
            offset._obj.value = 16
        elif fn == "pl_ipc_import":
            handle, off, out = args
            if rank == fail_rank:
                raise RuntimeError("fake import failure")
            out._obj.value = 0x10000 * (handle[0] + 1) + off
        elif fn == "pl_ipc_close":
            closed.append(args)
        else:
            raise AssertionError(fn)

    pe.call = fake_call
    try:
        ex = pe.PeerExchange(8, 64, device="cpu")
        results[f"ok{rank}"] = True
        results[f"gather{rank}"] = ex.peer_gather.tolist()
        ex.close()
    except pe.PeerExchangeUnavailable as e:
        results[f"ok{rank}"] = False
        results[f"msg{rank}"] = str(e)
    results[f"closed{rank}"] = len(closed)
    dist.barrier()
    dist.destroy_process_group()


def _run(fail_rank: int, world: int = 3) -> dict:
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    with ctx.Manager() as mgr:
        results = mgr.dict()
        port = _free_port()
        procs = [ctx.Process(target=_worker, args=(r, world, port, fail_rank, results)) for r in range(world)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout=120)
        assert all(p.exitcode == 0 for p in procs)
        return dict(results)


def test_peer_exchange_setup_succeeds_on_every_rank():
    res = _run(fail_rank=-1)
    for r in range(3):
        assert res[f"ok{r}"] is True
        g = res[f"gather{r}"]
        # own buffer at index r, the peers' mapped pointers (fake: 0x10000 * (peer + 1) + offset) elsewhere
        for p in range(3):
            if p != r:
                assert g[p] == 0x10000 * (p + 1) + 16
        assert res[f"closed{r}"] == 2 * 2  # two buffers of each of the two peers


@pytest.mark.parametrize("fail_rank", [0, 2])
def test_peer_exchange_failure_on_one_rank_is_raised_on_every_rank(fail_rank):
    res = _run(fail_rank=fail_rank)
    for r in range(3):
        assert res[f"ok{r}"] is False, r
        assert "peer mappings failed" in res[f"msg{r}"]
    # ranks that had mapped peers closed them; the failing rank mapped nothing
    assert res[f"closed{fail_rank}"] == 0
    for r in range(3):
        if r != fail_rank:
            assert res[f"closed{r}"] == 4
