"""Split-KV decode across 2 GPUs (config-5 shape) vs the same engine on one GPU.

Two processes, one per GPU, each hold half of every row's KV pages; each
layer exchanges the partial (O, LSE) states and merges them, either through
an NCCL all-gather plus a merge launch or through the peer-memory exchange
kernel (pl_splitkv_exchange_merge over CUDA IPC mappings).  Both exchanges
run in the same processes: their logits must be bit-identical on both ranks.
Rank 0 also runs the single-GPU engine on the same weights and prompts; the
logits of every decode step must agree and both ranks must produce the same
tokens.  Skipped with fewer than two GPUs.
"""

from __future__ import annotations

import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, results) -> None:
    import datetime

    import torch.distributed as dist

    from pagelora_b200.batch_engine import BatchDecodeEngine
    from pagelora_b200.synthetic import LoRASpec, ModelSpec, make_lora_weights, make_model_weights, random_prompt

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=dev)
    engines = []
    try:
        spec = ModelSpec("small-llama3", 2, 512, 8, 2, 64, 1024, 4096, 500000.0, 1e-5)
        lspec = LoRASpec(16, 32.0, ("q", "v"))
        w = make_model_weights(spec, seed=0, dtype=torch.float32, norm_jitter=0.1)
        w = {k: v.bfloat16() for k, v in w.items()}
        lo = make_lora_weights(spec, lspec, dtype=torch.bfloat16)
        prompts = [random_prompt(spec.vocab, n, seed=5 + i) for i, n in enumerate((700, 333, 96))]
        for exchange in ("nccl", "p2p"):
            eng = BatchDecodeEngine(spec, dict(w), adapters=[lo], lora_spec=lspec, row_adapter=[0, 0, 0],
                                    page_size=16, max_context=1024, device=dev, kv_shard=(rank, world),
                                    group=dist.group.WORLD, exchange=exchange)
            engines.append(eng)
            first = eng.prefill(prompts)
            eng.capture()
            toks, logits = [first], []
            for _ in range(5):
                toks.append(eng.step_host(toks[-1]))
                logits.append(eng.logits.float().cpu())
            eng._check_status()
            results[f"toks{rank}_{exchange}"] = toks
            results[f"logits{rank}_{exchange}"] = torch.stack(logits)
        toks = results[f"toks{rank}_nccl"]
        if rank == 0:
            ref = BatchDecodeEngine(spec, dict(w), adapters=[lo], lora_spec=lspec, row_adapter=[0, 0, 0],
                                    page_size=16, max_context=1024, device=dev)
            rtoks, rlogits = [ref.prefill(prompts)], []
            for t in toks[:-1]:
                rtoks.append(ref.step_host(t))
                rlogits.append(ref.logits.float().cpu())
            results["ref_toks"] = rtoks
            results["ref_logits"] = torch.stack(rlogits)
        torch.cuda.synchronize()
    finally:
        for e in engines:
            e.close()  # graphs released, peer mappings closed after a barrier
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_split_kv_two_gpus_matches_single_gpu():
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    with ctx.Manager() as mgr:
        results = mgr.dict()
        port = _free_port()
        procs = [ctx.Process(target=_worker, args=(r, 2, port, results)) for r in range(2)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout=300)
        assert all(p.exitcode == 0 for p in procs)
        res = dict(results)
    for ex in ("nccl", "p2p"):
        assert res[f"toks0_{ex}"] == res[f"toks1_{ex}"]
        assert torch.equal(res[f"logits0_{ex}"], res[f"logits1_{ex}"])  # every shard merges the same partials
    # the peer exchange merges in the same order with the same arithmetic as the all-gather path
    assert torch.equal(res["logits0_p2p"], res["logits0_nccl"])
    assert res["toks0_p2p"] == res["toks0_nccl"]
    err = float((res["logits0_nccl"] - res["ref_logits"]).abs().max())
    print(f"split-KV (2 GPUs) vs single GPU: max |logit err| {err:.3e}")
    assert err < 5e-2, err
    assert res["toks0_nccl"][:3] == res["ref_toks"][:3]
