"""Decode benchmark of the B200 PageLoRA hot path.

Workload: Qwen3-8B architecture (36 layers, hidden 4096, 32/8 heads,
head_dim 128, q/k norm, SwiGLU 12288, vocab 151936), random-init bf16
weights, rank-16 LoRA (alpha 32) on q/k/v/o through the no-merge delta
path, batch 1, 2048-token uniform-random prompt, greedy decode, page size
16, CUDA-graph decode.  A step is one decode token through all 36 layers,
the final norm, lm_head and argmax.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Under torchrun (N > 1) every rank decodes its own independent request
(request sharding: no collective on the data path) and rank 0 reports the
aggregate tok/s = N * K / max-over-ranks time.  ``--impl reference`` times
the CPU restatement of the reference decode path (the oracle port) on the
host cores; its per-step work is a bounded sample (2 full-size layers plus
lm_head at the benchmark's context, scaled to 36 layers).

Timing: W untimed warm-up steps, then K steps bracketed by a barrier and
cuda.synchronize, timed with CUDA events on the stream the kernels run on.
The weights (16 GB) exceed L2 (126 MB), so no flush is needed between steps.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

METRIC = "decode tok/s (Qwen3-8B arch, LoRA r16); attn+LoRA HBM GB/s vs 8 TB/s peak"
WORKLOAD = "config2"


def _peaks() -> tuple[float, str]:
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
        except Exception:
            pass
    return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int) -> None:
        self.gpu = gpu_index
        self.proc = None
        self.lines: list[str] = []
        self._thread = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self._thread = threading.Thread(target=self._read, daemon=True)
            self._thread.start()
        except Exception:
            self.proc = None
        return self

    def _read(self) -> None:
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
            if self._thread is not None:
                self._thread.join(timeout=2)

    def summary(self) -> dict:
        sm, mx, reasons = [], 0.0, set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = max(mx, float(parts[2]))
            except ValueError:
                continue
            for name, val in zip(names, parts[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx or None,
                "reasons": sorted(reasons), "samples": len(sm)}


def _dist():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


# -------------------------------------------------------------- CPU oracle
def cpu_decode_sample(context: int, steps: int, warmup: int) -> dict:
    """Time the oracle port's decode step on a bounded sample: 2 full-size
    Qwen3-8B layers + lm_head at the given context, scaled to 36 layers."""

    import numpy as np
    import torch

    from oracle.decoder import OracleDecoder
    from pagelora_b200.synthetic import WORKLOADS, ModelSpec, make_lora_weights, make_model_weights

    wl = WORKLOADS[WORKLOAD]
    full = wl.model
    sample_layers = 2
    # Tied embeddings: the head matvec has the full [vocab, hidden] cost without a second table.
    spec = ModelSpec(full.name + "-sample", sample_layers, full.hidden, full.num_qo_heads, full.num_kv_heads,
                     full.head_dim, full.intermediate, full.vocab, full.rope_theta, full.rms_eps, full.qk_norm,
                     tie_embeddings=True)
    torch.set_num_threads(os.cpu_count() or 1)
    weights = make_model_weights(spec, seed=0, dtype=torch.float32)
    loras = make_lora_weights(spec, wl.lora, dtype=torch.float32)
    pages = -(-(context + steps + warmup + 2) // wl.page_size)
    dec = OracleDecoder(spec, weights, loras, wl.lora.scale, page_size=wl.page_size, num_pages=pages + 2,
                        bf16=False)
    del weights
    rng = np.random.default_rng(0)
    # Fill the context with random K/V instead of a CPU prefill (decode cost
    # does not depend on where the cached K/V came from).
    n_ctx_pages = -(-context // wl.page_size)
    for _ in range(n_ctx_pages):
        dec.pages.append(dec.free.pop())
    dec.cache[:, dec.pages] = rng.normal(size=dec.cache[:, dec.pages].shape).astype(np.float32)
    dec.last = context - (n_ctx_pages - 1) * wl.page_size
    dec.pos = context
    # Split the step's time into layers and head by timing the head separately.
    head = dec.w.get("lm_head.weight", dec.w["model.embed_tokens.weight"])
    tok = 1
    for _ in range(warmup):
        tok, _ = dec.step(tok)
    t0 = time.perf_counter()
    for _ in range(steps):
        tok, _ = dec.step(tok)
    t_step = (time.perf_counter() - t0) / steps
    x = np.ones((1, spec.hidden), np.float32)
    t0 = time.perf_counter()
    for _ in range(steps):
        x @ head.T
    t_head = (time.perf_counter() - t0) / steps
    per_token = (t_step - t_head) / sample_layers * full.num_layers + t_head
    return {"value": 1.0 / per_token, "unit": "tok/s", "cores": os.cpu_count() or 1, "kind": "port",
            "sample": (f"oracle numpy decode step, {sample_layers} of {full.num_layers} full-size layers + lm_head at "
                       f"context {context}, {steps} steps, scaled to {full.num_layers} layers"),
            "s_per_token": per_token}


def run_reference(args) -> None:
    ws, rank, _ = _dist()
    if rank != 0:
        return
    steps = max(1, args.steps)
    cb = cpu_decode_sample(2048, steps, max(0, args.warmup))
    line = {"metric": METRIC, "impl": "reference", "value": cb["value"], "unit": "tok/s", "n_gpus": args.gpus,
            "steps": steps, "warmup": args.warmup, "ms_per_step": 1000.0 * cb["s_per_token"],
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": WORKLOAD, "model": "Qwen3-8B-arch random init", "global_batch": 1,
                       "context": 2048, "page_size": 16, "lora": "r16 q/k/v/o no-merge"},
            "cpu_baseline": {k: cb[k] for k in ("value", "unit", "cores", "kind", "sample")},
            "e2e": {"value": cb["value"], "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# --------------------------------------------------------------- GPU arm
def kernel_roofline(engine, peak_gbs: float) -> dict:
    """Per-launch CUDA-event timing of every launch of one decode step
    (eager, each launch bracketed by events on the launching stream), grouped
    by kernel; achieved GB/s = algorithmic bytes / measured duration."""

    import torch

    from pagelora_b200 import kernels as K

    s = engine.spec
    stream = torch.cuda.current_stream()
    records: list[tuple[str, float, object, object]] = []

    def timed(name: str, nbytes: float, fn, *a, **kw):
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        fn(*a, **kw)
        e1.record(stream)
        records.append((name, nbytes, e0, e1))

    bf = 2
    r = engine.lora_rank
    ctx_tokens = (len(engine.host_pages) - 1) * engine.page_size + engine.host_last + 1
    kv_bytes = ctx_tokens * s.num_kv_heads * s.head_dim * 2 * bf
    attn_bytes = kv_bytes + 2 * s.q_dim * bf + (engine.indices.numel() * 0)
    orig = (K.linear_lora_fused, K.paged_decode, K.lora_shrink_seg, K.qkv_rope_append)

    def gemv_bytes(x, weight, kw):
        t = x.shape[0]
        n, k = weight.shape
        nb = n * k * bf + t * k * bf * (2 if kw.get("prologue") == 2 else 1) + t * n * bf
        if kw.get("residual") is not None:
            nb += t * n * bf
        if kw.get("lora_b") is not None:
            nb += kw["lora_b"].numel() * bf + t * kw["lora_down"].shape[-1] * 4
        if kw.get("shrink_a") is not None:
            nb += kw["shrink_a"].numel() * bf + t * kw["shrink_a"].shape[0] * 4
        return nb

    def w_gemv(x, weight, **kw):
        timed("linear_lora_fused", gemv_bytes(x, weight, kw), orig[0], x, weight, **kw)

    def w_attn(*a, **kw):
        timed("paged_decode", attn_bytes, orig[1], *a, **kw)

    def w_shrink(x, a_stack, *rest, **kw):
        timed("lora_shrink_seg", a_stack.numel() * bf + x.numel() * bf + x.shape[0] * a_stack.shape[1] * 4,
              orig[2], x, a_stack, *rest, **kw)

    def w_rope(qkv, **kw):
        nb = qkv.numel() * bf + s.q_dim * bf + 2 * s.kv_dim * bf
        if kw.get("lora_b") is not None:
            nb += kw["lora_b"].numel() * bf
        timed("qkv_rope_append", nb, orig[3], qkv, **kw)

    K.linear_lora_fused, K.paged_decode, K.lora_shrink_seg, K.qkv_rope_append = w_gemv, w_attn, w_shrink, w_rope
    try:
        saved = [t.clone() for t in (engine.row_num_pages, engine.last_page_len, engine.row_pages, engine.token_buf)]
        engine.new_page_ids.fill_(engine.free_pages[-1] if engine.free_pages else 0)
        for _ in range(2):  # the second pass is the measured one
            records.clear()
            engine._decode_body()
            for dst, src in zip((engine.row_num_pages, engine.last_page_len, engine.row_pages, engine.token_buf),
                                saved):
                dst.copy_(src)
        torch.cuda.synchronize()
    finally:
        K.linear_lora_fused, K.paged_decode, K.lora_shrink_seg, K.qkv_rope_append = orig
    agg: dict[str, list[float]] = {}
    for name, nb, e0, e1 in records:
        ms = e0.elapsed_time(e1)
        a = agg.setdefault(name, [0, 0.0, 0.0])
        a[0] += 1
        a[1] += nb
        a[2] += ms
    out = {}
    for name, (n, nb, ms) in agg.items():
        gbs = nb / (ms * 1e-3) / 1e9
        out[name] = {"launches": n, "bytes_per_launch": nb / n, "us_per_launch": 1000.0 * ms / n,
                     "achieved_gbs": gbs, "frac_of_peak": gbs / peak_gbs}
    return out


def run_ours(args) -> None:
    import torch
    import torch.distributed as dist

    ws, rank, local = _dist()
    if ws > 1:
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=__import__("datetime").timedelta(seconds=600))
    device = torch.device("cuda", local if ws > 1 else 0)
    torch.cuda.set_device(device)

    from pagelora_b200 import build as plbuild
    from pagelora_b200._capi import load_library
    from pagelora_b200.engine import DecodeEngine
    from pagelora_b200.synthetic import WORKLOADS, make_lora_weights, make_model_weights, random_prompt

    if plbuild.is_stale():
        plbuild.build()
    load_library()
    wl = WORKLOADS[WORKLOAD]
    spec = wl.model
    steps, warmup = args.steps, max(3, args.warmup)
    weights = make_model_weights(spec, seed=0, device=device)
    loras = make_lora_weights(spec, wl.lora, device=device)
    max_len = wl.prompt_len + warmup + 2 * steps + 64
    engine = DecodeEngine(spec, weights, lora=loras, lora_spec=wl.lora, page_size=wl.page_size,
                          max_seq_len=max_len, device=device)
    del weights, loras
    prompt = random_prompt(spec.vocab, wl.prompt_len, seed=rank)
    first = engine.prefill(prompt)
    engine.capture()
    stream = torch.cuda.current_stream(device)

    def barrier():
        if ws > 1:
            dist.barrier()
        torch.cuda.synchronize(device)

    # ---- value: device-resident inputs, graph replay per step
    for _ in range(warmup):
        engine.step_device()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(device.index or 0) as clk:
        e0.record(stream)
        for _ in range(steps):
            engine.step_device()
        e1.record(stream)
        barrier()
    ms = e0.elapsed_time(e1)
    engine._check_status()

    # ---- e2e: through the public step API from pinned host memory
    first = engine.prefill(prompt)
    tok = first
    for _ in range(warmup):
        tok = engine.step_host(tok)
    barrier()
    h0, h1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    h0.record(stream)
    for _ in range(steps):
        tok = engine.step_host(tok)
    h1.record(stream)
    barrier()
    ms_e2e = h0.elapsed_time(h1)
    engine._check_status()

    # ---- per-kernel roofline (eager pass with CUDA events around each launch)
    peak, peak_kind = _peaks()
    kern = kernel_roofline(engine, peak)

    t = torch.tensor([ms, ms_e2e], device=device, dtype=torch.float64)
    if ws > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms, ms_e2e = float(t[0]), float(t[1])
    if rank == 0:
        value = ws * steps / (ms * 1e-3)
        e2e = ws * steps / (ms_e2e * 1e-3)
        dom = kern["linear_lora_fused"]
        cpu = cpu_decode_sample(wl.prompt_len, 3, 1) if ws == 1 else None
        # attention + LoRA bytes of one step over its measured kernel time
        att = kern.get("paged_decode", {})
        line = {
            "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": ws, "steps": steps, "warmup": warmup,
            "ms_per_step": ms / steps, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "bf16", "data": "synthetic",
            "config": {"workload": WORKLOAD, "model": "Qwen3-8B-arch random init", "global_batch": ws,
                       "prompt_len": wl.prompt_len, "page_size": wl.page_size,
                       "lora": "r16 alpha32 q/k/v/o no-merge", "parallelism": f"request-sharded x{ws}",
                       "cuda_graph": True, "l2": "weights 16 GB > L2 126 MB; no flush"},
            "e2e": {"value": e2e, "unit": "tok/s", "h2d_bytes_per_step": 4 + 8, "d2h_bytes_per_step": 8},
            "gpu_launches": engine.launches_per_step() * steps,
            "roofline": {"bound": "hbm", "kernel": "linear_lora_fused", "achieved": dom["achieved_gbs"],
                         "peak": peak, "unit": "GB/s", "frac": dom["achieved_gbs"] / peak, "peak_kind": peak_kind,
                         "traffic": None},
            "kernels": kern,
            "attention_gbs": att.get("achieved_gbs"),
            "clocks": clk.summary(),
        }
        if cpu is not None:
            line["cpu_baseline"] = {k: cpu[k] for k in ("value", "unit", "cores", "kind", "sample")}
        print(json.dumps(line), flush=True)
    if ws > 1:
        dist.destroy_process_group()


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=128)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    args = ap.parse_args()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
