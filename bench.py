"""Benchmark of the snapmind KV-cache hot path on B200.

Headline workload (one "step" = one decode step of the KV path over one batch):
paged GQA decode at the Llama-3-8B KV shape — 32 layers x (append one token per
sequence into the paged pool + paged GQA decode attention over the whole
context), 32 q heads / 8 kv heads, head_dim 128, bf16, block_size 16, 128
sequences per GPU with contexts uniform in [1024, 8192], shuffled block tables.
``value`` = decode tok/s of the whole job (sequences x steps / max-over-ranks
time); the projections and MLP GEMMs of a full model are not part of the path.

Secondary workload in the same line (``kv_append_gather``): the isolated paged
KV append + full gather at the same KV shape, 64 sequences with contexts
uniform in [512, 4096], pool = total blocks + 10%, in HBM GB/s of algorithmic
bytes.

Multi-GPU: one process per GPU (torchrun), each rank owns its own sequences,
pool and block tables — sequence sharding with no data-path collective
(weak scaling; the only collectives are the timing barrier and max).

``--impl reference`` times the reference algorithm on the host CPU instead:
the oracle port (per-token store loop, per-block fetch concatenation,
repeat_interleave + matmul + softmax + matmul) of the same workload over a
bounded sample of sequences, spread over all host cores with a spawn pool.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

METRIC = "decode tok/s/GPU (paged KV, Llama-3-8B shape); KV append/gather HBM GB/s"
L, HQ, H, D, BS = 32, 32, 8, 128, 16
DECODE_BATCH, DECODE_CTX = 128, (1024, 8192)
AG_BATCH, AG_CTX = 64, (512, 4096)
ELEM = 2  # bf16


# ----------------------------------------------------------------------------- helpers
def peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        out = {"hbm_gbs": float(d["hbm_gbs"]), "source": "measured"}
        if "bf16_tflops" in d:
            out["bf16_tflops"] = float(d["bf16_tflops"])
        return out
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


def profile_traffic(kernel: str) -> dict | None:
    """Per-launch DRAM bytes of a kernel from the committed ncu summary, if any."""
    p = ROOT / "profiles" / "traffic.json"
    if not p.exists():
        return None
    return json.loads(p.read_text()).get(kernel)


class ClockSampler:
    """nvidia-smi clock / throttle-reason samples during the timed region.

    One sampler per node: under torchrun local rank 0 samples every local GPU in one
    nvidia-smi process and the other ranks sample nothing, so N processes do not each
    poll the driver while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_indices: list[int]):
        self.gpus = list(gpu_indices)
        self.proc = None
        self.lines: list[str] = []
        self._first = None
        self._thread = None

    def _read(self):
        for ln in self.proc.stdout:
            if ln.strip():
                self.lines.append(ln)
                self._first.set()

    def __enter__(self):
        import threading

        self._first = threading.Event()
        if not self.gpus:
            return self
        try:
            # nvidia-smi counts every GPU of the node: map CUDA's visible indices through
            # CUDA_VISIBLE_DEVICES (indices or UUIDs, both of which --id accepts)
            visible = [v.strip() for v in os.environ.get("CUDA_VISIBLE_DEVICES", "").split(",") if v.strip()]
            ids = [visible[g] if g < len(visible) else str(g) for g in self.gpus]
            self.proc = subprocess.Popen(
                ["nvidia-smi", "--id=" + ",".join(ids), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "50"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return self
        self._thread = threading.Thread(target=self._read, daemon=True)
        self._thread.start()
        self._first.wait(timeout=5.0)  # sampling is live before the timed region starts
        self.lines.clear()
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            if self._thread is not None:
                self._thread.join(timeout=5)

    def summary(self) -> dict | None:
        rows = []
        for ln in getattr(self, "lines", []):
            parts = [x.strip() for x in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                rows.append((float(parts[1]), float(parts[2]), parts[5:9]))
            except ValueError:
                continue
        if not rows:
            return None
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for _, _, r in rows for i, v in enumerate(r) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(r[0] for r in rows), "sm_max_mhz": max(r[1] for r in rows),
                "reasons": reasons, "samples": len(rows)}


def host_memory_budget() -> int:
    """Bytes of host memory this process tree may still use: the smaller of the
    available RAM and what the container's cgroup limit leaves."""
    avail = None
    try:
        import psutil

        avail = psutil.virtual_memory().available
    except ImportError:
        pass
    for limit_f, usage_f in (("/sys/fs/cgroup/memory.max", "/sys/fs/cgroup/memory.current"),
                             ("/sys/fs/cgroup/memory/memory.limit_in_bytes",
                              "/sys/fs/cgroup/memory/memory.usage_in_bytes")):
        try:
            raw = Path(limit_f).read_text().strip()
            if raw == "max":
                continue
            left = int(raw) - int(Path(usage_f).read_text().strip())
            avail = left if avail is None else min(avail, left)
            break
        except (OSError, ValueError):
            continue
    return int(avail if avail is not None else 32 << 30)


def seeded_lengths(seed: int, n: int, lo: int, hi: int) -> np.ndarray:
    return np.random.RandomState(seed).randint(lo, hi + 1, size=n).astype(np.int64)


def shuffled_tables(seed: int, lens: np.ndarray, growth: int, slack: float = 1.1):
    """Block tables over a randomly permuted shared pool of total blocks + slack."""
    need = (lens + growth + BS - 1) // BS
    nb = int(math.ceil(need.sum() * slack))
    perm = np.random.RandomState(seed + 1).permutation(nb).astype(np.int32)
    width = int(need.max())
    tables = np.zeros((len(lens), width), np.int32)
    off = 0
    for b, n in enumerate(lens):
        k = (int(n) + BS - 1) // BS
        tables[b, :k] = perm[off:off + k]
        off += k
    return nb, width, tables, perm[off:]


# ----------------------------------------------------------------------------- GPU arm
def decode_config(world: int) -> dict:
    """The headline workload, as both arms report it."""
    return {
        "workload": f"paged GQA decode step, Llama-3-8B KV shape: {L} layers x (append 1 token/seq + "
                    "paged decode attention); 32 q / 8 kv heads, head_dim 128, bf16, block 16, "
                    "ctx U[1024,8192], shuffled block tables",
        "batch_per_gpu": DECODE_BATCH,
        "global_batch": DECODE_BATCH * world,
        "layers": L,
        "parallelism": f"dp{world} (sequence sharding, no data-path collective)",
        "l2": "inputs larger than L2 (about 2.4 GB of K/V per decode launch)",
    }


def run_b200(args, rank: int, world: int, dist) -> dict | None:
    import torch

    from snapmind_b200 import PagedKVPool

    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", 0)))
    torch.cuda.set_device(dev)
    steps, warmup = args.steps, args.warmup
    seed = 1234 + 7919 * rank
    if args.only == "e2e_llama":
        r = run_e2e_llama(args, dev, seed, dist, world, cpu_baseline=not args.no_cpu_baseline and world == 1)
        return {"metric": METRIC, "value": r["value"], "unit": r["unit"], "n_gpus": world, "steps": steps,
                "warmup": warmup, "ms_per_step": r["ms_per_token"], "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "f32", "data": "synthetic", "config": {"workload": r["workload"]},
                "e2e_llama": r}
    if args.only in ("tiered", "mla"):
        if args.only == "tiered":
            r = run_tiered(args, dev, seed, dist, world)
        else:
            r = run_mla_sparse(args, dev, seed, dist, world, cpu_baseline=not args.no_cpu_baseline and world == 1)
        if "omitted" in r:
            return {"metric": METRIC, "value": None, "unit": "tok/s", "n_gpus": world, "steps": steps,
                    "warmup": warmup, "ms_per_step": None, "higher_is_better": True, "scaling": "weak",
                    "vs_baseline": None, "dtype": "bf16", "data": "synthetic", "config": {"workload": "tiered"},
                    args.only: r}
        return {"metric": METRIC, "value": r["value"], "unit": r["unit"], "n_gpus": world, "steps": steps,
                "warmup": warmup, "ms_per_step": r["ms_per_step"], "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "bf16", "data": "synthetic", "config": {"workload": r["workload"]},
                args.only: r}
    if args.only == "head_shard":
        r = run_head_shard(args, dev, dist, world)
        return {"metric": METRIC, "value": r["value"], "unit": r["unit"], "n_gpus": world, "steps": steps,
                "warmup": warmup, "ms_per_step": r["ms_per_step"], "higher_is_better": True, "scaling": "strong",
                "vs_baseline": None, "dtype": "bf16", "data": "synthetic", "config": {"workload": r["workload"]},
                "roofline": r["roofline"], "head_shard": r}
    if args.only == "append_gather":
        ag = run_append_gather(args, dev, seed, dist, world)
        return {"metric": METRIC, "value": ag["value"], "unit": ag["unit"], "n_gpus": world, "steps": steps,
                "warmup": warmup, "ms_per_step": ag["ms_per_step"], "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "bf16", "data": "synthetic", "config": {"workload": ag["workload"]},
                "roofline": ag["roofline"], "gpu_launches": ag["gpu_launches"], "kv_append_gather": ag}

    # ---------------- decode workload ----------------
    lens = seeded_lengths(seed, DECODE_BATCH, *DECODE_CTX)
    growth = 2 * steps + warmup + 16  # the timed steps, then as many e2e steps
    nb, width, tables, free = shuffled_tables(seed, lens, growth)
    pool = PagedKVPool(L, H, D, nb, max_seqs=DECODE_BATCH, max_blocks_per_seq=width, block_size=BS,
                       dtype=torch.bfloat16, device=dev)
    g = torch.Generator(device=dev).manual_seed(seed)
    pool.k.normal_(generator=g)
    pool.v.normal_(generator=g)
    pool.set_state(tables, lens, free)
    q_all = torch.randn((L, DECODE_BATCH, HQ, D), device=dev, generator=g).to(torch.bfloat16)
    k_all = torch.randn((L, DECODE_BATCH, H, D), device=dev, generator=g).to(torch.bfloat16)
    v_all = torch.randn((L, DECODE_BATCH, H, D), device=dev, generator=g).to(torch.bfloat16)
    out = torch.empty((L, DECODE_BATCH, HQ, D), device=dev, dtype=torch.bfloat16)
    max_len = int(lens.max()) + growth
    split = 0

    def decode_step(events=None):
        pool.reserve(1, batch=DECODE_BATCH)
        for layer in range(L):
            # the layer's new token is stored by the decode launch itself (no append launch)
            if events is not None:
                events[layer][0].record()
            pool.decode(layer, q_all[layer], out=out[layer], max_seq_len=max_len, split_tokens=split,
                        append=(k_all[layer], v_all[layer]))
            if events is not None:
                events[layer][1].record()

    for _ in range(warmup):
        decode_step()
    pool.check()
    launches_per_step = 1 + L
    kv_tokens_before = int(pool.host_lens[:DECODE_BATCH].sum())
    ev = [[(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(L)]
          for _ in range(steps)]
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(dist)
    torch.cuda.synchronize()
    local_rank = int(os.environ.get("LOCAL_RANK", 0))
    local_world = int(os.environ.get("LOCAL_WORLD_SIZE", world))
    with ClockSampler(list(range(local_world)) if local_rank == 0 else []) as clocks:
        t0.record()
        for s in range(steps):
            decode_step(ev[s])
        t1.record()
        torch.cuda.synchronize()
    barrier(dist)
    ms = t0.elapsed_time(t1)
    pool.check()
    ms_max = reduce_max(dist, ms, dev)
    kernel_ms = [e0.elapsed_time(e1) for row in ev for (e0, e1) in row]
    # algorithmic bytes of one decode launch: every cached K and V row once (the new token's
    # included), q in, out back, and the new K and V rows read and stored;
    # step s (1-based) attends over kv_tokens_before + s * batch tokens
    mean_ctx_tokens = kv_tokens_before + DECODE_BATCH * (steps + 1) / 2.0
    bytes_per_launch = (mean_ctx_tokens * H * D * ELEM * 2 + 2 * DECODE_BATCH * HQ * D * ELEM
                        + 2 * 2 * DECODE_BATCH * H * D * ELEM)
    kernel_avg_ms = statistics.fmean(kernel_ms)
    kernel_avg_ms_slowest = reduce_max(dist, kernel_avg_ms, dev)  # every rank takes this collective
    achieved_gbs = bytes_per_launch / (kernel_avg_ms * 1e-3) / 1e9
    pk = peaks()
    traffic = profile_traffic("paged_decode")
    value = DECODE_BATCH * world * steps / (ms_max * 1e-3)

    # ---------------- e2e: host buffers through the public API ----------------
    # Every step copies its q/k/v from pinned host memory and its outputs back, inside the
    # timed region.  Device inputs and outputs are double-buffered: the copy stream moves
    # step s's outputs out and step s+1's inputs in while step s computes.
    q_h = torch.empty_like(q_all, device="cpu").pin_memory()
    k_h = torch.empty_like(k_all, device="cpu").pin_memory()
    v_h = torch.empty_like(v_all, device="cpu").pin_memory()
    q_h.copy_(q_all)
    k_h.copy_(k_all)
    v_h.copy_(v_all)
    o_h = [torch.empty_like(out, device="cpu").pin_memory() for _ in range(2)]
    bufs = [(torch.empty_like(q_all), torch.empty_like(k_all), torch.empty_like(v_all), torch.empty_like(out))
            for _ in range(2)]
    h2d_stream, d2h_stream = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    compute = torch.cuda.current_stream(dev)
    ev_in = [torch.cuda.Event() for _ in range(2)]
    ev_done = [torch.cuda.Event() for _ in range(2)]
    ev_out = [torch.cuda.Event() for _ in range(2)]

    def h2d(i):
        with torch.cuda.stream(h2d_stream):
            h2d_stream.wait_event(ev_done[i])  # the step that last read buffer i has finished
            qd, kd, vd, _ = bufs[i]
            qd.copy_(q_h, non_blocking=True)
            kd.copy_(k_h, non_blocking=True)
            vd.copy_(v_h, non_blocking=True)
            ev_in[i].record(h2d_stream)

    def e2e_step(s_idx):
        i = s_idx & 1
        qd, kd, vd, od = bufs[i]
        h2d(i ^ 1)  # the next step's inputs move while this step computes
        compute.wait_event(ev_in[i])
        compute.wait_event(ev_out[i])  # the outputs of two steps ago are on the host
        pool.reserve(1, batch=DECODE_BATCH)
        for layer in range(L):
            pool.decode(layer, qd[layer], out=od[layer], max_seq_len=max_len, split_tokens=split,
                        append=(kd[layer], vd[layer]))
        ev_done[i].record(compute)
        with torch.cuda.stream(d2h_stream):
            d2h_stream.wait_event(ev_done[i])
            o_h[i].copy_(od, non_blocking=True)
            ev_out[i].record(d2h_stream)

    e2e_steps = steps
    h2d(0)
    e2e_step(0)
    torch.cuda.synchronize()
    barrier(dist)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    tail = torch.cuda.Event()
    e0.record(compute)
    h2d(0)  # the first timed step's inputs are copied inside the timed region too
    for s_idx in range(e2e_steps):
        e2e_step(s_idx)
    tail.record(d2h_stream)
    compute.wait_event(tail)  # the last outputs are on the host
    e1.record(compute)
    torch.cuda.synchronize()
    barrier(dist)
    pool.check()
    e2e_ms = reduce_max(dist, e0.elapsed_time(e1) / e2e_steps, dev)
    h2d_bytes = (q_all.numel() + k_all.numel() + v_all.numel()) * ELEM
    d2h = out.numel() * ELEM
    del pool, q_all, k_all, v_all, out, bufs
    torch.cuda.empty_cache()

    # ---------------- append + gather workload ----------------
    ag = run_append_gather(args, dev, seed, dist, world) if args.only == "all" else None

    line = {
        "metric": METRIC,
        "value": round(value, 2),
        "unit": "tok/s",
        "n_gpus": world,
        "steps": steps,
        "warmup": warmup,
        "ms_per_step": round(ms_max / steps, 4),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (seeded N(0,1) K/V/q, seeded context lengths and shuffled block tables)",
        "config": decode_config(world),
        "roofline": {
            "kernel": "paged_gqa_decode (with the step's K/V append fused in)",
            "bound": "hbm",
            "achieved": round(achieved_gbs, 1),
            "peak": pk["hbm_gbs"],
            "peak_source": pk["source"],
            "unit": "GB/s",
            "frac": round(achieved_gbs / pk["hbm_gbs"], 4),
            "traffic": None if traffic is None else traffic.get("bytes_per_launch_scaled"),
            "algorithmic_bytes_per_launch": int(bytes_per_launch),
            "kernel_ms_avg": round(kernel_avg_ms, 4),
            "kernel_ms_avg_slowest_rank": round(kernel_avg_ms_slowest, 4),
        },
        "e2e": {
            "value": round(DECODE_BATCH * world / (e2e_ms * 1e-3), 2),
            "unit": "tok/s",
            "h2d_bytes_per_step": int(h2d_bytes),
            "d2h_bytes_per_step": int(d2h),
            "copies": "double-buffered on a copy stream, overlapping the previous step's compute",
        },
        "kv_append_gather": ag,
        "tiered": run_tiered(args, dev, seed, dist, world) if args.only == "all" else None,
        "mla_sparse": run_mla_sparse(args, dev, seed, dist, world,
                                     cpu_baseline=not args.no_cpu_baseline and world == 1)
        if args.only == "all" else None,
        "e2e_llama": run_e2e_llama(args, dev, seed, dist, world, cpu_baseline=not args.no_cpu_baseline and world == 1)
        if args.only == "all" else None,
        "gpu_launches": launches_per_step * steps,
        "clocks": clocks.summary(),
    }
    return line


# ----------------------------------------------------------------------------- TinyLlama end to end (config 1)
E2E_PROMPT, E2E_GEN_MAX, E2E_BATCH = 256, 256, 64


def _llama_harness():
    sys.path.insert(0, str(Path(__file__).resolve().parent / "tests"))
    import llama_harness

    return llama_harness


def run_e2e_llama(args, dev, seed, dist, world, cpu_baseline: bool) -> dict:
    """Greedy decode of a TinyLlama-shaped model (22 layers, d_model 2048, 32 q / 4 kv heads,
    head_dim 64, fp32, random N(0, 0.02) weights) whose attention is the ``gqa_paged`` plugin
    over a ``"paged"`` cache: one token per step, batch 1, after a 256-token prompt.  The next
    token stays on the device (argmax), so steps queue without host syncs.  The CPU baseline
    runs the same model with the reference attention math on the host cores."""
    import torch

    from snapmind_b200 import PagedGroupedQueryAttention, PagedKVCache

    lh = _llama_harness()
    sh = lh.TINYLLAMA
    with torch.device(dev):
        model = lh.LlamaHarness(sh, PagedGroupedQueryAttention)
    g = torch.Generator(device=dev).manual_seed(seed + 60)
    with torch.no_grad():
        for _, prm in model.named_parameters():
            if prm.dim() >= 2:
                prm.normal_(0.0, 0.02, generator=g)
            else:
                prm.fill_(1.0)
    model.eval()
    hd = sh.d_model // sh.n_heads
    cache = PagedKVCache(sh.max_seq_len, sh.n_layers, sh.n_kv_heads, hd,
                         max_blocks=sh.n_layers * sh.max_seq_len // 16, device=dev)
    kv = cache.layer_dicts()
    prompt = lh.prompt_ids(sh.vocab_size, E2E_PROMPT, seed + 61).to(dev)
    steps = max(1, min(args.steps, E2E_GEN_MAX))
    warmup = args.warmup
    # eager: one model forward per token, as the reference engine runs it
    with torch.no_grad():
        logits = model(prompt[None], kv_cache=kv)[0, -1]
        tok = logits.argmax(-1).view(1, 1)
        pos = E2E_PROMPT

        def step():
            nonlocal tok, pos
            out = model(tok, kv_cache=kv, position_ids=torch.tensor([pos], device=dev))
            tok = out[0, -1].argmax(-1).view(1, 1)
            pos += 1

        for _ in range(warmup):
            step()
        torch.cuda.synchronize(dev)
        barrier(dist)
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record()
        for _ in range(steps):
            step()
        t1.record()
        torch.cuda.synchronize(dev)
        barrier(dist)
    cache.check_device_errors()
    eager_ms = reduce_max(dist, t0.elapsed_time(t1), dev)
    # the same decode with the step captured in a CUDA graph (GraphDecoder)
    from snapmind_b200.engine import GraphDecoder

    cache.reset()
    eng = GraphDecoder(model, cache)
    eng.prefill(prompt)
    eng.begin(warmup + steps)
    eng.step(warmup)  # warm-up + capture, then replays
    torch.cuda.synchronize(dev)
    barrier(dist)
    g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    g0.record()
    eng.step(steps)
    g1.record()
    torch.cuda.synchronize(dev)
    barrier(dist)
    eng.finish()
    ms = reduce_max(dist, g0.elapsed_time(g1), dev)
    # many sequences decoded together on a PagedKVPool (BatchedGraphDecoder)
    from snapmind_b200 import PagedKVPool
    from snapmind_b200.engine import BatchedGraphDecoder

    nb_seq = (E2E_PROMPT + warmup + steps + 1 + 15) // 16
    pool = PagedKVPool(sh.n_layers, sh.n_kv_heads, hd, num_blocks=E2E_BATCH * nb_seq, max_seqs=E2E_BATCH,
                       max_blocks_per_seq=nb_seq, block_size=16, dtype=torch.float32, device=dev)
    prompts = torch.stack([lh.prompt_ids(sh.vocab_size, E2E_PROMPT, seed + 70 + i) for i in range(E2E_BATCH)])
    bdec = BatchedGraphDecoder(model, pool, E2E_BATCH)
    bdec.prefill(prompts)
    bdec.begin(warmup + steps)
    bdec.step(warmup)
    torch.cuda.synchronize(dev)
    barrier(dist)
    b0, b1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    b0.record()
    bdec.step(steps)
    b1.record()
    torch.cuda.synchronize(dev)
    barrier(dist)
    bdec.finish()
    batched_ms = reduce_max(dist, b0.elapsed_time(b1), dev)
    del pool, bdec
    res = {
        "value": round(world * steps / (ms * 1e-3), 2),
        "unit": "tok/s",
        "workload": f"greedy decode, TinyLlama shape ({sh.n_layers} layers, d_model {sh.d_model}, "
                    f"{sh.n_heads}/{sh.n_kv_heads} heads, head_dim {hd}, fp32), gqa_paged attention over a "
                    f"paged cache (block 16), batch 1 per GPU, {E2E_PROMPT}-token prompt; decode step "
                    f"captured in a CUDA graph (GraphDecoder)",
        "ms_per_token": round(ms / steps, 4),
        "eager_tok_s": round(world * steps / (eager_ms * 1e-3), 2),
        "eager_ms_per_token": round(eager_ms / steps, 4),
        "tokens_timed": steps,
        "gpu_launches_per_token": 3 * sh.n_layers,
        "batched": {
            "value": round(world * E2E_BATCH * steps / (batched_ms * 1e-3), 1),
            "unit": "tok/s",
            "batch_per_gpu": E2E_BATCH,
            "ms_per_step": round(batched_ms / steps, 4),
            "workload": f"{E2E_BATCH} sequences per GPU decoded together on a PagedKVPool (BatchedGraphDecoder: "
                        "device-side block reserve, batched append and paged decode, step in a CUDA graph)",
        },
    }
    del model, cache, kv
    torch.cuda.empty_cache()
    if cpu_baseline:
        res["cpu_baseline"] = _e2e_cpu_baseline(lh, sh)
    return res


def _e2e_cpu_baseline(lh, sh) -> dict:
    """The same model with the reference attention (dict growth + dense GQA) on the host
    cores: prefill of the prompt, then timed greedy decode steps."""
    import torch

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    model = lh.LlamaHarness(sh)
    with torch.no_grad():
        for _, prm in model.named_parameters():
            if prm.dim() >= 2:
                prm.normal_(0.0, 0.02)
            else:
                prm.fill_(1.0)
    model.eval()
    kv = {i: {"k": None, "v": None} for i in range(sh.n_layers)}
    prompt = lh.prompt_ids(sh.vocab_size, E2E_PROMPT, 7)
    n = 3
    with torch.no_grad():
        tok = model(prompt[None], kv_cache=kv)[0, -1].argmax(-1).view(1, 1)
        pos = E2E_PROMPT
        t = time.perf_counter()
        for _ in range(n):
            tok = model(tok, kv_cache=kv, position_ids=torch.tensor([pos]))[0, -1].argmax(-1).view(1, 1)
            pos += 1
        dt = time.perf_counter() - t
    return {"value": round(n / dt, 3), "unit": "tok/s", "cores": threads, "kind": "port",
            "sample": f"{n} greedy decode steps after a {E2E_PROMPT}-token prefill, batch 1, torch on "
                      f"{threads} host threads"}


# ----------------------------------------------------------------------------- tiered (config 4)
TIER_L, TIER_B, TIER_CTX, TIER_POOL, TIER_CHUNK, TIER_SINK, TIER_WINDOW, TIER_REQ = 32, 16, 32768, 1024, 64, 4, 1024, 8


def run_tiered(args, dev, seed, dist, world) -> dict:
    """Tiered KV pool at the Mistral-7B KV shape: 32 layers, 8 kv heads, head_dim 128, bf16;
    sequences of 32768 tokens with all chunks in host-pinned backing; a device pool of
    1024 chunks of 64 tokens (= 4096 blocks of 16 per layer); sink chunk + 1024-token
    window pinned; LRU eviction; 8 seeded-random cold chunks re-fetched per step
    (H2D one step ahead on a copy stream).  Reports decode tok/s with and without the
    re-fetch and the overlap 1 - exposed copy time / copy time."""
    import torch

    from snapmind_b200.tiered_pool import TieredKVPool

    # every chunk lives in host-pinned backing (4.5 GB per 32768-token sequence at this
    # shape).  The batch per rank is held fixed across GPU counts (weak scaling compares
    # like with like): when the ranks of this node cannot all pin it, every rank leaves
    # the line out instead of shrinking it.
    per_seq = TIER_L * 2 * H * D * 2 * (TIER_CTX + 4096)
    local_world = int(os.environ.get("LOCAL_WORLD_SIZE", world))
    B = max(1, args.tiered_batch)
    fits = B * per_seq <= 0.4 * host_memory_budget() / local_world
    if not all_ranks(dist, fits, dev):
        return {"omitted": f"{B} sequences x {per_seq / 1e9:.1f} GB of pinned host backing per rank x "
                           f"{local_world} ranks exceed this host's free memory; the batch per rank is held "
                           "fixed across GPU counts, so the line is left out rather than shrunk",
                "batch_per_gpu": B}
    steps = min(args.steps, 100)
    warmup = args.warmup
    max_tokens = TIER_CTX + 2 * (steps + warmup) + 2 * TIER_CHUNK
    pool = TieredKVPool(TIER_L, H, D, B, max_tokens, TIER_POOL, chunk=TIER_CHUNK, sink=TIER_SINK,
                        window=TIER_WINDOW, n_requests=TIER_REQ, dtype=torch.bfloat16, device=dev)
    # backing: one sequence's worth of seeded data replicated to every sequence
    g = torch.Generator(device=dev).manual_seed(seed + 40)
    n_chunks = TIER_CTX // TIER_CHUNK
    per = pool.backing[0, 0].numel()
    src = torch.randn((n_chunks, per), generator=g, device=dev).to(torch.bfloat16)
    for b in range(B):
        pool.backing[b, :n_chunks].view(n_chunks, per).copy_(src)
    del src
    rng = np.random.RandomState(seed + 41)
    lens = np.full(B, TIER_CTX, np.int64)
    pinned_per_seq = 1 + TIER_WINDOW // TIER_CHUNK
    extra = (TIER_POOL - B * (pinned_per_seq + 1)) // B  # leave room for the first new chunks
    resident = []
    for b in range(B):
        win = list(range(n_chunks - TIER_WINDOW // TIER_CHUNK, n_chunks))
        old = sorted(rng.choice(np.arange(1, n_chunks - len(win)), size=extra, replace=False).tolist())
        resident.append([0] + old + win)
    pool.install(lens, resident)
    q = torch.randn((TIER_L, B, HQ, D), generator=g, device=dev).to(torch.bfloat16)
    kn = torch.randn((TIER_L, B, H, D), generator=g, device=dev).to(torch.bfloat16)
    vn = torch.randn((TIER_L, B, H, D), generator=g, device=dev).to(torch.bfloat16)
    out = torch.empty((TIER_L, B, HQ, D), dtype=torch.bfloat16, device=dev)

    def run(n_steps: int, refetch: bool) -> float:
        recent: list = []
        nxt = pool.pick_requests(rng, TIER_REQ) if refetch else []
        if nxt:
            pool.prefetch(nxt)
        barrier(dist)
        torch.cuda.synchronize(dev)
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record()
        for _ in range(n_steps):
            req = nxt
            recent = (recent + req)[-4 * TIER_REQ:]
            nxt = pool.pick_requests(rng, TIER_REQ, exclude=set(recent)) if refetch else []
            pool.step(q, kn, vn, out, req, nxt)
        t1.record()
        torch.cuda.synchronize(dev)
        barrier(dist)
        return t0.elapsed_time(t1)

    run(warmup, True)
    ms_with = reduce_max(dist, run(steps, True), dev)
    h2d0 = pool.h2d_bytes
    ms_without = reduce_max(dist, run(steps, False), dev)
    pool.check()
    # copy time alone: the same 8-chunk prefetch, nothing else running
    reqs = pool.pick_requests(rng, TIER_REQ)
    torch.cuda.synchronize(dev)
    c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    c0.record(pool.copy_stream)
    for _ in range(10):
        pool.prefetch(reqs)
    c1.record(pool.copy_stream)
    torch.cuda.synchronize(dev)
    copy_ms = c0.elapsed_time(c1) / 10
    chunk_bytes = pool.chunk_host_bytes
    exposed = max(0.0, (ms_with - ms_without) / steps)
    # decode attention reads every resident K/V row of every layer once per step
    resident = float(pool.table_lens.float().sum().item())
    attn_bytes = resident * TIER_L * 2 * H * D * 2
    pk = peaks()
    res = {
        "value": round(B * world * steps / (ms_with * 1e-3), 1),
        "unit": "tok/s",
        "workload": f"tiered pool, Mistral-7B KV shape: {TIER_L} layers, 8 kv / 32 q heads, head_dim 128, bf16; "
                    f"{B} seqs x {TIER_CTX} tokens in host-pinned backing; device pool {TIER_POOL} chunks x "
                    f"{TIER_CHUNK} tokens; sink chunk + {TIER_WINDOW}-token window pinned; LRU; "
                    f"{TIER_REQ} seeded-random cold chunks re-fetched per step",
        "batch_per_gpu": B,
        "ms_per_step": round(ms_with / steps, 4),
        "ms_per_step_without_refetch": round(ms_without / steps, 4),
        "tok_s_without_refetch": round(B * world * steps / (ms_without * 1e-3), 1),
        "h2d_bytes_per_step": int(TIER_REQ * chunk_bytes),
        "h2d_gbs_copy_alone": round(TIER_REQ * chunk_bytes / (copy_ms * 1e-3) / 1e9, 1),
        "copy_ms_per_step_alone": round(copy_ms, 4),
        "overlap": round(1.0 - min(1.0, exposed / copy_ms), 4) if copy_ms > 0 else None,
        "resident_tokens_per_seq": int(pool.table_lens.float().mean().item()),
        "roofline": {
            "kernel": "paged_gqa_decode over resident slots (whole step, without re-fetch)",
            "bound": "hbm",
            "achieved": round(attn_bytes / (ms_without / steps * 1e-3) / 1e9, 1),
            "peak": pk["hbm_gbs"],
            "peak_source": pk["source"],
            "unit": "GB/s",
            "frac": round(attn_bytes / (ms_without / steps * 1e-3) / 1e9 / pk["hbm_gbs"], 4),
            "algorithmic_bytes_per_step": int(attn_bytes),
        },
        "h2d_bytes_measured": int(h2d0),
        "gpu_launches_per_step": 3 + TIER_L,
    }
    del pool
    torch.cuda.empty_cache()
    return res


# ----------------------------------------------------------------------------- MLA + indexer (config 5)
MLA_B, MLA_CTX, MLA_HEADS, MLA_RANK, MLA_ROPE, MLA_CHUNK, MLA_TOPK, MLA_DMODEL = 8, 131072, 128, 512, 64, 64, 32, 7168


def attended_positions(length: int, selected: list[int], chunk: int, sink: int, window: int) -> int:
    """How many positions one query attends: the sink prefix, the recent window and
    the selected chunks, each position once."""
    pos = np.zeros(length, bool)
    pos[: min(sink, length)] = True
    pos[max(0, length - window):] = True
    for c in selected:
        if 0 <= c * chunk < length:
            pos[c * chunk: (c + 1) * chunk] = True
    return int(pos.sum())


def mla_cpu_baseline(seed: int, n_seqs: int = 2, steps: int = 3) -> dict:
    """The step's chunk selection and sparse attention restated on the host (the oracle
    port): sigmoid-gated scores of every chunk key, stable top-32, then the absorbed
    MLA attention over the attended rows, per sequence, in float64 numpy with the
    host's BLAS threads.  A bounded sample: ``n_seqs`` sequences of the workload's
    length, ``steps`` timed steps after one warm-up."""
    import oracle.indexer as oidx
    import oracle.mla as omla

    rng = np.random.default_rng(seed + 60)
    n_chunks = MLA_CTX // MLA_CHUNK
    seqs = []
    for _ in range(n_seqs):
        sq = {
            "keys": rng.standard_normal((n_chunks, 128), dtype=np.float32),
            "q_idx": rng.standard_normal(128, dtype=np.float32),
            "q_lat": (rng.standard_normal((MLA_HEADS, MLA_RANK), dtype=np.float32) * 0.05),
            "q_pe": (rng.standard_normal((MLA_HEADS, MLA_ROPE), dtype=np.float32) * 0.05),
            # full-length caches; only the rows the selection attends are ever read, so
            # only those are filled (the rest stay untouched zero pages)
            "latent": np.zeros((MLA_CTX, MLA_RANK), np.float32),
            "rope": np.zeros((MLA_CTX, MLA_ROPE), np.float32),
        }
        sc = oidx.sigmoid_scores(sq["q_idx"], sq["keys"], 128 ** -0.5, 0.1)
        pos = omla.sparse_positions(MLA_CTX, [int(c) for c in oidx.stable_topk(sc, MLA_TOPK)], MLA_CHUNK, 4, 1024)
        sq["latent"][pos] = rng.standard_normal((len(pos), MLA_RANK), dtype=np.float32)
        sq["rope"][pos] = rng.standard_normal((len(pos), MLA_ROPE), dtype=np.float32)
        seqs.append(sq)
    scale = (128 + 64) ** -0.5

    def step():
        for sq in seqs:
            sc = oidx.sigmoid_scores(sq["q_idx"], sq["keys"], 128 ** -0.5, 0.1)
            top = [int(c) for c in oidx.stable_topk(sc, MLA_TOPK) if c >= 0]
            pos = omla.sparse_positions(MLA_CTX, top, MLA_CHUNK, 4, 1024)
            # gather the attended rows first, then widen (not the whole cache)
            omla.sparse_mla_decode(sq["q_lat"], sq["q_pe"], sq["latent"][pos], sq["rope"][pos],
                                   np.arange(len(pos)), scale)

    step()
    ts = []
    for _ in range(steps):
        t = time.perf_counter()
        step()
        ts.append(time.perf_counter() - t)
    per_step = statistics.median(ts)
    return {"value": round(n_seqs / per_step, 2), "unit": "tok/s (one MLA layer)", "cores": os.cpu_count() or 1,
            "kind": "port",
            "sample": f"{n_seqs} sequences x {MLA_CTX} tokens: sigmoid scores of {n_chunks} chunk keys, stable "
                      f"top-{MLA_TOPK}, absorbed MLA attention over the selected chunks + 4-token sink + "
                      f"1024-token window (float64 numpy, host BLAS threads); median of {steps} steps",
            "step_s": round(per_step, 4)}


def run_mla_sparse(args, dev, seed, dist, world, cpu_baseline: bool = False) -> dict:
    """One MLA layer at DeepSeek shape (128 heads, kv_lora_rank 512, rope 64, bf16), 8 seqs
    of 131072 tokens in the paged latent pool (block = 64-token chunk).  A step: reserve and
    append one latent row per sequence, add the key of a chunk that just completed, score
    all chunks (sigmoid(q.k/sqrt(128)+b) over 128-d projections) with a stable top-32, then
    sparse MLA decode over the selected chunks + 4-token sink + 1024-token window.  Also the
    full latent gather and the all-chunk key pooling in GB/s."""
    import torch

    from snapmind_b200.indexer import ChunkSelector
    from snapmind_b200.mla import MLALatentPool

    B = MLA_B
    # a step is ~0.15 ms: time 1000 of them (after a chunk's worth of warm-up) so that the
    # timed region is long enough for steady clocks
    steps = max(args.steps, 1000)
    warmup = max(args.warmup, MLA_CHUNK)
    ctx_chunks = MLA_CTX // MLA_CHUNK
    width = ctx_chunks + (steps + warmup) // MLA_CHUNK + 2
    nb = B * width
    pool = MLALatentPool(1, nb, B, width, block_size=MLA_CHUNK, kv_lora_rank=MLA_RANK, rope_dim=MLA_ROPE,
                         dtype=torch.bfloat16, device=dev)
    g = torch.Generator(device=dev).manual_seed(seed + 50)
    pool.latent.normal_(generator=g)
    pool.rope.normal_(generator=g)
    perm = np.random.RandomState(seed + 51).permutation(nb).astype(np.int32)
    tables = perm[: B * ctx_chunks].reshape(B, ctx_chunks)
    pool.set_state(tables, np.full(B, MLA_CTX), perm[B * ctx_chunks:])
    sel = ChunkSelector(pool, d_model=MLA_DMODEL, index_dim=128, seed=seed + 52)
    sel.update_keys(0, 0, ctx_chunks, batch=B)
    hidden = torch.randn((B, MLA_DMODEL), generator=g, device=dev).to(torch.bfloat16)
    q_lat = (torch.randn((B, MLA_HEADS, MLA_RANK), generator=g, device=dev) * 0.05).to(torch.bfloat16)
    q_pe = (torch.randn((B, MLA_HEADS, MLA_ROPE), generator=g, device=dev) * 0.05).to(torch.bfloat16)
    lat_new = torch.randn((B, 1, MLA_RANK), generator=g, device=dev).to(torch.bfloat16)
    rope_new = torch.randn((B, 1, MLA_ROPE), generator=g, device=dev).to(torch.bfloat16)
    scale = (128 + 64) ** -0.5
    launches = [0]

    n_chunks_dev = torch.full((B,), ctx_chunks, dtype=torch.int32, device=dev)  # complete chunks

    def core():  # one step that completes no chunk: every launch replayable
        pool.reserve_device(1, B)
        pool.append(0, lat_new, rope_new)
        idx, _ = sel.select(sel.query(hidden), n_chunks_dev, k=MLA_TOPK)
        pool.sparse_decode(0, q_lat, q_pe, idx, sink=4, window=1024, scale=scale)

    graphs: dict[int, torch.cuda.CUDAGraph] = {}

    # kernels per step: reserve, append, indexer query, top-k, sparse attention (+ the split merge when it splits)
    from snapmind_b200 import _lib as slib

    n_spl = slib.load().snapmind_sparse_mla_default_splits(B, MLA_HEADS, MLA_RANK, MLA_ROPE, MLA_CHUNK, 1)
    per_core = 5 + (1 if n_spl > 1 else 0)

    def capture(n_core: int) -> None:  # recorded, not run
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr):
            for _ in range(n_core):
                core()
        graphs[n_core] = gr

    def replay(n_core: int) -> None:  # n_core steps that complete no chunk, as one graph launch
        if not graphs:  # first: one eager step on a side stream (allocates the workspaces)
            side = torch.cuda.Stream(dev)
            side.wait_stream(torch.cuda.current_stream(dev))
            with torch.cuda.stream(side):
                core()
            torch.cuda.current_stream(dev).wait_stream(side)
            pool.account_host(1, B)
            launches[0] += per_core
            for n in (1, 8):
                capture(n)
            n_core -= 1
            if n_core == 0:
                return
            if n_core not in graphs:
                for _ in range(n_core):
                    replay(1)
                return
        graphs[n_core].replay()
        pool.account_host(n_core, B)
        launches[0] += per_core * n_core

    def run_steps(n: int) -> None:
        done = 0
        while done < n:
            length = int(pool.host_lens[0])  # every sequence has the same length here
            if (length + 1) % MLA_CHUNK == 0:  # this step completes a chunk: its key joins the index
                pool.reserve(1, batch=B)
                pool.append(0, lat_new, rope_new)
                sel.update_keys(0, (length + 1) // MLA_CHUNK - 1, 1, batch=B)
                n_chunks_dev.add_(1)
                idx, _ = sel.select(sel.query(hidden), n_chunks_dev, k=MLA_TOPK)
                pool.sparse_decode(0, q_lat, q_pe, idx, sink=4, window=1024, scale=scale)
                launches[0] += per_core + 1
                done += 1
                continue
            free = MLA_CHUNK - 1 - (length + 1) % MLA_CHUNK  # later steps before the completing one
            m = min(n - done, free + 1)
            while m > 0:
                c = 8 if m >= 8 else 1
                replay(c)
                m -= c
                done += c

    run_steps(warmup)
    pool.check()
    launches[0] = 0
    barrier(dist)
    torch.cuda.synchronize(dev)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    run_steps(steps)
    t1.record()
    torch.cuda.synchronize(dev)
    barrier(dist)
    pool.check()
    ms = reduce_max(dist, t0.elapsed_time(t1), dev)
    # kernel-only times: 20 back-to-back launches captured in a graph, replayed once
    qsel = sel.query(hidden)
    idx0, _ = sel.select(qsel, n_chunks_dev, k=MLA_TOPK)

    def graph_us(fn, reps=20):
        fn()
        torch.cuda.synchronize(dev)
        g_ = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g_):
            for _ in range(reps):
                fn()
        g_.replay()
        torch.cuda.synchronize(dev)
        e0_, e1_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0_.record()
        g_.replay()
        e1_.record()
        torch.cuda.synchronize(dev)
        return e0_.elapsed_time(e1_) * 1e3 / reps

    select_us = graph_us(lambda: sel.select(qsel, n_chunks_dev, k=MLA_TOPK))
    query_us = graph_us(lambda: sel.query(hidden))
    sparse_us = graph_us(lambda: pool.sparse_decode(0, q_lat, q_pe, idx0, sink=4, window=1024, scale=scale))
    # the dominant kernel (sparse attention + its split merge), each launch timed alone on the
    # launching stream after an L2 flush: the ~29 MB it reads would otherwise stay in the 126 MB L2.
    # The flush reads 256 MB (a sum): evicting by writing would leave dirty lines whose write-back
    # competes with the timed kernel.  The call is replayed from a CUDA graph, so its two launches
    # are queued while the flush runs and the events bracket device work only (an eager call's
    # host path can outlast the flush and leave the device idle inside the timed window).
    flush = torch.ones(64 << 20, dtype=torch.float32, device=dev)
    g1 = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g1):
        pool.sparse_decode(0, q_lat, q_pe, idx0, sink=4, window=1024, scale=scale)
    g1.replay()
    torch.cuda.synchronize(dev)
    evs = []
    for _ in range(20):
        flush.sum()
        a_, b_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a_.record()
        g1.replay()
        b_.record()
        evs.append((a_, b_))
    torch.cuda.synchronize(dev)
    del flush, g1
    attn_us = statistics.fmean(a_.elapsed_time(b_) for a_, b_ in evs) * 1e3
    # algorithmic work of one launch: every attended row (selected chunks, sink, window) read
    # once at 1152 B and scored + accumulated by 128 heads; q in, latent output out
    length = int(pool.host_lens[0])
    att_tokens = sum(attended_positions(length, idx0[b].tolist(), MLA_CHUNK, 4, 1024) for b in range(B))
    sparse_bytes = att_tokens * (MLA_RANK + MLA_ROPE) * 2 + B * MLA_HEADS * (MLA_RANK + MLA_ROPE + MLA_RANK) * 2
    sparse_flops = att_tokens * MLA_HEADS * 2 * ((MLA_RANK + MLA_ROPE) + MLA_RANK)
    key_bytes = B * (int(pool.host_lens[0]) // MLA_CHUNK) * 128 * 4
    # full latent gather and all-chunk key pooling (HBM-bound)
    length = int(pool.host_lens[0])
    lo = torch.empty((B, length, MLA_RANK), dtype=torch.bfloat16, device=dev)
    ro = torch.empty((B, length, MLA_ROPE), dtype=torch.bfloat16, device=dev)
    pool.gather(0, B, length, out=(lo, ro))  # warm
    sel.update_keys(0, 0, length // MLA_CHUNK, batch=B)  # warm (workspace at this size)
    torch.cuda.synchronize(dev)
    e = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
    e[0].record()
    pool.gather(0, B, length, out=(lo, ro))
    e[1].record()
    sel.update_keys(0, 0, length // MLA_CHUNK, batch=B)
    e[2].record()
    torch.cuda.synchronize(dev)
    gather_ms = e[0].elapsed_time(e[1])
    pool_ms = e[1].elapsed_time(e[2])
    gather_bytes = 2 * B * length * (MLA_RANK + MLA_ROPE) * 2  # read pool + write output
    pool_bytes = B * (length // MLA_CHUNK) * MLA_CHUNK * MLA_RANK * 2
    pk = peaks()
    t_hbm = sparse_bytes / (pk["hbm_gbs"] * 1e9)
    t_tc = sparse_flops / (pk["bf16_tflops"] * 1e12) if pk.get("bf16_tflops") else 0.0
    traffic = profile_traffic("sparse_mla")
    roofline = {
        "kernel": "sparse_mla_umma_kernel + sparse_mla_merge_kernel",
        "bound": "hbm" if t_hbm >= t_tc else "tensor",
        "achieved": round(sparse_bytes / (attn_us * 1e-6) / 1e9, 1) if t_hbm >= t_tc
        else round(sparse_flops / (attn_us * 1e-6) / 1e12, 1),
        "peak": pk["hbm_gbs"] if t_hbm >= t_tc else pk["bf16_tflops"],
        "peak_source": pk["source"],
        "unit": "GB/s" if t_hbm >= t_tc else "TFLOP/s",
        "frac": round(max(t_hbm, t_tc) / (attn_us * 1e-6), 4),
        "hbm_frac": round(t_hbm / (attn_us * 1e-6), 4),
        "tensor_frac": round(t_tc / (attn_us * 1e-6), 4) if t_tc else None,
        "traffic": None if traffic is None else traffic.get("bytes_per_launch_scaled"),
        "algorithmic_bytes_per_launch": int(sparse_bytes),
        "flops_per_launch": int(sparse_flops),
        "attended_tokens_per_launch": int(att_tokens),
        "kernel_us_avg": round(attn_us, 2),
        "timing": "20 calls (one graph replay each: the attention and its merge), each after reading 256 MB to flush L2, CUDA events on the launching stream",
    }
    res = {
        "value": round(B * world * steps / (ms * 1e-3), 1),
        "unit": "tok/s (one MLA layer)",
        "workload": f"MLA latent cache + indexer + sparse attention, one layer: {MLA_HEADS} heads, kv_lora_rank "
                    f"{MLA_RANK}, rope {MLA_ROPE}, bf16, {B} seqs x {MLA_CTX} tokens, chunk {MLA_CHUNK}, "
                    f"top-{MLA_TOPK} + 4-token sink + 1024-token window",
        "ms_per_step": round(ms / steps, 4),
        "latent_gather_gbs": round(gather_bytes / (gather_ms * 1e-3) / 1e9, 1),
        "latent_gather_frac": round(gather_bytes / (gather_ms * 1e-3) / 1e9 / pk["hbm_gbs"], 4),
        "chunk_pool_gbs": round(pool_bytes / (pool_ms * 1e-3) / 1e9, 1),
        "chunk_pool_frac": round(pool_bytes / (pool_ms * 1e-3) / 1e9 / pk["hbm_gbs"], 4),
        "gpu_launches": launches[0],
        "select_us": round(select_us, 2),
        "query_us": round(query_us, 2),
        "select_key_gbs": round(key_bytes / (select_us * 1e-6) / 1e9, 1),
        "sparse_attn_us": round(sparse_us, 2),
        "sparse_attn_gbs": round(sparse_bytes / (sparse_us * 1e-6) / 1e9, 1),
        "sparse_attn_tflops": round(sparse_flops / (sparse_us * 1e-6) / 1e12, 2),
        "sparse_attn_tensor_frac": round(sparse_flops / (sparse_us * 1e-6) / 1e12 / pk["bf16_tflops"], 4)
        if pk.get("bf16_tflops") else None,
        "roofline": roofline,
    }
    if cpu_baseline:
        res["cpu_baseline"] = mla_cpu_baseline(seed)
    del pool, lo, ro
    torch.cuda.empty_cache()
    return res


def run_append_gather(args, dev, seed, dist, world) -> dict:
    import torch

    from snapmind_b200 import PagedKVPool

    steps, warmup = args.steps, args.warmup
    lens = seeded_lengths(seed + 17, AG_BATCH, *AG_CTX)
    nb, width, tables, free = shuffled_tables(seed + 17, lens, steps + warmup + 4)
    pool = PagedKVPool(L, H, D, nb, max_seqs=AG_BATCH, max_blocks_per_seq=width, block_size=BS,
                       dtype=torch.bfloat16, device=dev)
    g = torch.Generator(device=dev).manual_seed(seed + 17)
    pool.k.normal_(generator=g)
    pool.v.normal_(generator=g)
    pool.set_state(tables, lens, free)
    k_new = torch.randn((L, AG_BATCH, H, 1, D), device=dev, generator=g).to(torch.bfloat16)
    v_new = torch.randn((L, AG_BATCH, H, 1, D), device=dev, generator=g).to(torch.bfloat16)
    max_tokens = int(lens.sum()) + AG_BATCH * (steps + warmup + 1)
    k_out = torch.empty((L, max_tokens * H * D), dtype=torch.bfloat16, device=dev)
    v_out = torch.empty_like(k_out)

    # the packed output of each layer is contiguous: a per-step view of the right size
    def step(evs=None):
        pool.reserve(1, batch=AG_BATCH)
        if evs is not None:
            evs[0].record()
        pool.append(None, k_new, v_new)
        if evs is not None:
            evs[1].record()
        per_layer = int(pool.host_lens[:AG_BATCH].sum()) * H * D
        ko = k_out.view(-1)[: L * per_layer].view(L, per_layer)
        vo = v_out.view(-1)[: L * per_layer].view(L, per_layer)
        pool.gather(batch=AG_BATCH, out=(ko, vo))
        if evs is not None:
            evs[2].record()

    for _ in range(warmup):
        step()
    pool.check()
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(steps)]
    tok_before = int(pool.host_lens[:AG_BATCH].sum())
    barrier(dist)
    torch.cuda.synchronize()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    for s in range(steps):
        step(evs[s])
    t1.record()
    torch.cuda.synchronize()
    barrier(dist)
    pool.check()
    ms = reduce_max(dist, t0.elapsed_time(t1), dev)
    tok_after = int(pool.host_lens[:AG_BATCH].sum())
    row = H * D * ELEM  # bytes of one token's K (or V) in one layer
    append_bytes = 2 * 2 * AG_BATCH * L * row  # K and V, read + write
    mean_tokens = (tok_before + AG_BATCH + tok_after) / 2.0
    gather_bytes = 2 * 2 * mean_tokens * L * row
    total_bytes = (append_bytes + gather_bytes) * steps
    append_ms = statistics.fmean(e[0].elapsed_time(e[1]) for e in evs)
    gather_ms = statistics.fmean(e[1].elapsed_time(e[2]) for e in evs)
    # the append kernel alone: an eager call's event pair also spans the host's launch path
    # (the device waits for it), so replay 20 appends of the step's token (each rewrites the
    # same rows with the same bytes) from one CUDA graph and time the replay
    pool.append(None, k_new, v_new)
    torch.cuda.synchronize()
    g_app = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g_app):
        for _ in range(20):
            pool.append(None, k_new, v_new)
    g_app.replay()
    torch.cuda.synchronize()
    a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a0.record()
    g_app.replay()
    a1.record()
    torch.cuda.synchronize()
    append_kernel_ms = a0.elapsed_time(a1) / 20
    del g_app
    pool.check()
    pk = peaks()
    gather_gbs = gather_bytes / (gather_ms * 1e-3) / 1e9
    traffic = profile_traffic("kv_gather")
    res = {
        "value": round(total_bytes * world / (ms * 1e-3) / 1e9, 1),
        "unit": "GB/s",
        "workload": "paged KV append (1 token/seq, all 32 layers, one launch) + full gather of all "
                    "layers, Llama-3-8B KV shape, 64 seqs/GPU, ctx U[512,4096], pool = blocks + 10%",
        "ms_per_step": round(ms / steps, 4),
        "append_ms": round(append_ms, 4),
        "gather_ms": round(gather_ms, 4),
        "append_gbs": round(append_bytes / (append_ms * 1e-3) / 1e9, 1),
        "append_kernel_us": round(append_kernel_ms * 1e3, 2),
        "append_kernel_gbs": round(append_bytes / (append_kernel_ms * 1e-3) / 1e9, 1),
        "append_kernel_frac": round(append_bytes / (append_kernel_ms * 1e-3) / 1e9 / pk["hbm_gbs"], 4),
        "roofline": {
            "kernel": "kv_gather",
            "bound": "hbm",
            "achieved": round(gather_gbs, 1),
            "peak": pk["hbm_gbs"],
            "peak_source": pk["source"],
            "unit": "GB/s",
            "frac": round(gather_gbs / pk["hbm_gbs"], 4),
            "traffic": None if traffic is None else traffic.get("bytes_per_launch_scaled"),
            "algorithmic_bytes_per_launch": int(gather_bytes),
        },
        "gpu_launches": 3 * steps,
    }
    del pool, k_out, v_out
    torch.cuda.empty_cache()
    return res


def run_head_shard(args, dev, dist, world) -> dict:
    """KV-head-sharded decode: every rank serves the same batch with H/N kv heads.

    Timings of one step (all layers) over the same shards: the local decodes
    alone; per layer, the decode + NCCL all-gather of the head slices (+ reorder)
    and the decode whose epilogue stores the rows into every rank's buffer over
    NVLink + the bounded epoch wait; and both with one exchange for the whole
    step (one all-gather of every layer's slices, or one epoch signal and wait
    after the last layer's peer stores).  Whole-job throughput counts each sequence's token once
    (all ranks serve the same sequences)."""
    import torch

    from snapmind_b200 import PagedKVPool
    from snapmind_b200.head_shard import HeadShardedDecode, PeerHeadShardedDecode, head_range, shard_query

    if world < 2 or H % world:
        raise SystemExit("head_shard needs 2, 4 or 8 ranks")
    rank = dist.get_rank()
    seed = 4321  # the same sequences on every rank
    B = args.batch
    lens = seeded_lengths(seed, B, *DECODE_CTX)
    nb, width, tables, free = shuffled_tables(seed, lens, 0)
    lo, hi = head_range(H, world, rank)
    pool = PagedKVPool(L, hi - lo, D, nb, max_seqs=B, max_blocks_per_seq=width, block_size=BS,
                       dtype=torch.bfloat16, device=dev)
    g = torch.Generator(device=dev).manual_seed(seed + rank)
    pool.k.normal_(generator=g)
    pool.v.normal_(generator=g)
    pool.set_state(tables, lens, free)
    q_all = torch.randn((L, B, HQ, D), device=dev, generator=torch.Generator(device=dev).manual_seed(seed))
    q_all = q_all.to(torch.bfloat16)
    out = torch.empty((L, B, HQ, D), device=dev, dtype=torch.bfloat16)
    local = torch.empty((B, HQ // world, D), device=dev, dtype=torch.bfloat16)
    max_len = int(lens.max())
    nccl = HeadShardedDecode(pool, HQ, world, rank)
    fused = PeerHeadShardedDecode(pool, HQ, world, rank, max_batch=B, n_layers=L)
    steps, warmup = args.steps, max(args.warmup, 3)

    def step_local():
        for layer in range(L):
            pool.decode(layer, shard_query(q_all[layer], H, world, rank), out=local, max_seq_len=max_len)

    local_all = torch.empty((L, B, HQ // world, D), device=dev, dtype=torch.bfloat16)

    def step_local_one_launch():  # the baseline of the one-exchange-per-step forms
        pool.decode_layers(q_all[:, :, rank * (HQ // world):(rank + 1) * (HQ // world)], out=local_all,
                           max_seq_len=max_len)

    def step_nccl():
        for layer in range(L):
            nccl.decode(layer, q_all[layer], out=out[layer], max_seq_len=max_len)

    def step_fused():
        for layer in range(L):
            fused.decode(layer, q_all[layer], out=out[layer], max_seq_len=max_len)

    # one exchange per step: the outputs of all layers in one all-gather / one epoch signal
    def step_nccl_per_step():
        nccl.decode_step(q_all, out=out, max_seq_len=max_len)

    def step_fused_per_step():
        fused.decode_step(q_all, max_seq_len=max_len)

    def timed(fn) -> float:
        for _ in range(warmup):
            fn()
        barrier(dist)
        torch.cuda.synchronize()
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record()
        for _ in range(steps):
            fn()
        t1.record()
        torch.cuda.synchronize()
        barrier(dist)
        return reduce_max(dist, t0.elapsed_time(t1) / steps, dev)

    ms_local = timed(step_local)
    ms_local_step = timed(step_local_one_launch)
    ms_nccl = timed(step_nccl)
    ref = out.clone()
    ms_fused = timed(step_fused)
    same_layer = bool(torch.equal(out, ref))  # per-layer forms: the same split plan
    ms_nccl_step = timed(step_nccl_per_step)
    ref_step = out.clone()
    ms_fused_step = timed(step_fused_per_step)
    same_step = bool(torch.equal(fused.decode_step(q_all, max_seq_len=max_len), ref_step))  # one-launch forms
    fused.check()
    pool.check()
    fused.close()
    kv_bytes = float(lens.sum()) * (hi - lo) * D * ELEM * 2 * L  # this rank's K/V rows per step
    pk = peaks()
    res = {
        "workload": f"head-sharded decode, {B} seqs x ctx {DECODE_CTX[0]}-{DECODE_CTX[1]}, {L} layers, "
                    f"Hq {HQ} / H {H} over {world} ranks ({(hi - lo)} kv heads each), D {D}, bf16",
        "value": round(B * 1e3 / ms_fused_step, 1),
        "unit": "tok/s",
        "ms_per_step": round(ms_fused_step, 4),
        "ms_per_step_local_decode_only": round(ms_local, 4),
        "ms_per_step_local_decode_one_launch": round(ms_local_step, 4),
        "ms_per_step_nccl_all_gather": round(ms_nccl, 4),
        "ms_per_step_fused_peer_stores": round(ms_fused, 4),
        "ms_per_step_nccl_one_gather_per_step": round(ms_nccl_step, 4),
        "ms_per_step_fused_one_signal_per_step": round(ms_fused_step, 4),
        "exposed_exchange_us_per_layer": {
            "nccl": round((ms_nccl - ms_local) * 1e3 / L, 2),
            "fused": round((ms_fused - ms_local) * 1e3 / L, 2),
            # against the local decode of every layer in one launch, as these forms run it
            "nccl_one_gather_per_step": round((ms_nccl_step - ms_local_step) * 1e3 / L, 2),
            "fused_one_signal_per_step": round((ms_fused_step - ms_local_step) * 1e3 / L, 2),
        },
        "fused_equals_nccl": {"per_layer": same_layer, "one_exchange_per_step": same_step},
        "exchange_bytes_per_layer_per_rank": B * (HQ // world) * D * ELEM * (world - 1),
        "roofline": {
            "kernel": "paged_gqa_decode (peer stores, every layer in one launch) per rank, whole step",
            "bound": "hbm",
            "achieved": round(kv_bytes / (ms_fused_step * 1e-3) / 1e9, 1),
            "peak": pk["hbm_gbs"],
            "peak_source": pk["source"],
            "unit": "GB/s",
            "frac": round(kv_bytes / (ms_fused_step * 1e-3) / 1e9 / pk["hbm_gbs"], 4),
        },
        "gpu_launches_per_step": {"local": L, "nccl": 3 * L, "fused": 2 * L, "nccl_one_gather_per_step": 3,
                                  "fused_one_signal_per_step": 2},
    }
    del pool
    torch.cuda.empty_cache()
    return res


def barrier(dist):
    if dist is not None:
        dist.barrier()


def all_ranks(dist, flag: bool, dev) -> bool:
    """True when ``flag`` holds on every rank (the same answer on all of them)."""
    if dist is None:
        return bool(flag)
    import torch

    t = torch.tensor([1 if flag else 0], dtype=torch.int32, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MIN)
    return bool(t.item())


def reduce_max(dist, x: float, dev) -> float:
    if dist is None:
        return x
    import torch

    t = torch.tensor([x], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ----------------------------------------------------------------------------- CPU (reference algorithm)
def _cpu_build(seed: int, unit_lens: list[int]):
    """One reference-layout paged cache, with its own pool, per (sequence, layer) unit
    of the sample: ``unit_lens`` holds each unit's context length."""
    import oracle.paged as op

    rng = np.random.RandomState(seed)
    caches = []
    for n in unit_lens:
        c = op.PagedKVCacheOracle(max_seq_len=n + 64, n_layers=1, n_heads=H, head_dim=D, block_size=BS)
        k = rng.standard_normal((1, H, n, D)).astype(np.float32)
        v = rng.standard_normal((1, H, n, D)).astype(np.float32)
        # prefill without the per-token loop (not timed), same slot layout as store()
        nbk = (n + BS - 1) // BS
        blocks = [c.free_blocks.pop() for _ in range(nbk)]
        c.block_tables[0] = blocks
        for j, p in enumerate(blocks):
            t0, t1 = j * BS, min(n, (j + 1) * BS)
            c.k[p, : t1 - t0] = k[0, :, t0:t1].transpose(1, 0, 2)
            c.v[p, : t1 - t0] = v[0, :, t0:t1].transpose(1, 0, 2)
        c.slot_counts[0] = n
        caches.append(c)
    q = rng.standard_normal((1, HQ, 1, D)).astype(np.float32)
    kv = rng.standard_normal((1, H, 1, D)).astype(np.float32)
    return caches, q, kv


def _cpu_decode(caches, q, kv):
    """One decode step of every (sequence, layer) unit: store + fetch + GQA math (reference path)."""
    import oracle.gqa as og

    for c in caches:
        c.store(0, kv, kv, 0)
        k, v = c.fetch(0)
        og.gqa_attention(q, k, v, D ** -0.5, dtype=np.float32)
        c.slot_counts[0] -= 1  # the sample's context stays fixed across steps


def _cpu_worker(conn, seed: int, unit_lens: list[int]):
    caches, q, kv = _cpu_build(seed, unit_lens)
    conn.send("ready")
    while conn.recv() == "step":
        _cpu_decode(caches, q, kv)
        conn.send("done")


def cpu_sample_size(requested: int) -> int:
    """Sequences in the CPU sample: as requested, but at most what fits in a
    quarter of the free host memory (each holds 32 fp32 layer pools, about
    1.2 GB at the mean context)."""
    per_seq = L * (sum(DECODE_CTX) // 2 + 64) * H * D * 4 * 2
    return max(1, min(requested, int(0.25 * host_memory_budget() // per_seq)))


def cpu_reference_timing(n_seqs: int, steps: int, warmup: int, seed: int = 99) -> dict:
    """Time the reference algorithm on ``n_seqs`` sampled sequences, one worker
    process per core (each owning a fixed share of the sample)."""
    import multiprocessing as mp

    cores = os.cpu_count() or 1
    lens = seeded_lengths(seed, n_seqs, *DECODE_CTX).tolist()
    units = [n for n in lens for _ in range(L)]  # (sequence, layer) pairs, each with its own pool
    workers = max(1, min(cores, len(units)))
    ctx = mp.get_context("spawn")
    procs, conns = [], []
    # one BLAS thread per worker process: the workers themselves cover the cores
    thread_vars = ("OMP_NUM_THREADS", "OPENBLAS_NUM_THREADS", "MKL_NUM_THREADS")
    saved = {k: os.environ.get(k) for k in thread_vars}
    os.environ.update({k: "1" for k in thread_vars})
    try:
        for w in range(workers):
            parent, child = ctx.Pipe()
            p = ctx.Process(target=_cpu_worker, args=(child, seed + w, units[w::workers]), daemon=True)
            p.start()
            procs.append(p)
            conns.append(parent)
    finally:
        for k, v in saved.items():
            if v is None:
                os.environ.pop(k, None)
            else:
                os.environ[k] = v
    try:
        for c in conns:
            c.recv()
        times = []
        for i in range(warmup + steps):
            t = time.perf_counter()
            for c in conns:
                c.send("step")
            for c in conns:
                c.recv()
            if i >= warmup:
                times.append(time.perf_counter() - t)
    finally:
        for c in conns:
            try:
                c.send("stop")
            except OSError:
                pass
        for p in procs:
            p.join(timeout=10)
            if p.is_alive():
                p.terminate()
    step_s = statistics.median(times)
    return {"value": round(n_seqs / step_s, 3), "unit": "tok/s", "cores": workers, "kind": "port",
            "sample": f"{n_seqs} sequences (ctx U[1024,8192]) x {L} layers per step, each (sequence, layer) "
                      f"with its own fp32 pool; reference algorithm (per-token store, per-block fetch concat, "
                      f"repeat_interleave/matmul/softmax/matmul) in {workers} worker processes; "
                      f"{warmup} warm-up + median of {steps} steps",
            "step_s": round(step_s, 3)}


def run_reference_arm(args, rank: int, world: int) -> dict | None:
    """The reference's CPU implementation of the headline workload (the oracle port)
    on rank 0's host cores: --warmup untimed and --steps timed steps, each over a
    bounded sample of the decode batch, reported on the B200 arm's config."""
    if rank != 0:
        return None
    n_seqs = cpu_sample_size(args.cpu_sample)
    res = cpu_reference_timing(n_seqs=n_seqs, steps=args.steps, warmup=args.warmup)
    return {
        "impl": "reference",
        "metric": METRIC,
        "value": res["value"],
        "unit": "tok/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(res["step_s"] * 1e3, 2),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic (seeded N(0,1) K/V/q, seeded context lengths)",
        "config": decode_config(world),
        "cpu_baseline": {k: res[k] for k in ("value", "unit", "cores", "kind", "sample")},
        "e2e": {"value": res["value"], "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


# ----------------------------------------------------------------------------- main
def _set_workload(batch: int, ag_batch: int, layers: int) -> None:
    global DECODE_BATCH, AG_BATCH, L
    DECODE_BATCH, AG_BATCH, L = batch, ag_batch, layers


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--cpu-sample", type=int, default=min(128, max(8, os.cpu_count() or 8)))
    ap.add_argument("--no-cpu-baseline", action="store_true")
    # smaller cases of the same kernels (profiling captures); defaults are the benchmark config
    ap.add_argument("--batch", type=int, default=DECODE_BATCH, help="decode sequences per GPU")
    ap.add_argument("--ag-batch", type=int, default=AG_BATCH, help="append/gather sequences per GPU")
    ap.add_argument("--layers", type=int, default=L)
    ap.add_argument("--only", choices=["all", "decode", "append_gather", "tiered", "mla", "e2e_llama", "head_shard"], default="all")
    ap.add_argument("--tiered-batch", type=int, default=TIER_B)
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3) if args.impl == "b200" else args.warmup
    _set_workload(args.batch, args.ag_batch, args.layers)

    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))

    if args.impl == "reference":
        line = run_reference_arm(args, rank, world)
        if line is not None:
            print(json.dumps(line), flush=True)
        return

    # the CPU baseline's spawn pool starts before any CUDA work on this process
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_reference_timing(n_seqs=cpu_sample_size(args.cpu_sample), steps=3, warmup=1)

    dist = None
    if world > 1:
        import datetime

        import torch
        import torch.distributed as tdist

        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", 0)))
        tdist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300))
        dist = tdist
    try:
        line = run_b200(args, rank, world, dist)
    finally:
        if dist is not None:
            dist.destroy_process_group()
    if rank == 0 and line is not None:
        if cpu is not None:
            line["cpu_baseline"] = {k: cpu[k] for k in ("value", "unit", "cores", "kind", "sample")}
        print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
