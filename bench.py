#!/usr/bin/env python
"""Benchmark of the B200 attention stage on BASELINE.json's workloads.

Default (the headline): Qwen2.5-Coder-3B-shaped decode over
all 36 layers -- 16 q heads, 2 KV heads, head_dim 128, 4096 cached f16 tokens
(N(0,1)*0.5), fp32 queries, RoPE theta 1e6 -- appending one token per layer
per step and attending over 4097..4352 tokens across 256 steps.  One step =
one te_attention_decode call over the 36 layers (RoPE + f16 append + split-K
flash decode + LSE combine, one kernel launch).

  metric  decode-attn KV GB/s: algorithmic bytes (KV read + append + q/out) per
          step / device time per step
  e2e     the same through the C ABI with host buffers (pinned q/k/v in, out
          back to host every step)
  prefill BASELINE config 3 (2048-token causal prefill, 36 layers) TFLOP/s

Run under torchrun for N GPUs: each rank decodes its own independent sequence
(sequence sharding, weak scaling; no collective on the data path); the time is
the max over ranks.  `--impl reference` times the reference's own CPU attention
(TinyEngine's c/src/ops.c built into oracle/_ref) on the host cores instead.
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

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

# Config 2 shapes.
LAYERS, HEADS, KV_HEADS, HEAD_DIM = 36, 16, 2, 128
CTX0, DECODE_STEPS, THETA = 4096, 256, 1e6
# Config 3 shapes.
PREFILL_TOKENS = 2048

METRIC = "decode-attn KV GB/s (% of HBM peak) @Qwen-3B ctx4K; prefill attn TFLOPS"


def step_bytes(n_attended: int, layers: int = LAYERS, heads: int = HEADS, kv_heads: int = KV_HEADS,
               head_dim: int = HEAD_DIM, appended: bool = True) -> int:
    """Algorithmic bytes of one decode step of one sequence: per layer, read the
    K and V cache of the tokens cached before the step (f16), read q and the
    new raw k/v (fp32), write the appended f16 k/v row and the fp32 output."""
    cached = n_attended - 1 if appended else n_attended
    kv_read = 2 * cached * kv_heads * head_dim * 2
    qo = 2 * heads * head_dim * 4
    new = (2 * kv_heads * head_dim * 4 + 2 * kv_heads * head_dim * 2) if appended else 0
    return layers * (kv_read + qo + new)


def decode3b_lens(steps: int) -> list[int]:
    """Tokens attended by each of `steps` config-2 decode steps: step i appends
    one token and attends CTX0 + (i mod 256) + 1 (the cache is wound back to
    CTX0 every 256 steps)."""
    return [CTX0 + (i % DECODE_STEPS) + 1 for i in range(steps)]


def decode3b_workload(steps: int) -> str:
    lens = decode3b_lens(steps)
    return (f"decode3b: BASELINE config 2 -- Qwen2.5-Coder-3B decode, 36 layers, H16/Hkv2/hd128, f16 KV, "
            f"RoPE theta 1e6, 1 token appended per layer-step; {steps} steps attending {min(lens)}..{max(lens)} "
            f"tokens (the config's full range 4097..{CTX0 + DECODE_STEPS} is {DECODE_STEPS} steps)")


def prefill_flops(s: int = PREFILL_TOKENS, layers: int = LAYERS) -> int:
    """Causal-exact FLOPs: QK^T and PV over the lower triangle incl. diagonal."""
    return layers * 4 * HEADS * HEAD_DIM * s * (s + 1) // 2


def load_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.is_file():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.rows: list[tuple[float, list[str]]] = []  # (host arrival time, fields)
        self.proc = None
        self.window = None  # (t0, t1) of the timed region, host clock

    def __enter__(self):
        # No idle sleep here: the caller keeps the GPU busy (warm replays)
        # while nvidia-smi starts, then marks the timed window.
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append((time.perf_counter(), [x.strip() for x in line.split(",")]))

    def mark(self, t0: float, t1: float) -> None:
        """The timed region's host-clock span: only samples inside it are summarised."""
        self.window = (t0, t1)

    def __exit__(self, *exc):
        if self.proc:
            time.sleep(0.12)  # the sample that covers the region's last 100 ms
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        rows = [r for t, r in self.rows if len(r) >= 9
                and (self.window is None or self.window[0] <= t <= self.window[1] + 0.1)]
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unavailable"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


# ---------------------------------------------------------------------------
# reference / CPU baseline
# ---------------------------------------------------------------------------

class CpuDecode:
    """The reference CPU attention (te_attention_decode_f32) on decode
    layer-steps (config 2 by default): each call rotates q (te_rope_f32) and
    attends one layer's fp32-widened f16 cache of n tokens; independent layers
    run on `threads` host threads (ctypes releases the GIL during each C call).
    With a position, a call first does the decode step's append as the
    reference's CPU decode does (c/src/qwen.c:1013-1036): te_rope_f32 of the new
    k row at that position, both rows rounded to the cache's f16 and stored at
    that row, then attends tokens 0..position."""

    def __init__(self, kind: str, threads: int, n_layers: int = LAYERS, n: int = CTX0 + 1, heads: int = HEADS,
                 kv_heads: int = KV_HEADS, scale: float = 0.5, shared_kv: bool = False, capacity: int = 0):
        from oracle import oracle as O
        self.lib = O.ref() if kind == "reference" else O.port()
        self.threads = threads
        self.n, self.heads, self.kv_heads = n, heads, kv_heads
        self.n_layers = n_layers
        rows = max(n, capacity)
        rng = np.random.default_rng(0)
        shape = rows * kv_heads * HEAD_DIM
        def cache():
            return (rng.standard_normal(shape, dtype=np.float32) * scale).astype(np.float16).astype(np.float32)
        if shared_kv:  # one K and one V shared by the layer calls (large caches: bounded set-up time)
            k, v = cache(), cache()
            self.ks, self.vs = [k] * n_layers, [v] * n_layers
        else:
            self.ks = [cache() for _ in range(n_layers)]
            self.vs = [cache() for _ in range(n_layers)]
        self.qs = [rng.standard_normal(heads * HEAD_DIM).astype(np.float32) for _ in range(n_layers)]
        self.kn = [(rng.standard_normal(kv_heads * HEAD_DIM) * scale).astype(np.float32) for _ in range(n_layers)]
        self.vn = [(rng.standard_normal(kv_heads * HEAD_DIM) * scale).astype(np.float32) for _ in range(n_layers)]
        from concurrent.futures import ThreadPoolExecutor
        self.pool = ThreadPoolExecutor(max_workers=threads)

    def _one(self, i, pos=None):
        row = self.kv_heads * HEAD_DIM
        if pos is not None:
            k = self.kn[i].copy()
            self.lib.rope_f32(k, self.kv_heads, HEAD_DIM, pos, THETA)
            self.ks[i][pos * row:(pos + 1) * row] = k.astype(np.float16)
            self.vs[i][pos * row:(pos + 1) * row] = self.vn[i].astype(np.float16)
        last = self.n - 1 if pos is None else pos
        q = self.qs[i].copy()
        self.lib.rope_f32(q, self.heads, HEAD_DIM, last, THETA)
        return self.lib.attention_decode_f32(q, self.ks[i], self.vs[i], last, self.heads, self.kv_heads,
                                             HEAD_DIM)

    def step(self, pos=None) -> int:
        """One decode step: every layer once (appending at `pos` when given).
        Returns the number of layer calls."""
        list(self.pool.map(lambda i: self._one(i, pos), range(self.n_layers)))
        return self.n_layers

    def sample(self, budget_s: float):
        """Whole steps until budget_s has passed; returns (GB/s, calls, seconds)."""
        calls = 0
        t0 = time.perf_counter()
        while True:
            calls += self.step()
            if time.perf_counter() - t0 >= budget_s:
                break
        dt = time.perf_counter() - t0
        return step_bytes(self.n, 1, self.heads, self.kv_heads, appended=False) * calls / dt / 1e9, calls, dt

    def close(self):
        self.pool.shutdown()


def run_reference(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from oracle import oracle as O
    kind = "reference" if O.ref_available() else "port"
    threads = O.host_cores()
    # one step of the reference arm = one 36-layer decode step of config 2 on
    # all host threads: per layer, RoPE + f16 append of the new k/v row, then
    # attention over the tokens cached so far -- the same lengths as the GPU arm
    cpu = CpuDecode(kind, threads, capacity=CTX0 + DECODE_STEPS)
    lens = decode3b_lens(args.steps)
    for i in range(max(args.warmup, 0)):
        cpu.step(CTX0 + i % DECODE_STEPS)
    t0 = time.perf_counter()
    calls = 0
    for n in lens:
        calls += cpu.step(n - 1)
    dt = time.perf_counter() - t0
    cpu.close()
    value = sum(step_bytes(n) for n in lens) / dt / 1e9
    # the same layer calls on one host thread, a bounded sample beside the all-thread figure
    c1 = CpuDecode(kind, 1, n_layers=4)
    gbs1, calls1, dt1 = c1.sample(3.0)
    c1.close()
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": "GB/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dt / args.steps * 1e3, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": decode3b_workload(args.steps), "parallelism": "cpu threads"},
        "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": threads, "kind": kind,
                         "sample": f"{args.steps} steps x {LAYERS} layer calls (te_rope_f32 + f16 append + "
                                   f"te_attention_decode_f32 over {min(lens)}..{max(lens)} tokens, the f16 cache "
                                   f"widened to fp32)",
                         "single_thread": {"value": round(gbs1, 3), "unit": "GB/s", "cores": 1,
                                           "sample": f"{calls1} layer calls in {dt1:.1f} s on 1 thread"}},
        "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------

def run_gpu(args) -> None:
    import torch
    import torch.distributed as dist

    from tinymetalagent_b200 import TE_ATTN_ADVANCE, TE_ATTN_HOST_BUFFERS, TE_ATTN_QKV_BIAS, AttnEngine

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))

    hbm_peak, tc_peak, peak_src = load_peaks()
    eng = AttnEngine(local, decode_chunk_tokens=args.chunk)
    stream = torch.cuda.ExternalStream(eng.stream)
    if args.gemv_only or args.qwen_only:
        # one measurement alone (e.g. under a profiler): one JSON line
        if args.gemv_only:
            res = run_gemv(eng, stream, hbm_peak, peak_src, args, world, rank)
        else:
            res = run_qwen(eng, stream, hbm_peak, peak_src, args)
            if not args.no_qwen_prefill:
                res["prompt_prefill"] = run_qwen_prefill(eng, stream, args)
        eng.close()
        if rank == 0:
            print(json.dumps(res))
        if world > 1:
            dist.destroy_process_group()
        return
    if args.only_configs:
        # BASELINE configs 4 and 5 alone (e.g. a scaling sweep): one JSON line
        res = {"ragged7b": run_ragged7b(eng, stream, hbm_peak, peak_src, args, world, rank),
               "long7b": run_long7b(eng, stream, hbm_peak, peak_src, args, world, rank), "n_gpus": world}
        eng.close()
        if rank == 0:
            print(json.dumps(res), flush=True)
        if world > 1:
            dist.destroy_process_group()
        return
    cap = CTX0 + DECODE_STEPS
    cache = eng.kv_cache(layers=LAYERS, max_seqs=1, max_tokens_per_seq=cap, kv_heads=KV_HEADS, head_dim=HEAD_DIM,
                         rope_theta=THETA)
    g = torch.Generator(device="cuda").manual_seed(1234 + rank)
    with torch.cuda.stream(stream):
        for layer in range(LAYERS):
            k = (torch.randn((CTX0, KV_HEADS, HEAD_DIM), generator=g, device="cuda") * 0.5).half()
            v = (torch.randn((CTX0, KV_HEADS, HEAD_DIM), generator=g, device="cuda") * 0.5).half()
            stream.synchronize()
            cache.write_f16(layer, 0, 0, k, v)
        q = torch.randn((LAYERS, 1, HEADS, HEAD_DIM), generator=g, device="cuda")
        kn = torch.randn((LAYERS, 1, KV_HEADS, HEAD_DIM), generator=g, device="cuda") * 0.5
        vn = torch.randn((LAYERS, 1, KV_HEADS, HEAD_DIM), generator=g, device="cuda") * 0.5
        out = torch.empty((LAYERS, 1, HEADS, HEAD_DIM), device="cuda")
    stream.synchronize()

    def barrier():
        if world > 1:
            dist.barrier()

    def step(flags=0, host=None):
        if cache.length(0) >= cap:
            cache.truncate(0, CTX0)
        if host is None:
            cache.decode(0, LAYERS, [0], q, out, HEADS, k_new=kn, v_new=vn, flags=TE_ATTN_ADVANCE | flags)
        else:
            hq, hk, hv, ho = host
            cache.decode(0, LAYERS, [0], hq, ho, HEADS, k_new=hk, v_new=hv,
                         flags=TE_ATTN_ADVANCE | TE_ATTN_HOST_BUFFERS)

    # ---- device-timed decode -------------------------------------------
    # The K steps are captured once into a CUDA graph (each step is one decode
    # launch with that step's lengths baked in) and replayed, so the timing is
    # of the device work, not of Python-side launch overhead.
    for _ in range(max(args.warmup, 3)):
        step()
    eng.synchronize()
    cache.truncate(0, CTX0)
    cache.reserve(0, cap)
    # step i attends CTX0 + (i mod 256) + 1 tokens (the cache wraps back to CTX0 every 256 steps)
    lens = decode3b_lens(args.steps)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

    def time_region(fn):
        """One timed region: barrier + synchronize, events around fn() on the engine's stream."""
        barrier()
        torch.cuda.synchronize()
        ev0.record(stream)
        fn()
        ev1.record(stream)
        ev1.synchronize()
        return ev0.elapsed_time(ev1)

    def eager_k():
        cache.truncate(0, CTX0)
        for _ in range(args.steps):
            step()

    def regions_for(ms_est):
        """Timed regions (each exactly K steps) to cover args.min_timed_ms; the
        same count on every rank, since each region starts with a barrier."""
        r = max(5, int(np.ceil(args.min_timed_ms / max(ms_est, 1e-3))))
        r = min(r, 100000)
        if world > 1:
            t = torch.tensor([float(r)], device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            r = int(t.item())
        return r

    graph = None
    if not args.no_graph:
        cache.truncate(0, CTX0)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            for _ in range(args.steps):
                step()
        with torch.cuda.stream(stream):
            graph.replay()  # warm
        stream.synchronize()

    def run_k():
        if graph is not None:
            with torch.cuda.stream(stream):
                graph.replay()
        else:
            eager_k()

    # the same decode with the fused projection-bias prologue (TE_ATTN_QKV_BIAS:
    # the layer's q/k/v biases added inside the decode launch before RoPE and
    # the f16 append), captured now and timed in the same sustained window
    graph_b = None
    if not args.no_graph:
        gb = torch.Generator(device="cuda").manual_seed(4321 + rank)
        cache.set_qkv_bias(0, HEADS, torch.randn((LAYERS, HEADS * HEAD_DIM), generator=gb, device="cuda") * 0.1,
                           torch.randn((LAYERS, KV_HEADS * HEAD_DIM), generator=gb, device="cuda") * 0.1,
                           torch.randn((LAYERS, KV_HEADS * HEAD_DIM), generator=gb, device="cuda") * 0.1)
        cache.truncate(0, CTX0)
        graph_b = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph_b, stream=stream):
            for _ in range(args.steps):
                step(flags=TE_ATTN_QKV_BIAS)
        cache.truncate(0, CTX0)

    def replay_b():
        with torch.cuda.stream(stream):
            graph_b.replay()

    # Timed: R regions, each exactly K steps (one replay of the K-step graph)
    # bracketed by a barrier and a synchronize on both sides and timed alone
    # with CUDA events; the reported time is the median region (max over
    # ranks).  The clock sampler starts first and the GPU stays busy with warm
    # replays while nvidia-smi comes up, so the timed regions see loaded clocks.
    with ClockSampler(local) as clocks:
        t_end = time.perf_counter() + 0.4
        while time.perf_counter() < t_end:
            run_k()
            stream.synchronize()
        n_regions = regions_for(time_region(run_k))
        t_start = time.perf_counter()
        times = [time_region(run_k) for _ in range(n_regions)]
        clocks.mark(t_start, time.perf_counter())
        # eager launches (host loop) and the bias variant in the same sustained window, for comparison
        eager_ms = float(np.median([time_region(eager_k) for _ in range(max(5, n_regions // 4))]))
        ms_b = float(np.median([time_region(replay_b) for _ in range(max(5, n_regions // 4))])) \
            if graph_b is not None else None
    launches = args.steps  # one decode launch per step in each timed region
    eng.synchronize()
    ms = float(np.median(times))
    spread = (float(np.percentile(times, 90)) - float(np.percentile(times, 10))) / ms
    if graph is not None:
        del graph
    cache.truncate(0, CTX0)
    ms_max = ms
    if world > 1:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_max = float(t.item())
    bytes_rank = sum(step_bytes(n) for n in lens)
    value = bytes_rank * world / (ms_max / 1e3) / 1e9
    kernel_gbs = bytes_rank / (ms / 1e3) / 1e9
    qkv_bias = None
    if graph_b is not None:
        del graph_b
        cache.truncate(0, CTX0)
        if world > 1:
            t = torch.tensor([ms_b], device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms_b = float(t.item())
        value_b = bytes_rank * world / (ms_b / 1e3) / 1e9
        qkv_bias = {"metric": "config 2 decode with the fused QKV-bias prologue (TE_ATTN_QKV_BIAS)",
                    "value": round(value_b, 3), "unit": "GB/s", "ms_per_step": round(ms_b / args.steps, 5),
                    "relative_to_plain": round(value_b / value, 4),
                    "timing": "median of timed regions in the headline's sustained window"}

    # ---- e2e through the C ABI with host buffers -------------------------
    hq = torch.empty(q.shape, dtype=torch.float32, pin_memory=True).copy_(q)
    hk = torch.empty(kn.shape, dtype=torch.float32, pin_memory=True).copy_(kn)
    hv = torch.empty(vn.shape, dtype=torch.float32, pin_memory=True).copy_(vn)
    ho = torch.empty(out.shape, dtype=torch.float32, pin_memory=True)
    host = (hq, hk, hv, ho)
    cache.truncate(0, CTX0)
    for _ in range(max(args.warmup, 3)):
        step(host=host)
    cache.truncate(0, CTX0)
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    t_wall = time.perf_counter()
    for _ in range(args.steps):
        step(host=host)
    e1.record(stream)
    e1.synchronize()
    wall_ms = (time.perf_counter() - t_wall) * 1e3
    e2e_ms = max(e0.elapsed_time(e1), wall_ms)
    if world > 1:
        t = torch.tensor([e2e_ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())
    e2e_value = bytes_rank * world / (e2e_ms / 1e3) / 1e9
    h2d = (hq.numel() + hk.numel() + hv.numel()) * 4
    d2h = ho.numel() * 4

    # ---- CPU baseline (rank 0, N=1 only) ---------------------------------
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        from oracle import oracle as O
        kind = "reference" if O.ref_available() else "port"
        threads = O.host_cores()
        cd = CpuDecode(kind, threads)
        gbs, calls, dt = cd.sample(args.cpu_seconds * 2 / 3)
        cd.close()
        # the same layer calls on one host thread (the reference's function is single-threaded)
        c1 = CpuDecode(kind, 1, n_layers=4)
        gbs1, calls1, dt1 = c1.sample(args.cpu_seconds / 3)
        c1.close()
        cpu = {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": kind,
               "sample": f"{calls} config-2 layer calls (N={CTX0 + 1}, 16 heads) in {dt:.1f} s on {threads} threads",
               "single_thread": {"value": round(gbs1, 3), "unit": "GB/s", "cores": 1,
                                 "sample": f"{calls1} config-2 layer calls in {dt1:.1f} s on 1 thread"}}

    # ---- prefill: 2048-token causal prefill over 36 layers ----
    prefill = None
    if not args.no_prefill:
        prefill = run_prefill(eng, stream, tc_peak, peak_src, args, world, rank, local)

    # ---- quantized matrix-vector products (the projections' building block) ----
    gemv = None
    if not args.no_gemv:
        gemv = run_gemv(eng, stream, hbm_peak, peak_src, args, world, rank)

    # ---- the qwen2 decode step (projections + attention + glue), one GPU ----
    qwen = qwen_prefill = None
    if not args.no_qwen and world == 1:
        qwen = run_qwen(eng, stream, hbm_peak, peak_src, args)
        qwen_prefill = run_qwen_prefill(eng, stream, args)

    # ---- BASELINE configs 4 (sequence-sharded batch) and 5 (KV split + NCCL merge) ----
    ragged = long = None
    if not args.no_configs:
        cache.close()
        cache = None
        ragged = run_ragged7b(eng, stream, hbm_peak, peak_src, args, world, rank)
        long = run_long7b(eng, stream, hbm_peak, peak_src, args, world, rank)

    # DRAM traffic of one decode launch, as measured by ncu on this kernel
    # version (config 2 at ctx 4097) and stored in the profiles folder; not a
    # measurement of this run.
    traffic = traffic_src = None
    tfile = ROOT / "profiles" / "traffic.json"
    if tfile.is_file():
        td = json.loads(tfile.read_text())
        traffic = td.get("decode_f16_kernel_decode3b_bytes_per_launch")
        traffic_src = td.get("source")

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 3), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_max / args.steps, 5), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f16 KV, fp32 q/accumulate", "data": "synthetic",
            "config": {"workload": decode3b_workload(args.steps),
                       "parallelism": f"sequence-sharded x{world}" if world > 1 else "single GPU",
                       "l2": "per-step KV (151 MB) exceeds the 126 MB L2",
                       "kernel": "decode_f16_kernel<128,8>: stream-K or cluster split; fused RoPE-append + "
                                 "flash decode (fp32 q as f16 hi + lo) + LSE combine",
                       "timing": (f"median of {n_regions} timed regions, each one replay of the {args.steps}-step "
                                  f"CUDA graph ({sum(times):.0f} ms in all)") if not args.no_graph
                                 else f"median of {n_regions} timed regions of {args.steps} eager steps",
                       "region_spread_p10_p90": round(spread, 4),
                       "eager_ms_per_step": round(eager_ms / args.steps, 5)},
            "roofline": {"bound": "hbm", "achieved": round(kernel_gbs, 1), "peak": hbm_peak, "unit": "GB/s",
                         "frac": round(kernel_gbs / hbm_peak, 4), "traffic": traffic, "traffic_source": traffic_src,
                         "peak_source": f"{peak_src} (burst copy)"},
            "e2e": {"value": round(e2e_value, 3), "unit": "GB/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h},
            "gpu_launches": int(launches),
            "clocks": clocks.summary(),
            "cpu_baseline": cpu,
            "prefill": prefill,
            "decode3b_qkv_bias": qkv_bias,
            "gemv_gguf": gemv,
            "qwen_decode_step": qwen,
            "qwen_prompt_prefill": qwen_prefill,
            "ragged7b": ragged,
            "long7b": long,
        }
        print(json.dumps(line), flush=True)
    if cache is not None:
        cache.close()
    eng.close()
    if world > 1:
        dist.destroy_process_group()


def _measure_prefill(eng, stream, args, world, rank, layers, heads, kv_heads, hd, s, extra_flags=0):
    """One te_attention_prefill call per step over `layers` layers of an
    s-token prompt (f16 Q/K/V N(0,1), RoPE theta 1e6): device time per call
    (CUDA events over the steps, max over ranks), the tcgen05 kernel's own time
    (events the library records around it), and launches per call."""
    import torch
    import torch.distributed as dist

    from tinymetalagent_b200 import TE_ATTN_ADVANCE, TE_ATTN_INPUT_F16
    cache = eng.kv_cache(layers=layers, max_seqs=1, max_tokens_per_seq=s, kv_heads=kv_heads, head_dim=hd,
                         rope_theta=THETA)
    g = torch.Generator(device="cuda").manual_seed(99 + rank)
    with torch.cuda.stream(stream):
        q = torch.randn((layers, s, heads, hd), generator=g, device="cuda").half()
        k = torch.randn((layers, s, kv_heads, hd), generator=g, device="cuda").half()
        v = torch.randn((layers, s, kv_heads, hd), generator=g, device="cuda").half()
        out = torch.empty((layers, s, heads, hd), device="cuda")
    stream.synchronize()

    def step():
        cache.truncate(0, 0)
        cache.prefill(0, layers, 0, q, k, v, s, heads, out, TE_ATTN_ADVANCE | TE_ATTN_INPUT_F16 | extra_flags)

    for _ in range(3):
        step()
    eng.synchronize()
    steps = max(3, min(args.prefill_steps, 50))
    launches0 = eng.launch_count
    ms = _time_steps(stream, step, steps, world, dist) / steps
    eng.synchronize()
    launches = int(eng.launch_count - launches0)
    # the tensor-core kernel alone: CUDA events the library records around it
    # on its stream (same calls, timed separately from the loop above)
    eng.time_kernels(True)
    kms = []
    for _ in range(steps):
        step()
        kms.append(eng.last_kernel_ms())
    eng.time_kernels(False)
    kernel_ms = float(np.mean(kms))
    if world > 1:
        t = torch.tensor([kernel_ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        kernel_ms = float(t.item())
    cache.close()
    del q, k, v, out
    return ms, kernel_ms, launches // steps, steps


def run_prefill(eng, stream, tc_peak, peak_src, args, world, rank, local):
    """Config 3: f16 Q/K/V for 2048 tokens x 36 layers; one te_attention_prefill call
    (RoPE + f16 append, query prep, tcgen05 flash prefill) per step, device-timed.
    Beside it: the same call with TE_ATTN_EXACT_Q (the rotated query as f16 hi + lo
    parts, one head per item), and head_dim 64 at the Qwen2.5-0.5B shape."""
    from tinymetalagent_b200 import TE_ATTN_EXACT_Q
    s = PREFILL_TOKENS
    ms, kernel_ms, launches, steps = _measure_prefill(eng, stream, args, world, rank, LAYERS, HEADS, KV_HEADS,
                                                      HEAD_DIM, s)
    flops = prefill_flops(s, LAYERS)
    tflops = flops / (ms / 1e3) / 1e12
    kernel_tflops = flops / (kernel_ms / 1e3) / 1e12
    res = {"metric": "causal prefill attention TFLOP/s (BASELINE config 3)", "value": round(tflops * world, 2),
           "unit": "TFLOP/s", "ms_per_step": round(ms, 4), "steps": steps,
           "workload": "S=2048, H16/Hkv2/hd128, 36 layers, f16 Q/K/V; one te_attention_prefill call per step "
                       "(RoPE + K/V append + query preparation pass, then the tcgen05 attention kernel)",
           "flops_per_step": flops, "gpu_launches": launches * steps,
           "kernel_ms_per_step": round(kernel_ms, 4),
           "roofline": {"bound": "tensor", "achieved": round(kernel_tflops, 1), "peak": tc_peak, "unit": "TFLOP/s",
                        "frac": round(kernel_tflops / tc_peak, 4), "kernel": "prefill_tc_kernel<128> (CUDA events)",
                        "whole_call_frac": round(tflops / tc_peak, 4),
                        "peak_source": f"{peak_src} (bf16 dense burst)"}}
    if not args.no_prefill_variants:
        ms_x, kms_x, _, _ = _measure_prefill(eng, stream, args, world, rank, LAYERS, HEADS, KV_HEADS, HEAD_DIM, s,
                                             TE_ATTN_EXACT_Q)
        res["exact_q"] = {"metric": "config 3 with TE_ATTN_EXACT_Q (rotated query as f16 hi + lo, one head per item)",
                          "value": round(flops / (ms_x / 1e3) / 1e12 * world, 2), "unit": "TFLOP/s",
                          "ms_per_step": round(ms_x, 4), "kernel_ms_per_step": round(kms_x, 4),
                          "kernel_frac": round(flops / (kms_x / 1e3) / 1e12 / tc_peak, 4),
                          "relative_to_single_rounding": round(ms / ms_x, 4)}
        L5, H5, K5, D5 = 24, 14, 2, 64  # Qwen2.5-0.5B attention shape
        f5 = L5 * 4 * H5 * D5 * s * (s + 1) // 2
        ms_5, kms_5, _, _ = _measure_prefill(eng, stream, args, world, rank, L5, H5, K5, D5, s)
        res["hd64"] = {"metric": "causal prefill TFLOP/s, head_dim 64 (Qwen2.5-0.5B shape)",
                       "workload": "S=2048, H14/Hkv2/hd64, 24 layers, f16 Q/K/V N(0,1), RoPE theta 1e6",
                       "value": round(f5 / (ms_5 / 1e3) / 1e12 * world, 2), "unit": "TFLOP/s",
                       "flops_per_step": f5, "ms_per_step": round(ms_5, 4), "kernel_ms_per_step": round(kms_5, 4),
                       "roofline": {"bound": "tensor", "achieved": round(f5 / (kms_5 / 1e3) / 1e12, 1),
                                    "peak": tc_peak, "unit": "TFLOP/s",
                                    "frac": round(f5 / (kms_5 / 1e3) / 1e12 / tc_peak, 4),
                                    "kernel": "prefill_tc_kernel<64> (CUDA events)"}}
    return res


# Config 4 / 5 shapes (Qwen2.5-7B: 28 layers, 28 query heads, 4 KV heads).
L7, H7, KV7 = 28, 28, 4


def _time_steps(stream, fn, steps, world, dist):
    """Device time of `steps` calls of fn() on `stream` (barrier + sync both
    sides), max over ranks, in ms."""
    import torch
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        fn()
    e1.record(stream)
    e1.synchronize()
    ms = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    return ms


def run_gemv(eng, stream, hbm_peak, peak_src, args, world, rank):
    """te_matvec_gguf on a 32768 x 8192 GGUF matrix (Q4_0 151 MB, Q8_0 285 MB -- both beyond the
    126 MB L2, so every call streams the weights from HBM), one fp32 input vector; weight bytes
    per second against the measured copy peak."""
    import torch
    import torch.distributed as dist
    rows, cols = 32768, 8192
    res = {"metric": "GGUF matrix-vector weight bandwidth (te_matvec_gguf)", "unit": "GB/s",
           "shape": f"{rows}x{cols}, 1 vector", "peak": hbm_peak, "peak_source": f"{peak_src} (burst copy)"}
    g = torch.Generator(device="cuda").manual_seed(77 + rank)
    x = torch.randn((1, cols), generator=g, device="cuda")
    y = torch.empty((1, rows), device="cuda")
    for name, quant, width in (("q4_0", 4, 18), ("q8_0", 8, 34)):
        with torch.cuda.stream(stream):
            w = torch.randint(0, 256, (rows, cols // 32, width), generator=g, device="cuda", dtype=torch.uint8)
            w[:, :, 0:2] = (torch.randn((rows, cols // 32), generator=g, device="cuda") * 0.02).half() \
                .view(torch.uint8).view(rows, cols // 32, 2)
        stream.synchronize()
        calls = 20

        def run():
            for _ in range(calls):
                eng.matvec_gguf(quant, w, rows, cols, x, y, 1)

        for _ in range(3):
            eng.matvec_gguf(quant, w, rows, cols, x, y, 1)
        ms = _time_steps(stream, run, 1, world, dist)
        nbytes = w.numel() + x.numel() * 4 + y.numel() * 4
        gbs = nbytes * calls / (ms / 1e3) / 1e9
        res[name] = {"value": round(gbs * world, 1), "per_gpu_gbs": round(gbs, 1), "us_per_call": round(ms * 1e3 / calls, 2),
                     "weight_bytes": int(w.numel()), "frac": round(gbs / hbm_peak, 4)}
        del w
    if rank == 0 and world == 1 and not args.no_cpu:
        from oracle import oracle as O
        if O.ref_available():
            import numpy as np
            sys.path.insert(0, str(ROOT / "tests" / "golden"))
            from make_golden import quant_matrix
            r_cpu = 8192
            wq = quant_matrix(np.random.default_rng(5), 2, r_cpu, cols)
            xc = np.random.default_rng(6).standard_normal(cols).astype(np.float32)
            ref = O.ref()
            ref.model_matvec_f32(2, wq, r_cpu, cols, xc)
            t0 = time.perf_counter()
            n = 0
            while time.perf_counter() - t0 < 2.0:
                ref.model_matvec_f32(2, wq, r_cpu, cols, xc)
                n += 1
            dt = time.perf_counter() - t0
            res["cpu_baseline"] = {"value": round(wq.size * n / dt / 1e9, 3), "unit": "GB/s", "kind": "reference",
                                   "cores": O.host_cores(),
                                   "sample": f"{n} calls of te_model_matvec_f32 (Q4_0 {r_cpu}x{cols}, its pthread "
                                             f"row split) in {dt:.1f} s"}
    return res


QWEN_SHAPE = dict(layers=24, hidden=896, heads=14, kv_heads=2, ffn=4864, vocab=151936, context=1024)


def _qwen_decode_times(eng, stream, dec, toks, steps):
    """Eager steps (forward_token + project_next, argmax read back each step) and the same window recorded
    as one CUDA graph (capture_greedy) and replayed: (eager ms, graph ms as the median of 5 replays,
    library launches per eager step)."""
    import torch
    prompt = len(toks)
    for pos, t in enumerate(toks):
        dec.forward_token(t, pos)
    nxt = dec.project_next()
    for _ in range(3):  # warm-up steps, then restart from the same position
        dec.forward_token(nxt, prompt)
        dec.project_next()
    launches0 = eng.launch_count
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record(stream)
    t0 = time.perf_counter()
    pos = prompt
    first = nxt
    for _ in range(steps):
        dec.forward_token(nxt, pos)
        nxt = dec.project_next()
        pos += 1
    e1.record(stream)
    e1.synchronize()
    wall_ms = (time.perf_counter() - t0) * 1e3
    ms = max(e0.elapsed_time(e1), wall_ms)
    launches = eng.launch_count - launches0
    dec.cache.truncate(0, prompt)
    dec.capture_greedy(prompt, steps)
    dec.replay_greedy(first)  # warm
    torch.cuda.synchronize()
    reps = []
    for _ in range(5):
        e0.record(stream)
        dec.replay_greedy(first)
        e1.record(stream)
        e1.synchronize()
        reps.append(e0.elapsed_time(e1))
    return ms, float(np.median(reps)), launches / steps


def run_qwen(eng, stream, hbm_peak, peak_src, args):
    """QwenDecoder (the te_qwen_forward_token-compatible decode step) on a synthetic model of
    Qwen2.5-0.5B's shape -- 24 layers, hidden 896, 14 heads of 64 over 2 KV heads, FFN 4864, vocabulary
    151 936; Q4_0 projections, Q8_0 embedding and lm_head -- written as a GGUF file at run time (no
    model file is available offline).  A step is one greedy token after a 16-token prompt: the value is
    the whole-token step kernel (one launch per token: every layer, the head and the argmax) recorded
    as one CUDA graph and replayed; beside it the same window on the per-op path (five launches per
    layer), and eager steps of both.  Device time on the engine's stream.  Beside them, the
    reference's own CPU forward pass on the same file."""
    import tempfile
    import shutil
    sys.path.insert(0, str(ROOT / "tests" / "golden"))
    from gguf_synth import GGML_Q4_0, write_qwen2
    from tinymetalagent_b200.qwen import QwenDecoder

    tmp = Path(tempfile.mkdtemp(prefix="qwen_bench_"))
    try:
        path = tmp / "qwen2_0p5b_shape.gguf"
        write_qwen2(path, quant_attn=GGML_Q4_0, quant_ffn=GGML_Q4_0, seed=3, **QWEN_SHAPE)
        prompt, steps = 16, args.qwen_steps
        ctx = prompt + steps + 8
        rng = np.random.default_rng(9)
        toks = [int(t) for t in rng.integers(0, QWEN_SHAPE["vocab"], prompt)]
        out = {}
        for fused in (True, False):
            dec = QwenDecoder(eng, path, ctx, fused_step=fused)
            weight_bytes = sum(int(v.numel()) for lay in dec.layers for k, v in lay.items()
                               if k in ("qkv", "o", "gu", "down")) + int(dec._head.numel())
            out[fused] = _qwen_decode_times(eng, stream, dec, toks, steps)
            dec.close()
        ms, graph_ms, lpt = out[True]
        ms2, graph_ms2, lpt2 = out[False]
        tps, graph_tps = steps / (ms / 1e3), steps / (graph_ms / 1e3)
        graph_gbs = weight_bytes * graph_tps / 1e9
        res = {"metric": "qwen2 decode step (QwenDecoder, whole-token step kernel: greedy steps recorded as one "
                         "CUDA graph, replayed)",
               "value": round(graph_tps, 1), "unit": "tokens/s", "ms_per_token": round(graph_ms / steps, 4),
               "steps": steps, "context_tokens": f"{prompt + 1}..{prompt + steps}",
               "eager": {"value": round(tps, 1), "unit": "tokens/s", "ms_per_token": round(ms / steps, 4),
                         "library_launches_per_token": round(lpt, 1),
                         "note": "forward_token (one step launch) + project_next (per-op head, torch argmax) "
                                 "from Python, argmax read back every step"},
               "per_op": {"value": round(steps / (graph_ms2 / 1e3), 1), "unit": "tokens/s",
                          "ms_per_token": round(graph_ms2 / steps, 4),
                          "library_launches_per_token": round(lpt2, 1),
                          "eager_value": round(steps / (ms2 / 1e3), 1),
                          "note": "te_matvec_gguf_fused + te_attention_decode + te_matvec_gguf, five launches "
                                  "per layer, recorded as one CUDA graph"},
               "model": "synthetic Qwen2.5-0.5B shape: 24 layers, H14/Hkv2/hd64, hidden 896, FFN 4864, "
                        "vocab 151936, Q4_0 projections, Q8_0 embedding/lm_head",
               "weight_bytes_per_token": weight_bytes,
               "roofline": {"bound": "hbm", "achieved": round(graph_gbs, 1), "peak": hbm_peak, "unit": "GB/s",
                            "frac": round(graph_gbs / hbm_peak, 4), "peak_source": f"{peak_src} (burst copy)",
                            "per_op_achieved": round(weight_bytes * steps / (graph_ms2 / 1e3) / 1e9, 1),
                            "note": "weight bytes read once per token over the graph-replay time"},
               "library_launches_per_token": 1.0}
        if not args.no_cpu:
            from oracle import oracle as O
            if O.ref_qwen_available():
                ref = O.RefQwen(path, ctx)
                for p_, t in enumerate(toks):
                    ref.forward(t, p_)
                _, rt = ref.project()
                n, t0 = 0, time.perf_counter()
                while time.perf_counter() - t0 < 3.0 and prompt + n < ctx:
                    ref.forward(rt, prompt + n)
                    _, rt = ref.project()
                    n += 1
                dt = time.perf_counter() - t0
                ref.close()
                res["cpu_baseline"] = {"value": round(n / dt, 2), "unit": "tokens/s", "kind": "reference",
                                       "cores": O.host_cores(),
                                       "sample": f"{n} tokens of te_qwen_forward_token + te_qwen_project_next "
                                                 f"(its CPU path, pthread matvec row split) in {dt:.1f} s"}
        return res
    finally:
        shutil.rmtree(tmp, ignore_errors=True)


QWEN_PREFILL_SHAPE = dict(layers=28, hidden=1536, heads=12, kv_heads=2, ffn=8960, vocab=151936, context=1024)


def run_qwen_prefill(eng, stream, args):
    """QwenDecoder.prefill_prompt on a synthetic model of Qwen2.5-1.5B's shape (28 layers, hidden 1536,
    12 heads of 128 over 2 KV heads, FFN 8960, vocabulary 151 936; Q4_0 projections, Q8_0 embedding and
    lm_head), a 512-token prompt: prompt tokens/s, device time on the engine's stream (the call's fused
    projections of 8 tokens per launch and one attention prefill per layer).  Beside it, the reference's
    CPU forward pass on the same file, token by token (a bounded sample)."""
    import tempfile
    import shutil
    import torch
    sys.path.insert(0, str(ROOT / "tests" / "golden"))
    from gguf_synth import GGML_Q4_0, write_qwen2
    from tinymetalagent_b200.qwen import QwenDecoder

    tmp = Path(tempfile.mkdtemp(prefix="qwen_prefill_bench_"))
    try:
        path = tmp / "qwen2_1p5b_shape.gguf"
        write_qwen2(path, quant_attn=GGML_Q4_0, quant_ffn=GGML_Q4_0, seed=4, **QWEN_PREFILL_SHAPE)
        T = 512
        dec = QwenDecoder(eng, path, T + 8, fused_step=False)
        prompt = [int(t) for t in np.random.default_rng(10).integers(0, QWEN_PREFILL_SHAPE["vocab"], T)]
        dec.prefill_prompt(prompt)  # warm
        dec.project_next()
        times = []
        for _ in range(3):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            torch.cuda.synchronize()
            e0.record(stream)
            dec.prefill_prompt(prompt, position=0)
            e1.record(stream)
            e1.synchronize()
            times.append(e0.elapsed_time(e1))
        launches0 = eng.launch_count
        dec.prefill_prompt(prompt, position=0)
        launches = eng.launch_count - launches0
        dec.close()
        ms = min(times)
        res = {"metric": "qwen2 prompt prefill (QwenDecoder.prefill_prompt)", "value": round(T / (ms / 1e3), 1),
               "unit": "prompt tokens/s", "ms_per_prompt": round(ms, 3), "prompt_tokens": T,
               "model": "synthetic Qwen2.5-1.5B shape: 28 layers, H12/Hkv2/hd128, hidden 1536, FFN 8960, "
                        "vocab 151936, Q4_0 projections, Q8_0 embedding/lm_head",
               "library_launches": int(launches), "timing": "best of 3 calls, CUDA events"}
        if not args.no_cpu:
            from oracle import oracle as O
            if O.ref_qwen_available():
                ref = O.RefQwen(path, T + 8)
                n, t0 = 0, time.perf_counter()
                while time.perf_counter() - t0 < 3.0 and n < T:
                    ref.forward(prompt[n], n)
                    n += 1
                dt = time.perf_counter() - t0
                ref.close()
                res["cpu_baseline"] = {"value": round(n / dt, 2), "unit": "prompt tokens/s", "kind": "reference",
                                       "cores": O.host_cores(),
                                       "sample": f"the first {n} prompt tokens through te_qwen_forward_token "
                                                 f"(its CPU path) in {dt:.1f} s"}
        return res
    finally:
        shutil.rmtree(tmp, ignore_errors=True)


def cpu_sample_7b(n: int, budget_s: float):
    """Bounded sample of the reference CPU attention on 7B-shaped layer calls
    (H28/Hkv4/hd128, n cached tokens, N(0,1) f16 cache) on all host threads."""
    from oracle import oracle as O
    kind = "reference" if O.ref_available() else "port"
    threads = O.host_cores()
    cd = CpuDecode(kind, threads, n_layers=min(L7, threads), n=n, heads=H7, kv_heads=KV7, scale=1.0,
                   shared_kv=n > 16384)
    gbs, calls, dt = cd.sample(budget_s)
    cd.close()
    return {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": kind,
            "sample": f"{calls} layer calls (N={n}, H28/Hkv4) in {dt:.1f} s on {threads} threads"}


def run_ragged7b(eng, stream, hbm_peak, peak_src, args, world, rank):
    """Qwen2.5-7B-shaped batched decode -- 28 layers,
    H28/Hkv4/hd128, 64 independent sequences of seeded uniform-random length in
    [256, 8192], f16 KV N(0,1).  Sequences are sharded across ranks (longest
    first onto the least-loaded rank); each rank runs one te_attention_decode
    per step over all its sequences and layers (RoPE + append + stream-K split
    decode), captured in a CUDA graph.  Strong scaling: 64 sequences in total."""
    import torch
    import torch.distributed as dist

    from tinymetalagent_b200 import TE_ATTN_ADVANCE, TE_ATTN_INPUT_F16, TE_ATTN_NO_ROPE
    from tinymetalagent_b200.dist import shard_sequences
    lens = np.random.default_rng(7).integers(256, 8193, size=64)
    mine = shard_sequences(lens.tolist(), world)[rank]
    steps = args.cfg_steps
    n_my = len(mine)
    cap = int(lens[mine].max()) + steps + 1
    cache = eng.kv_cache(layers=L7, max_seqs=n_my, max_tokens_per_seq=cap, kv_heads=KV7, head_dim=HEAD_DIM,
                         rope_theta=THETA)
    g = torch.Generator(device="cuda").manual_seed(4000 + rank)
    with torch.cuda.stream(stream):
        blk_k = torch.randn((8192, KV7, HEAD_DIM), generator=g, device="cuda").half()
        blk_v = torch.randn((8192, KV7, HEAD_DIM), generator=g, device="cuda").half()
        q = torch.randn((L7, n_my, H7, HEAD_DIM), generator=g, device="cuda")
        kn = torch.randn((L7, n_my, KV7, HEAD_DIM), generator=g, device="cuda")
        vn = torch.randn((L7, n_my, KV7, HEAD_DIM), generator=g, device="cuda")
        out = torch.empty((L7, n_my, H7, HEAD_DIM), device="cuda")
    stream.synchronize()
    for j, sid in enumerate(mine):
        n = int(lens[sid])
        for layer in range(L7):
            off = (layer * 977 + int(sid) * 131) % (8192 - n + 1)  # a different window of the random block per layer
            flags = TE_ATTN_INPUT_F16 | TE_ATTN_NO_ROPE | (TE_ATTN_ADVANCE if layer == L7 - 1 else 0)
            cache.append_rope(layer, 1, j, blk_k[off:off + n], blk_v[off:off + n], n, flags)
        cache.reserve(j, n + steps + 1)
    eng.synchronize()
    slots = list(range(n_my))

    def rewind():
        for j, sid in enumerate(mine):
            cache.truncate(j, int(lens[sid]))

    def step():
        cache.decode(0, L7, slots, q, out, H7, k_new=kn, v_new=vn, flags=TE_ATTN_ADVANCE)

    for _ in range(3):
        step()
    eng.synchronize()
    rewind()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for _ in range(steps):
            step()
    rewind()
    with torch.cuda.stream(stream):
        graph.replay()  # warm
    stream.synchronize()

    def replay():
        with torch.cuda.stream(stream):
            graph.replay()

    ms = _time_steps(stream, replay, 1, world, dist)
    del graph
    bytes_rank = sum(step_bytes(int(lens[sid]) + i + 1, L7, H7, KV7) for sid in mine for i in range(steps))
    t = torch.tensor([float(bytes_rank)], device="cuda")
    if world > 1:
        dist.all_reduce(t)
    bytes_all = float(t.item())
    gbs = bytes_all / (ms / 1e3) / 1e9
    cache.close()
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu = cpu_sample_7b(int(np.median(lens)), args.cpu_seconds / 2)
    return {"metric": "batched decode tokens/s (BASELINE config 4)", "cpu_baseline": cpu, "value": round(64 * steps / (ms / 1e3), 1),
            "unit": "tokens/s", "scaling": "strong", "steps": steps, "ms_per_step": round(ms / steps, 4),
            "workload": "ragged7b: 64 sequences, lengths U[256, 8192] (seed 7), 28 layers, H28/Hkv4/hd128, "
                        "f16 KV N(0,1), one token appended per sequence and layer per step",
            "sequences_per_rank": n_my, "kv_gbs": round(gbs, 1),
            "roofline": {"bound": "hbm", "achieved": round(gbs / world, 1), "peak": hbm_peak, "unit": "GB/s",
                         "frac": round(gbs / world / hbm_peak, 4), "per": "GPU (max-over-ranks time)",
                         "peak_source": f"{peak_src} (burst copy)"}}


def run_long7b(eng, stream, hbm_peak, peak_src, args, world, rank):
    """one 32768-token sequence, 28 layers, H28/Hkv4/hd128,
    f16 KV N(0,1), RoPE theta 1e6.  The KV sequence is split across ranks
    (contiguous token ranges); per step every rank computes partial (acc, m, l)
    records over its range (the tail rank also appends the new token) and the
    records are merged by log-sum-exp: by default inside the same decode launch
    (--long-exchange fused: each finished group's record is stored into every
    rank's memory over NVLink, every rank merges its own output), or by an NCCL
    all-gather plus te_attention_merge_partials (nccl), or by the push kernel
    (p2p).  Strong scaling: one sequence in total."""
    import torch
    import torch.distributed as dist

    from tinymetalagent_b200 import TE_ATTN_ADVANCE, TE_ATTN_INPUT_F16, TE_ATTN_NO_ROPE
    from tinymetalagent_b200.dist import KVSplitDecoder, ShardSpec
    n_ctx = 32768
    steps = args.long_steps
    spec = ShardSpec.plan(rank, world, n_ctx)
    n_local = spec.end - spec.begin
    extra = steps + 8 if spec.is_tail else 0
    cache = eng.kv_cache(layers=L7, max_seqs=1, max_tokens_per_seq=n_local + extra, kv_heads=KV7, head_dim=HEAD_DIM,
                         max_position=n_ctx + steps + 16, rope_theta=THETA)
    cache.reset(0, spec.begin)
    g = torch.Generator(device="cuda").manual_seed(5000 + rank)
    for layer in range(L7):
        with torch.cuda.stream(stream):
            k = torch.randn((n_local, KV7, HEAD_DIM), generator=g, device="cuda").half()
            v = torch.randn((n_local, KV7, HEAD_DIM), generator=g, device="cuda").half()
        stream.synchronize()
        cache.append_rope(layer, 1, 0, k, v, n_local, TE_ATTN_INPUT_F16 | TE_ATTN_NO_ROPE |
                          (TE_ATTN_ADVANCE if layer == L7 - 1 else 0))
        del k, v
    if spec.is_tail:
        cache.reserve(0, n_local + extra)
    eng.synchronize()
    with torch.cuda.stream(stream):
        q = torch.randn((L7, 1, H7, HEAD_DIM), generator=g, device="cuda")
        kn = torch.randn((L7, 1, KV7, HEAD_DIM), generator=g, device="cuda")
        vn = torch.randn((L7, 1, KV7, HEAD_DIM), generator=g, device="cuda")
    stream.synchronize()
    exchange = args.long_exchange if world > 1 else "local"
    dec = KVSplitDecoder(spec, L7, H7, HEAD_DIM, cache=cache, engine=eng, device="cuda",
                         exchange="nccl" if exchange == "local" else exchange)

    def step():
        with torch.cuda.stream(stream):  # NCCL and the engine share the engine's stream
            dec.step(q, kn, vn)

    def rewind():  # back to n_ctx cached tokens (the tail rank drops what it appended)
        eng.synchronize()
        if spec.is_tail:
            cache.truncate(0, n_local)
        dec.length = n_ctx

    for _ in range(4):
        step()
    rewind()
    # The K steps (partial decode, NCCL all-gather, merge) are captured in one
    # CUDA graph on the engine's stream and replayed, as for config 2.
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for _ in range(steps):
            dec.step(q, kn, vn)
    rewind()
    with torch.cuda.stream(stream):
        graph.replay()  # warm
    rewind()

    def replay():
        with torch.cuda.stream(stream):
            graph.replay()

    ms = _time_steps(stream, replay, 1, world, dist)
    eng.synchronize()
    del graph
    if world > 1:
        dist.barrier()  # every rank's last step is done before the exchange areas go away
    dec.close()
    bytes_all = sum(step_bytes(n_ctx + i + 1, L7, H7, KV7) for i in range(steps))
    gbs = bytes_all / (ms / 1e3) / 1e9
    cache.close()
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu = cpu_sample_7b(n_ctx + 1, args.cpu_seconds / 2)
    return {"metric": "long-context decode tokens/s (BASELINE config 5)", "cpu_baseline": cpu, "value": round(steps / (ms / 1e3), 1),
            "unit": "tokens/s", "scaling": "strong", "steps": steps, "ms_per_step": round(ms / steps, 4),
            "workload": "long7b: one sequence of 32768 cached tokens, 28 layers, H28/Hkv4/hd128, f16 KV N(0,1), "
                        f"KV split over {world} rank(s), "
                        + {"local": "one rank: partial records merged by te_attention_merge_partials; ",
                           "p2p": "NVLink push of (acc, m, l) into the peers + LSE merge in one kernel per step; ",
                           "fused": "exchange fused into the decode launch (each finished (layer, kv head) group's "
                                    "record stored into every rank's memory over NVLink; every rank merges its own "
                                    "output); ",
                           "nccl": "NCCL all-gather of (acc, m, l) + LSE merge per step; "}[exchange]
                        + "steps captured in one CUDA graph",
            "exchange": exchange,
            "tokens_per_rank": n_local, "kv_gbs": round(gbs, 1),
            "roofline": {"bound": "hbm", "achieved": round(gbs / world, 1), "peak": hbm_peak, "unit": "GB/s",
                         "frac": round(gbs / world / hbm_peak, 4), "per": "GPU (max-over-ranks time)",
                         "peak_source": f"{peak_src} (burst copy)"}}


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=DECODE_STEPS)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--min-timed-ms", type=float, default=200.0,
                    help="config 2: timed K-step regions are repeated until they span this much device time")
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline sample")
    ap.add_argument("--chunk", type=int, default=0, help="split-K chunk tokens (multiple of 64; 0 = auto)")
    ap.add_argument("--no-prefill", action="store_true", help="skip the config-3 prefill measurement")
    ap.add_argument("--no-graph", action="store_true", help="time the decode steps as eager launches")
    ap.add_argument("--prefill-steps", type=int, default=10)
    ap.add_argument("--no-prefill-variants", action="store_true",
                    help="skip the exact-query and head_dim-64 prefill measurements")
    ap.add_argument("--no-configs", action="store_true", help="skip the config-4 / config-5 measurements")
    ap.add_argument("--only-configs", action="store_true", help="run only the config-4 / config-5 measurements")
    ap.add_argument("--no-gemv", action="store_true", help="skip the GGUF matrix-vector measurement")
    ap.add_argument("--no-qwen", action="store_true", help="skip the qwen2 decode-step measurement")
    ap.add_argument("--qwen-steps", type=int, default=64, help="decode steps timed for the qwen2 decode step")
    ap.add_argument("--no-qwen-prefill", action="store_true",
                    help="with --qwen-only: skip the prompt-prefill measurement")
    ap.add_argument("--qwen-only", action="store_true",
                    help="run only the qwen2 decode-step measurements (whole-token step kernel and per-op path)")
    ap.add_argument("--gemv-only", action="store_true",
                    help="run only the GGUF matrix-vector measurement (Q4_0: launches 1-23, Q8_0: 24-46)")
    ap.add_argument("--cfg-steps", type=int, default=16, help="decode steps timed for config 4")
    ap.add_argument("--long-steps", type=int, default=128, help="decode steps timed for config 5")
    ap.add_argument("--long-exchange", choices=["nccl", "p2p", "fused"], default="fused",
                    help="config 5 at N>1: NCCL all-gather + merge, the NVLink exchange kernel, or the exchange "
                         "fused into the decode launch")
    args = ap.parse_args()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_gpu(args)


if __name__ == "__main__":
    main()
